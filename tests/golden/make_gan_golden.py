"""Generates tests/golden/gan_upstream.npz from the upstream RVC discriminator and losses of the
reference tree (knowledge/rvc_original/infer/module/models.py:928-1094, train/losses.py:4-40), run
here where the reference tree exists; the fixture is committed and travels, the reference does not.

One GAN step in the order of train/train.py:500-525, in float64:
  1. MultiPeriodDiscriminator on (y, y_hat detached), discriminator_loss, backward;
  2. torch.optim.AdamW on the discriminator (lr 1e-4, betas (0.8, 0.99), eps 1e-9 as the 40k
     training config; torch's default weight decay 0.01), t = 1;
  3. the updated discriminator on (y, y_hat), generator_loss + feature_loss, backward to y_hat.
Stored: the step-1 logits (real discriminators then generated, each flattened), the three losses,
dL/dy_hat, and per parameter the step-1 gradient's norm, sum and 24 sampled entries with the
sampled parameters after AdamW (the parameters themselves are rebuilt from the seed by
oracle/gan_ref.init_params).  B = 2, T = 2400: not a multiple of 7, 11 or 17, so the reflect
padding of those periods is pinned too.

  WUBU_REFERENCE=<reference tree> python tests/golden/make_gan_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import gan_ref as D  # noqa: E402
from oracle import generator_ref as G  # noqa: E402
from oracle.refpath import reference_root  # noqa: E402

B, T = 2, 2400
SEED = 3
N_SAMPLES = 24
ADAM = dict(lr=1e-4, betas=(0.8, 0.99), eps=1e-9, weight_decay=0.01)


def inputs():
    y = 0.3 * G.counter_normal(41, 1, B * T).reshape(B, T)
    y_hat = 0.5 * y + 0.2 * G.counter_normal(41, 2, B * T).reshape(B, T)
    return y, y_hat


def sample_idx(name, n):
    u1, _ = G.counter_uniform_pair(5, G._name_stream(name), np.arange(N_SAMPLES, dtype=np.uint64))
    return np.unique(np.minimum((u1 * n).astype(np.int64), n - 1))


def main():
    ref = reference_root()
    if ref is None:
        raise SystemExit("reference tree not found: set WUBU_REFERENCE")
    sys.path.insert(0, os.path.join(ref, "knowledge", "rvc_original"))
    import torch
    from infer.module import models as up
    from train import losses as upl

    P = D.init_params(D.PERIODS_V1, SEED)
    net = up.MultiPeriodDiscriminator().double()
    sd = net.state_dict()
    assert list(sd) == list(P), set(sd) ^ set(P)
    with torch.no_grad():
        for n, p in net.named_parameters():
            p.copy_(torch.tensor(np.asarray(P[n], np.float64)).reshape(p.shape))
    y, y_hat = inputs()
    yt = torch.tensor(y)[:, None]
    yg = torch.tensor(y_hat)[:, None]

    # 1. discriminator step
    dr, dg, _, _ = net(yt, yg.detach())
    loss_d, _, _ = upl.discriminator_loss(dr, dg)
    opt = torch.optim.AdamW(net.parameters(), **ADAM)
    opt.zero_grad()
    loss_d.backward()
    logits = np.concatenate([a.detach().numpy().reshape(-1) for a in dr] + [a.detach().numpy().reshape(-1) for a in dg])
    names = [n for n, _ in net.named_parameters()]
    grads = {n: p.grad.detach().numpy().reshape(-1).copy() for n, p in net.named_parameters()}
    opt.step()
    after = {n: p.detach().numpy().reshape(-1).copy() for n, p in net.named_parameters()}

    # 2. generator side through the updated discriminator
    yg = yg.clone().requires_grad_(True)
    dr, dg, fr, fg = net(yt, yg)
    loss_fm = upl.feature_loss(fr, fg)
    loss_gen, _ = upl.generator_loss(dg)
    net.zero_grad()
    (loss_gen + loss_fm).backward()

    gnorm, gsum, offs, idxs, gval, pval = [], [], [0], [], [], []
    for n in names:
        g = grads[n]
        ix = sample_idx(n, g.size)
        gnorm.append(np.linalg.norm(g))
        gsum.append(g.sum())
        idxs.append(ix)
        gval.append(g[ix])
        pval.append(after[n][ix])
        offs.append(offs[-1] + ix.size)
    out = os.path.join(HERE, "gan_upstream.npz")
    np.savez_compressed(out, B=B, T=T, seed=SEED, y=y, y_hat=y_hat, logits=logits,
                        loss_d=float(loss_d), loss_gen=float(loss_gen), loss_fm=float(loss_fm),
                        dldy_hat=yg.grad.numpy()[:, 0].copy(), names=np.array(names),
                        gnorm=np.array(gnorm), gsum=np.array(gsum), offs=np.array(offs),
                        idx=np.concatenate(idxs), gval=np.concatenate(gval), pval=np.concatenate(pval),
                        lr=ADAM["lr"], betas=np.array(ADAM["betas"]), eps=ADAM["eps"], wd=ADAM["weight_decay"])
    print("wrote", out, "loss_d", float(loss_d), "loss_gen", float(loss_gen), "loss_fm", float(loss_fm))


if __name__ == "__main__":
    main()
