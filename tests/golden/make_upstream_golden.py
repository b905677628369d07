"""Generates tests/golden/generator_upstream.npz from the upstream torch GeneratorNSF of the reference
tree (knowledge/rvc_original/infer/module/models.py:403-514, ResBlock1 modules.py:227-322), run
here where the reference tree exists; the fixture is committed and travels, the reference does not.

The generator is the 40 kHz configuration with weight norm on the upsampling and resblock
convolutions, cond(g) and the noise convolutions; its source is replaced by
SourceModuleHnNSF(harmonic_num=8) (models.py:346-400; GeneratorNSF itself builds harmonic_num=0,
models.py:422-424) and the SineGen draws (torch.rand initial phases, torch.randn_like noise) by the
counter generator of oracle/generator_ref.py, so the oracle can rebuild every input.  It runs in
float64.  Stored: the forward waveform and, per parameter, the gradient's norm, element sum and 24
sampled entries (the parameters themselves are rebuilt from the seed).

  WUBU_REFERENCE=<reference tree> python tests/golden/make_upstream_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import generator_ref as G  # noqa: E402
from oracle.refpath import reference_root  # noqa: E402
from wuburvc_b200 import model  # noqa: E402

N_SAMPLES = 24
WSEED = 21
B, F = 1, 4


def config():
    # upstream's last activation is F.leaky_relu(x) with torch's default slope 0.01 (models.py:509)
    return model.config("40k", final_slope=0.01)


def inputs(cfg):
    T = F * model.hop(cfg)
    dim = cfg["harmonic_num"] + 1
    z = G.counter_normal(23, 1, B * 192 * F).reshape(B, 192, F)
    g = G.counter_normal(23, 2, B * 256).reshape(B, 256, 1)
    f0 = (G.counter_uniform_pair(23, 3, np.arange(B * F, dtype=np.uint64))[0] * 320 + 80).reshape(B, F)
    f0[0, 1] = 0.0  # one unvoiced frame
    dldy = G.counter_normal(23, 4, B * T).reshape(B, 1, T)
    noise = G.counter_normal(23, 5, B * T * dim).reshape(B, T, dim)
    rand_ini = G.counter_rand_ini(23, 6, dim)
    return z, f0, g, dldy, noise, rand_ini


def params(cfg):
    # non-zero biases so that every bias path is pinned too
    return G.init_params_ref(cfg, WSEED, bias_std=0.01)


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

    cfg = config()
    P = params(cfg)
    z, f0, g, dldy, noise, rand_ini = inputs(cfg)
    gen = up.GeneratorNSF(192, "1", [3, 7, 11], [[1, 3, 5]] * 3, list(cfg["upsample_rates"]), 512,
                          list(cfg["upsample_kernels"]), 256, cfg["sr"])
    gen.m_source = up.SourceModuleHnNSF(cfg["sr"], harmonic_num=cfg["harmonic_num"])
    gen = gen.double()
    names = [n for n, _ in gen.named_parameters()]
    assert {"dec." + n for n in names} == set(P), set(P) ^ {"dec." + n for n in names}
    with torch.no_grad():
        for n, p in gen.named_parameters():
            p.copy_(torch.tensor(np.asarray(P["dec." + n], np.float64)).reshape(p.shape))
    dim = cfg["harmonic_num"] + 1
    orig_rand, orig_randn_like = torch.rand, torch.randn_like
    torch.rand = lambda *a, **k: torch.tensor(rand_ini, dtype=torch.float64).view(1, 1, dim).clone()
    torch.randn_like = lambda x, *a, **k: torch.tensor(noise, dtype=x.dtype)
    try:
        audio = gen(torch.tensor(z), torch.tensor(f0), g=torch.tensor(g))
    finally:
        torch.rand, torch.randn_like = orig_rand, orig_randn_like
    audio.backward(torch.tensor(dldy))
    out = {"audio": audio.detach().numpy()[0, 0].astype(np.float64)}
    gnames, gnorm, gsum, offs, idxs, gval = [], [], [], [0], [], []
    for n, p in gen.named_parameters():
        gr = p.grad.detach().numpy().reshape(-1).astype(np.float64)
        idx = sample_idx("dec." + n, gr.size)
        gnames.append("dec." + n)
        gnorm.append(np.linalg.norm(gr))
        gsum.append(gr.sum())
        idxs.append(idx)
        gval.append(gr[idx])
        offs.append(offs[-1] + idx.size)
    out.update(names=np.array(gnames), gnorm=np.array(gnorm), gsum=np.array(gsum), offs=np.array(offs),
               idx=np.concatenate(idxs).astype(np.int64), gval=np.concatenate(gval))
    path = os.path.join(HERE, "generator_upstream.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(gnames), "gradients")


if __name__ == "__main__":
    main()
