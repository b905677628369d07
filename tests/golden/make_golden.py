"""Generates the golden fixtures in tests/golden/ from the reference itself (run here, where
the reference tree exists; the fixtures are committed and travel, the reference does not).

  decoder_40k.npz  the reference C trainer (src/wubu_train.c, built by oracle/Makefile into
                   oracle/_ref/libwubu_ref.so): decoder forward, backward with an injected dL/dy,
                   and one AdamW step, 40 kHz, F=8.  Stored: audio, per-tensor gradient norm / sum /
                   sampled entries, sampled parameters after AdamW.
  decoder_32k.npz  same for the 32 kHz upsampling config (F=5).
  sinegen.npz      the upstream SineGen / SourceModuleHnNSF
                   (knowledge/rvc_original/infer/module/models.py:267-400) with harmonic_num=8,
                   its torch.rand / torch.randn_like draws replaced by the counter generator of
                   oracle/generator_ref.py so the result is reproducible.

Inputs and weights come from the counter generator (seeded), so every consumer can rebuild them.

  python tests/golden/make_golden.py      (needs the reference tree -- WUBU_REFERENCE -- and oracle/_ref)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import generator_ref as G  # noqa: E402
from oracle import ref_oracle  # noqa: E402
from wuburvc_b200 import model  # noqa: E402

from oracle.refpath import reference_root  # noqa: E402

REF = reference_root()
N_SAMPLES = 24
ADAM = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, wd=1e-4)


def sample_idx(name, n):
    u1, _ = G.counter_uniform_pair(5, G._name_stream(name), np.arange(N_SAMPLES, dtype=np.uint64))
    return np.unique(np.minimum((u1 * n).astype(np.int64), n - 1))


def decoder_inputs(cfg, F, seed=11):
    T = F * model.hop(cfg)
    z = G.counter_normal(seed, 1, 192 * F).reshape(1, 192, F).astype(np.float32)
    dldy = G.counter_normal(seed, 2, T).reshape(1, 1, T).astype(np.float32)
    return z, dldy


def decoder_fixture(tag, cfg, F, wseed=1):
    P = G.init_params_ref(cfg, wseed)
    z, dldy = decoder_inputs(cfg, F)
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"], lr=ADAM["lr"],
                                betas=ADAM["betas"], eps=ADAM["eps"], wd=ADAM["wd"])
    audio = ref.forward(z[0])
    ref.backward(dldy[0, 0])
    grads = ref.grads()
    ref.adamw()
    after = ref.params()
    gnorm, gsum, offs, idxs, gval, pval = [], [], [0], [], [], []
    for n in ref.names:
        g = grads[n].astype(np.float64)
        idx = sample_idx(n, g.size)
        gnorm.append(np.linalg.norm(g))
        gsum.append(g.sum())
        idxs.append(idx)
        gval.append(grads[n][idx])
        pval.append(after[n][idx])
        offs.append(offs[-1] + idx.size)
    out = {"audio": audio, "F": np.int64(F), "wseed": np.int64(wseed), "names": np.array(ref.names),
           "gnorm": np.array(gnorm), "gsum": np.array(gsum), "offs": np.array(offs, dtype=np.int64),
           "idx": np.concatenate(idxs).astype(np.int64), "gval": np.concatenate(gval).astype(np.float32),
           "pval": np.concatenate(pval).astype(np.float32)}
    path = os.path.join(HERE, f"decoder_{tag}.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, "audio", audio.shape)


def sinegen_fixture():
    sys.path.insert(0, os.path.join(REF, "knowledge", "rvc_original"))
    import torch
    from infer.module import models as up

    B, F, upp, dim, sr = 2, 8, 400, 9, 40000
    T = F * upp
    f0 = G.counter_uniform_pair(3, 1, np.arange(B * F, dtype=np.uint64))[0].reshape(B, F) * 320 + 80
    f0[:, 2] = 0.0
    f0[1, 5:7] = 0.0
    f0 = f0.astype(np.float32)
    noise = G.counter_normal(3, 2, B * T * dim).reshape(B, T, dim).astype(np.float32)
    rand_ini = G.counter_rand_ini(3, 4, dim).astype(np.float32)
    lin_w = ((2 * G.counter_uniform_pair(3, 5, np.arange(dim, dtype=np.uint64))[0] - 1) / 3).astype(np.float32)
    lin_b = np.float32(0.05)

    src = up.SourceModuleHnNSF(sr, harmonic_num=dim - 1, is_half=False)
    with torch.no_grad():
        src.l_linear.weight.copy_(torch.tensor(lin_w).view(1, dim))
        src.l_linear.bias.fill_(float(lin_b))
    orig_rand, orig_randn_like = torch.rand, torch.randn_like
    torch.rand = lambda *a, **k: torch.tensor(rand_ini).view(1, 1, dim).clone()
    torch.randn_like = lambda x, *a, **k: torch.tensor(noise, dtype=x.dtype)
    try:
        sine, uv, _ = src.l_sin_gen(torch.tensor(f0), upp)
        har, _, _ = src(torch.tensor(f0), upp)
    finally:
        torch.rand, torch.randn_like = orig_rand, orig_randn_like
    path = os.path.join(HERE, "sinegen.npz")
    np.savez_compressed(path, f0=f0, rand_ini=rand_ini, lin_w=lin_w, lin_b=lin_b, noise_seed=np.int64(3),
                        sine=sine.detach().numpy()[:, ::5, :].astype(np.float32),
                        har=har.detach().numpy()[..., 0].astype(np.float32))
    print("wrote", path)


if __name__ == "__main__":
    if REF is None:
        raise SystemExit("reference tree not found: set WUBU_REFERENCE")
    if not ref_oracle.available():
        raise SystemExit("build oracle/_ref first: make -C oracle")
    decoder_fixture("40k", model.decoder_only("40k"), F=8)
    decoder_fixture("32k", model.decoder_only("32k"), F=5)
    sinegen_fixture()
