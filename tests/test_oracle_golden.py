"""Pins the fp64 oracle (oracle/generator_ref.py) against golden vectors produced by the
reference itself (tests/golden/make_golden.py): the reference C trainer's decoder forward,
backward and AdamW, and the upstream torch SineGen / SourceModuleHnNSF."""
import os

import numpy as np
import pytest
import torch

from oracle import generator_ref as G
from wuburvc_b200 import model

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300)


def load_decoder(tag):
    d = np.load(os.path.join(GOLD, f"decoder_{tag}.npz"))
    names = [str(n) for n in d["names"]]
    return d, names


def decoder_case(tag):
    cfg = model.decoder_only(tag)
    d, names = load_decoder(tag)
    F = int(d["F"])
    P = G.init_params_ref(cfg, int(d["wseed"]))
    T = F * model.hop(cfg)
    z = G.counter_normal(11, 1, 192 * F).reshape(1, 192, F).astype(np.float32)
    dldy = G.counter_normal(11, 2, T).reshape(1, 1, T).astype(np.float32)
    return cfg, d, names, P, z, dldy


@pytest.mark.parametrize("tag", ["40k", "32k"])
def test_oracle_matches_reference_decoder(tag):
    cfg, d, names, P, z, dldy = decoder_case(tag)
    audio, grads = G.train_grads(P, cfg, z, None, None, None, None, dldy)
    # forward: reference fp32 vs oracle fp64
    assert rel(audio[0, 0], d["audio"]) < 1e-5
    # the registry is the same set of tensors
    assert set(names) == set(P.keys())
    gnorm = d["gnorm"]
    errs = []
    for i, n in enumerate(names):
        g = grads[n].reshape(-1)
        errs.append(abs(np.linalg.norm(g) - gnorm[i]) / max(gnorm[i], 1e-300))
        idx = d["idx"][d["offs"][i]:d["offs"][i + 1]]
        gv = d["gval"][d["offs"][i]:d["offs"][i + 1]]
        # sampled entries: fp32 reference vs fp64 oracle, kink flips allowed at a tiny rate
        close = np.abs(g[idx] - gv) <= 2e-3 * np.abs(gv).max() + 1e-12
        assert close.mean() > 0.9, n
    # gradient norms per tensor: the reference's own fp32 noise floor is ~1e-3 on worst tensors
    assert np.median(errs) < 1e-4
    assert max(errs) < 1e-2


@pytest.mark.parametrize("tag", ["40k"])
def test_oracle_adamw_matches_reference(tag):
    """AdamW restatement (bias correction applied twice) on the reference's own gradients."""
    cfg, d, names, P, z, dldy = decoder_case(tag)
    # reconstruct the full reference gradient is not stored; check the update formula on the
    # sampled entries: p1 = p0 - (lr_eff*(m/b1c)/(sqrt(v/b2c)+eps) + lr*wd*p0) at t=1
    for i, n in enumerate(names):
        sl = slice(d["offs"][i], d["offs"][i + 1])
        idx, gv, pv = d["idx"][sl], d["gval"][sl], d["pval"][sl]
        p0 = P[n].reshape(-1)[idx].astype(np.float32).copy()
        m = np.zeros_like(p0)
        v = np.zeros_like(p0)
        G.adamw_step(p0, gv, m, v, 1, 1e-3, 0.9, 0.999, 1e-8, 1e-4)
        np.testing.assert_allclose(p0, pv, rtol=1e-6, atol=1e-9)


def test_oracle_sine_source_matches_upstream():
    d = np.load(os.path.join(GOLD, "sinegen.npz"))
    cfg = model.config("40k")
    f0 = d["f0"].astype(np.float64)
    B, F = f0.shape
    T = F * 400
    noise = G.counter_normal(int(d["noise_seed"]), 2, B * T * 9).reshape(B, T, 9).astype(np.float32)
    t = lambda a: torch.tensor(np.asarray(a, np.float64))
    har = G.sine_source(t(f0), cfg, t(d["lin_w"]), t(np.array([d["lin_b"]])), t(noise), t(d["rand_ini"]))
    # upstream computes the phase in fp32 (rad cumsum, 9x harmonic multiply): ~1e-5 phase error
    assert rel(har[:, 0, :].numpy(), d["har"]) < 2e-4


def test_counter_generator_is_standard_normal():
    x = G.counter_normal(0, 1, 200000)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    r = G.counter_rand_ini(0, 1, 9)
    assert r[0] == 0 and np.all((r >= 0) & (r < 1))


def test_oracle_matches_upstream_generator_nsf():
    """The full NSF generator of the oracle (cond(g), noise convs, weight norm (g, v), 9-harmonic
    source + l_linear, ResBlock1 stacks) against the upstream torch GeneratorNSF run in float64
    (tests/golden/make_upstream_golden.py): the forward waveform and every one of the 243 parameter
    gradients (norm, element sum, sampled entries).  Upstream forms the source's per-frame phase
    carry in float32 (models.py:313, rad[..., -1:].float()), the oracle in float64: that ~1e-7 phase
    difference leaves the forward within ~1e-8 and the gradients of the tensors fed by the source
    (noise convs, l_linear) within ~5e-7; the others agree to ~1e-9."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("mk", os.path.join(GOLD, "make_upstream_golden.py"))
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    d = np.load(os.path.join(GOLD, "generator_upstream.npz"))
    cfg = mk.config()
    P = mk.params(cfg)
    z, f0, g, dldy, noise, rand_ini = mk.inputs(cfg)
    audio, grads = G.train_grads(P, cfg, z, f0, g, noise, rand_ini, dldy)
    assert rel(audio[0, 0], d["audio"]) < 1e-7
    names = [str(n) for n in d["names"]]
    assert set(names) == set(grads) and len(names) == 243
    errs = []
    for i, n in enumerate(names):
        gr = grads[n].reshape(-1)
        gn = d["gnorm"][i]
        sl = slice(d["offs"][i], d["offs"][i + 1])
        e = max(abs(np.linalg.norm(gr) - gn) / gn, np.abs(gr[d["idx"][sl]] - d["gval"][sl]).max() / gn,
                abs(gr.sum() - d["gsum"][i]) / (gn * np.sqrt(gr.size)))
        assert e < 2e-6, (n, e)
        errs.append(e)
    assert np.median(errs) < 1e-8
