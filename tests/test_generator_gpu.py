"""Parity of the CUDA training step (through the C ABI) with the reference and the oracle.

Gates (the target tolerances for bf16 GEMM operands with fp32 accumulation):
  forward waveform      rel-L2 <= 2e-3
  every parameter grad  rel-L2 <= 1e-2
Compared against
  * the reference C trainer's own outputs (tests/golden/decoder_*.npz) for the decoder it trains;
  * the fp64 oracle (oracle/generator_ref.py) for the full NSF generator (source, cond, noise
    convs, weight norm, Snake), which the reference C trainer does not implement.
"""
import os

import numpy as np
import pytest
import torch

from oracle import generator_ref as G
from oracle import ref_oracle
from wuburvc_b200 import Generator, flatten, model, unflatten

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FWD_TOL = 2e-3
GRAD_TOL = 1e-2


def rel(a, b):
    a, b = np.asarray(a, np.float64).reshape(-1), np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def nsf_inputs(cfg, B, F, seed=5):
    T = F * model.hop(cfg)
    z = G.counter_normal(seed, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    g = G.counter_normal(seed, 2, B * 256).reshape(B, 256).astype(np.float32)
    f0 = (G.counter_uniform_pair(seed, 3, np.arange(B * F, dtype=np.uint64))[0] * 320 + 80).reshape(B, F)
    f0[G.counter_uniform_pair(seed, 4, np.arange(B * F, dtype=np.uint64))[0].reshape(B, F) < 0.2] = 0
    f0 = f0.astype(np.float32)
    dldy = G.counter_normal(seed, 6, B * T).reshape(B, T).astype(np.float32)
    return z, f0, g, dldy


def grad_report(cfg, gpu_flat, ref_named):
    named = unflatten(cfg, gpu_flat)
    errs = {}
    for n, r in ref_named.items():
        if np.linalg.norm(r) == 0:
            continue
        errs[n] = rel(named[n].reshape(-1), np.asarray(r).reshape(-1))
    return errs


# ------------------------------------------------------------------------------------------
# decoder (the reference C trainer's model) against the reference's own golden outputs
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("tag", ["40k", "32k"])
def test_decoder_matches_reference_c_trainer(tag):
    cfg = model.decoder_only(tag)
    d = np.load(os.path.join(GOLD, f"decoder_{tag}.npz"))
    names = [str(n) for n in d["names"]]
    F = int(d["F"])
    P = G.init_params_ref(cfg, int(d["wseed"]))
    T = F * model.hop(cfg)
    z = G.counter_normal(11, 1, 192 * F).reshape(1, 192, F).astype(np.float32)
    dldy = G.counter_normal(11, 2, T).reshape(1, T).astype(np.float32)
    gen = Generator(cfg, 1, F, lr=1e-3, weight_decay=1e-4)
    p0 = flatten(cfg, P)
    gen.set_params(p0)
    gen.upload(z, dldy=dldy)
    audio = gen.forward()
    assert rel(audio[0], d["audio"]) <= FWD_TOL
    gen.backward()
    grads = unflatten(cfg, gen.get_grads())
    worst = 0.0
    for i, n in enumerate(names):
        g = grads[n].reshape(-1).astype(np.float64)
        gn = d["gnorm"][i]
        e = abs(np.linalg.norm(g) - gn) / gn
        worst = max(worst, e)
        # direction, not only the norm: the reference's sampled entries and its element sum.  A
        # gradient within rel-L2 GRAD_TOL differs from the reference by at most GRAD_TOL*||g|| in
        # every entry and by at most GRAD_TOL*||g||*sqrt(n) in the sum (Cauchy-Schwarz)
        sl = slice(d["offs"][i], d["offs"][i + 1])
        idx, gv = d["idx"][sl], d["gval"][sl].astype(np.float64)
        assert np.abs(g[idx] - gv).max() <= GRAD_TOL * gn, n
        assert abs(g.sum() - d["gsum"][i]) <= GRAD_TOL * gn * np.sqrt(g.size), n
    assert worst <= GRAD_TOL
    # every tensor by rel-L2 against the reference trainer run live (it travels, built in oracle/_ref)
    if ref_oracle.available():
        ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
        ref.forward(z[0])
        ref.backward(dldy[0])
        live = ref.grads()
        ref.close()
        bad = {n: rel(grads[n], live[n]) for n in names if rel(grads[n], live[n]) > GRAD_TOL}
        assert not bad, bad
    # one AdamW step on the device against the AdamW restatement (itself pinned to the
    # reference's wubu_adamw_step by test_oracle_adamw_matches_reference) on the same gradients
    gflat = gen.get_grads()
    gen.adamw()
    got = gen.get_params()
    exp = p0.copy()
    G.adamw_step(exp, gflat, np.zeros_like(exp), np.zeros_like(exp), 1, 1e-3, 0.9, 0.999, 1e-8, 1e-4)
    np.testing.assert_allclose(got, exp, rtol=2e-5, atol=1e-9)
    gen.close()


# ------------------------------------------------------------------------------------------
# full NSF generator against the fp64 oracle
# ------------------------------------------------------------------------------------------
def run_nsf_case(cfg, B, F, device_noise=False, wseed=2, stream=9):
    z, f0, g, dldy = nsf_inputs(cfg, B, F)
    T = F * model.hop(cfg)
    dim = cfg["harmonic_num"] + 1
    noise = G.counter_normal(0, stream, B * T * dim).reshape(B, T, dim)
    rand_ini = G.counter_rand_ini(0, stream, dim)
    P = G.init_params_ref(cfg, wseed)
    gen = Generator(cfg, B, F, seed=0)
    gen.set_params(flatten(cfg, P))
    gen.upload(z, f0, g, None if device_noise else noise.astype(np.float32), dldy)
    audio = gen.forward(noise_stream=stream)
    gen.backward()
    gflat = gen.get_grads()
    gen.close()
    a64, g64 = G.train_grads(P, cfg, z, f0, g[:, :, None], noise, rand_ini, dldy[:, None, :])
    return audio, a64[:, 0, :], grad_report(cfg, gflat, g64)


@pytest.mark.parametrize("device_noise", [False, True])
def test_nsf_generator_40k_matches_oracle(device_noise):
    cfg = model.config("40k")
    audio, a64, errs = run_nsf_case(cfg, B=2, F=8, device_noise=device_noise)
    assert rel(audio, a64) <= FWD_TOL
    bad = {n: e for n, e in errs.items() if e > GRAD_TOL}
    assert not bad, sorted(bad.items(), key=lambda x: -x[1])[:8]


def test_snake_generator_48k_matches_oracle():
    cfg = model.config("48k_snake")
    audio, a64, errs = run_nsf_case(cfg, B=1, F=4)
    assert rel(audio, a64) <= FWD_TOL
    bad = {n: e for n, e in errs.items() if e > GRAD_TOL}
    assert not bad, sorted(bad.items(), key=lambda x: -x[1])[:8]


def test_train_step_graph_equals_separate_calls():
    cfg = model.config("40k")
    B, F = 2, 4
    z, f0, g, dldy = nsf_inputs(cfg, B, F)
    P = flatten(cfg, G.init_params_ref(cfg, 3))
    a = Generator(cfg, B, F)
    a.set_params(P)
    a.upload(z, f0, g, None, dldy)
    a.forward(noise_stream=4)
    a.backward()
    a.adamw()
    pa = a.get_params()
    b = Generator(cfg, B, F)
    b.set_params(P)
    out = np.empty((B, b.T), np.float32)
    b.train_step(z, f0, g, None, dldy, noise_stream=4, audio_out=out)
    pb = b.get_params()
    assert rel(pb, pa) < 1e-6
    assert np.isfinite(out).all()
    a.close()
    b.close()


def test_training_reduces_mse():
    """Three AdamW steps on an MSE target must reduce the loss (src/test_train_cuda.c:130-143)."""
    cfg = model.decoder_only("40k")
    B, F = 2, 8
    gen = Generator(cfg, B, F, lr=1e-3)
    gen.set_params(flatten(cfg, G.init_params_ref(cfg, 4)))
    z = G.counter_normal(1, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    target = (0.3 * G.counter_normal(1, 2, B * gen.T)).reshape(B, gen.T).astype(np.float32)
    losses = []
    for it in range(4):
        gen.upload(z, dldy=np.zeros((B, gen.T), np.float32))
        y = gen.forward()
        losses.append(float(np.mean((y - target) ** 2)))
        gen.upload(z, dldy=(2 * (y - target) / y.size).astype(np.float32))
        gen.backward()
        gen.adamw()
    assert losses[-1] < losses[0]
    gen.close()


def test_operand_beyond_fp16_range_falls_back_to_bf16_pairs():
    """Forward GEMM operands are fp16 hi + lo/2048 pairs, which cannot hold 65504 or more.  When an
    operand reaches it the step's update is skipped on the device, the context switches for good to
    bf16 hi + lo pairs and the call recomputes the step: the caller sees a normal result, and the
    update is applied exactly once (same parameters as a context that was already on bf16 pairs).
    The asynchronous step reports the skip once through sync and leaves the parameters unchanged."""
    cfg = model.decoder_only("40k")
    B, F = 1, 4
    P = flatten(cfg, G.init_params_ref(cfg, 1))
    z = G.counter_normal(2, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    bad = z.copy()
    bad[0, 5, 2] = 1e5
    T = F * model.hop(cfg)
    dldy = G.counter_normal(2, 2, B * T).reshape(B, T).astype(np.float32)

    d = Generator(cfg, B, F)
    d.set_params(P)
    d.upload(z)
    want = d.forward()
    d.upload(bad, dldy=dldy)
    assert np.isfinite(d.forward()).all()  # recomputed on bf16 pairs
    d.upload(z)
    assert rel(d.forward(), want) < 1e-4  # bf16 pairs: ~2^-17 per operand
    d.close()

    a = Generator(cfg, B, F)  # the step overflows, is skipped, switched and recomputed
    a.set_params(P)
    a.train_step(bad, dldy=dldy)
    pa = a.get_params()
    a.close()

    b = Generator(cfg, B, F)  # switched by its first forward, then one step
    b.set_params(P)
    b.upload(bad, dldy=dldy)
    b.forward()
    b.set_params(P)
    b.train_step(bad, dldy=dldy)
    assert np.array_equal(b.get_params(), pa)
    b.close()

    c = Generator(cfg, B, F)
    c.set_params(P)
    c.upload(bad, dldy=dldy)
    c.step_async(0)
    with pytest.raises(RuntimeError, match="code -7"):
        c.sync()
    assert np.array_equal(c.get_params(), P)  # the overflowing step changed nothing
    c.step_async(0)
    c.sync()
    assert np.array_equal(c.get_params(), pa)
    c.close()


@pytest.mark.parametrize("tag", ["40k", "48k_snake"])
def test_forward_only_mode_gives_the_same_waveform_and_refuses_training(tag):
    """Inference mode skips the backward-only tensors: the waveform is bit-identical, backward and
    the training steps are refused while it is on, and after it is switched off a step equals a
    fresh context's step."""
    cfg = model.config(tag)
    B, F = 2, 8
    T = F * model.hop(cfg)
    P = flatten(cfg, G.init_params_ref(cfg, 9))
    z = G.counter_normal(12, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    g = G.counter_normal(12, 2, B * 256).reshape(B, 256).astype(np.float32)
    f0 = np.full((B, F), 180.0, np.float32)
    dldy = G.counter_normal(12, 3, B * T).reshape(B, T).astype(np.float32)
    ref = Generator(cfg, B, F)
    ref.set_params(P)
    ref.upload(z, f0, g, None, dldy)
    want = ref.forward(noise_stream=4)
    ref.train_step(z, f0, g, None, dldy, noise_stream=5)
    want_params = ref.get_params()
    ref.close()
    gen = Generator(cfg, B, F)
    gen.set_params(P)
    gen.set_forward_only(True)
    gen.upload(z, f0, g, None, dldy)
    assert np.array_equal(gen.forward(noise_stream=4), want)
    with pytest.raises(RuntimeError):
        gen.backward()
    with pytest.raises(RuntimeError):
        gen.train_step(z, f0, g, None, dldy, noise_stream=5)
    gen.set_forward_only(False)
    gen.train_step(z, f0, g, None, dldy, noise_stream=5)
    assert np.array_equal(gen.get_params(), want_params)
    gen.close()


@pytest.mark.parametrize("tag,B,F", [("40k", 2, 32), ("48k_snake", 1, 36), ("32k", 2, 40)])
def test_fast_inference_forward_matches_oracle(tag, B, F):
    """Fast inference (single fp16 GEMM operands, forward-only): the waveform within the 2e-3 forward
    gate of the fp64 oracle (the exact pairs reach ~1e-6), and the exact forward-only mode unchanged."""
    cfg = model.config(tag)
    z, f0, g, dldy = nsf_inputs(cfg, B, F)
    T = F * model.hop(cfg)
    dim = cfg["harmonic_num"] + 1
    stream = 9
    noise = G.counter_normal(0, stream, B * T * dim).reshape(B, T, dim)
    rand_ini = G.counter_rand_ini(0, stream, dim)
    P = G.init_params_ref(cfg, 2)
    gen = Generator(cfg, B, F, seed=0)
    gen.set_params(flatten(cfg, P))
    gen.upload(z, f0, g, noise.astype(np.float32), None)
    gen.set_forward_only(True)
    exact = gen.forward(noise_stream=stream)
    gen.set_forward_only(True, fast=True)
    fast = gen.forward(noise_stream=stream)
    gen.set_forward_only(True)
    again = gen.forward(noise_stream=stream)
    gen.close()
    a64, _ = G.train_grads(P, cfg, z, f0, g[:, :, None], noise, rand_ini, np.zeros((B, 1, T)))
    e_fast, e_exact = rel(fast, a64[:, 0, :]), rel(exact, a64[:, 0, :])
    print(f"\n[fast inference {tag}] forward rel-L2 fast {e_fast:.2e}, exact {e_exact:.2e}")
    assert e_fast <= FWD_TOL
    assert e_exact <= 1e-5
    assert np.array_equal(again, exact)


def test_fast_inference_range_error_returns_to_the_exact_pairs():
    """A fast-inference forward (single fp16 operands) whose operand reaches 65504 is recomputed on the
    range-safe bf16 pairs, and the context stays on them (asking for the fast mode again keeps them)."""
    cfg = model.decoder_only("40k")
    B, F = 1, 4
    P = flatten(cfg, G.init_params_ref(cfg, 1))
    z = G.counter_normal(2, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    bad = z.copy()
    bad[0, 5, 2] = 1e5
    ref = Generator(cfg, B, F)  # a context already on the bf16 pairs
    ref.set_params(P)
    ref.upload(bad)
    ref.forward()
    want = ref.forward()
    ref.close()
    gen = Generator(cfg, B, F)
    gen.set_params(P)
    gen.set_forward_only(True, fast=True)
    gen.upload(bad)
    got = gen.forward()  # overflows, falls back, recomputes
    assert np.isfinite(got).all()
    assert np.array_equal(got, want)
    gen.set_forward_only(True, fast=True)
    assert np.array_equal(gen.forward(), want)
    gen.close()
