"""The drop-in path end to end on the GPU: the reference's own model struct, training registry and
AdamW state (built by the reference's src/wubu_train.c, oracle/_ref) handed to the shim
(wuburvc_b200/shim/wubu_train_b200.c), which implements the reference's CUDA entry points on this
library.

* wubu_train_forward_cuda / wubu_train_backward_cuda give exactly the library's forward and
  gradients (same kernels, same inputs), the gradients written into the reference's registry by name;
* wubu_train_step_cuda equals the library's gradients followed by the reference's own host AdamW
  (wubu_adamw_step of the caller's WuBuAdamW) exactly, with the reference step's loss (MSE, and the
  multi-scale spectral term when WUBU_SPECTRAL_WEIGHT is not 0);
* the reference's own A/B program src/test_train_cuda.c, linked unmodified against the shim
  (oracle/_ref/test_train_cuda_shim, its model loader stubbed by a seeded synthetic 40 kHz decoder),
  passes: forward correlation > 0.999 against the reference CPU decoder, every gradient entry above
  1e-4 within 15 % of the reference CPU backward, loss decreasing over three shim steps;
* wubu_generator_nsf_cuda (the CLI's --cuda generator) equals the library's forward of the same
  full NSF generator and matches the fp64 oracle."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from oracle import generator_ref as G
from oracle import ref_oracle
from wuburvc_b200 import Generator, flatten, model, unflatten
from wuburvc_b200._lib import lib

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "wuburvc_b200", "shim", "libwubu_train_b200.so")
AB_PROGRAM = os.path.join(ROOT, "oracle", "_ref", "test_train_cuda_shim")
vp, ip = ctypes.c_void_p, ctypes.c_int
needs_shim = pytest.mark.skipif(not (os.path.exists(SHIM) and ref_oracle.available()),
                                reason="shim / oracle/_ref not built")


def shim_lib():
    s = ctypes.CDLL(SHIM)
    s.wubu_train_cache_alloc_cuda.restype = vp
    s.wubu_train_cache_free_cuda.argtypes = [vp]
    s.wubu_train_forward_cuda.argtypes = [vp, vp, ip, vp, ip, vp]
    s.wubu_train_backward_cuda.argtypes = [vp, vp, vp, vp, vp]
    s.wubu_train_step_cuda.argtypes = [vp, vp, vp, vp, ip, vp, ip, ctypes.POINTER(ctypes.c_float), ip]
    s.wubu_generator_nsf_cuda.argtypes = [vp, vp, ip, ip, vp, vp, vp, ip, ip, ip]
    return s


def ptr(a):
    return a.ctypes.data_as(vp)


def rel(a, b):
    a, b = np.asarray(a, np.float64).reshape(-1), np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def library_grads(cfg, P, mel, dldy, precision="bf16"):
    gen = Generator(cfg, 1, mel.shape[1], precision=precision)
    gen.set_params(flatten(cfg, P))
    gen.upload(mel[None], dldy=dldy[None])
    audio = gen.forward()[0]
    gen.backward()
    grads = unflatten(cfg, gen.get_grads())
    gen.close()
    return audio, grads


@needs_shim
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_forward_and_backward_through_the_shim_equal_the_library(precision, monkeypatch):
    """Also in the fp32 mode, which the shim takes from WUBU_B200_PRECISION."""
    if precision == "fp32":
        monkeypatch.setenv("WUBU_B200_PRECISION", "fp32")
    else:
        monkeypatch.delenv("WUBU_B200_PRECISION", raising=False)
    cfg = model.decoder_only("40k")
    F = 8
    T = F * model.hop(cfg)
    P = G.init_params_ref(cfg, 7)
    mel = G.counter_normal(21, 1, 192 * F).reshape(192, F).astype(np.float32)
    dldy = G.counter_normal(21, 2, T).astype(np.float32)
    want_audio, want = library_grads(cfg, P, mel, dldy, precision)
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    R = ref_oracle.lib()
    s = shim_lib()
    cache = s.wubu_train_cache_alloc_cuda()
    audio = np.zeros(T, np.float32)
    assert s.wubu_train_forward_cuda(R.refh_model(ref.h), ptr(mel), F, ptr(audio), T, cache) == T
    assert np.array_equal(audio, want_audio)
    assert s.wubu_train_backward_cuda(R.refh_model(ref.h), cache, ptr(mel), ptr(dldy), R.refh_registry(ref.h)) == 0
    got = ref.grads()  # the reference registry's gradient arrays, written by the shim
    assert len(got) == 155
    for n in ref.names:
        assert np.array_equal(got[n], want[n].reshape(-1)), n
    s.wubu_train_cache_free_cuda(cache)
    ref.close()


def step_loss_gradient(audio, wav, spectral):
    """dL/dy and the loss as the reference step forms them (src/wubu_train_cuda.cu:812-850), float32
    operations in the same order; the spectral gradient from the library (as the shim takes it)."""
    n = audio.size
    nf = np.float32(n)
    mse = np.cumsum((audio - wav) * (audio - wav), dtype=np.float32)[-1] / nf
    d = np.float32(2) * (audio - wav) / nf
    total = mse
    if spectral:
        ds = np.empty(n, np.float32)
        spec = np.zeros(1, np.float32)
        assert lib().wubu_b200_stft_loss_grad_host(ptr(audio), ptr(wav), 1, n, 3, ptr(ds), ptr(spec)) == 0
        g2 = np.sqrt(np.cumsum(ds * ds, dtype=np.float32)[-1] / nf, dtype=np.float32)
        scale = np.float32(1.0) * np.float32(0.5) * (np.float32(2.0) / nf) * np.sqrt(mse, dtype=np.float32) / g2
        d = d + ds * np.float32(scale)
        total = mse + spec[0]
    return d.astype(np.float32), np.float32(total)


@needs_shim
@pytest.mark.parametrize("spectral", [False, True])
def test_reference_host_step_through_the_shim(spectral, monkeypatch):
    monkeypatch.setenv("WUBU_SPECTRAL_WEIGHT", "1" if spectral else "0")
    cfg = model.decoder_only("40k")
    F = 9 if spectral else 8
    T = F * model.hop(cfg)
    P = G.init_params_ref(cfg, 7)
    mel = G.counter_normal(13, 1, 192 * F).reshape(192, F).astype(np.float32)
    wav = (0.1 * G.counter_normal(13, 2, T)).astype(np.float32)
    # expected: the library's forward, the reference step's loss gradient, the library's gradients,
    # then the reference's own AdamW on them
    gen = Generator(cfg, 1, F)
    gen.set_params(flatten(cfg, P))
    gen.upload(mel[None], dldy=np.zeros((1, T), np.float32))
    audio = gen.forward()[0]
    gen.close()
    d, total = step_loss_gradient(audio, wav, spectral)
    _, grads = library_grads(cfg, P, mel, d)
    exp = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    exp.set_grads(grads)
    exp.adamw()
    want = exp.params()
    exp.close()

    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    R = ref_oracle.lib()
    loss = ctypes.c_float(0.0)
    rc = shim_lib().wubu_train_step_cuda(R.refh_model(ref.h), R.refh_registry(ref.h), R.refh_optimizer(ref.h),
                                         ptr(mel), F, ptr(wav), T, ctypes.byref(loss), 1)
    assert rc in (0, 1)
    assert loss.value == total
    got = ref.params()
    for n in ref.names:
        assert np.array_equal(got[n], want[n]), n
    ref.close()


@pytest.mark.skipif(not os.path.exists(AB_PROGRAM), reason="the reference's A/B program was not built")
def test_reference_ab_program_passes_on_the_shim():
    """src/test_train_cuda.c, unmodified, linked against the shim (oracle/Makefile ab-program)."""
    r = subprocess.run([AB_PROGRAM], capture_output=True, text=True, timeout=600)
    print(r.stderr[-2500:])
    assert "FORWARD corr=" in r.stderr and "GRADS A/B" in r.stderr
    assert "TEST_DONE PASS" in r.stderr
    assert r.returncode == 0


@needs_shim
@pytest.mark.parametrize("use_snake,fast", [(0, False), (1, False), (0, True), (1, True)])
def test_generator_nsf_cuda_equals_library_and_matches_oracle(use_snake, fast, monkeypatch):
    """wubu_generator_nsf_cuda (src/wubu_rvc_real.h:95) on a reference model holding the full NSF
    generator as RVC checkpoints do: one-harmonic source (l_linear 1 x 1), cond(g), noise convs,
    de-normalised weights.  Without noise injection the source is deterministic, so the result must
    equal the library's own forward of the same generator (in the same inference mode) and match
    the fp64 oracle; WUBU_B200_INFERENCE=fast selects the single-fp16 mode."""
    import torch

    if fast:
        monkeypatch.setenv("WUBU_B200_INFERENCE", "fast")
    else:
        monkeypatch.delenv("WUBU_B200_INFERENCE", raising=False)

    cfg = model.config("40k", harmonic_num=0, weight_norm=False,
                       activation="snake" if use_snake else "lrelu")
    F = 16
    T = F * model.hop(cfg)
    P = G.init_params_ref(cfg, 9)
    z = G.counter_normal(31, 1, 192 * F).reshape(192, F).astype(np.float32)
    g = G.counter_normal(31, 2, 256).astype(np.float32)
    f0 = (G.counter_uniform_pair(31, 3, np.arange(F, dtype=np.uint64))[0] * 320 + 80).astype(np.float32)
    f0[[2, 7, 8]] = 0.0
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"], sample_rate=cfg["sr"])
    R = ref_oracle.lib()
    out = np.full(T, np.nan, np.float32)
    n = shim_lib().wubu_generator_nsf_cuda(R.refh_model(ref.h), ptr(z), F, 192, ptr(f0), ptr(g), ptr(out), T, 0,
                                           use_snake)
    assert n == T
    ref.close()
    gen = Generator(cfg, 1, F)
    gen.set_params(flatten(cfg, P))
    gen.set_forward_only(True, fast=fast)
    gen.upload(z[None], f0[None], g[None], np.zeros((1, T, 1), np.float32), None)
    want = gen.forward()[0]
    gen.close()
    assert np.array_equal(out, want)
    t = lambda a: torch.tensor(np.asarray(a, np.float64))
    Pt = {k: t(v) for k, v in P.items()}
    with torch.no_grad():
        a64 = G.forward(Pt, cfg, t(z[None]), t(f0[None]), t(g[None, :, None]), t(np.zeros((1, T, 1))), t(np.zeros(1)))
    assert rel(out, a64.numpy()[0, 0]) <= 2e-3
