"""The drop-in path end to end: the reference's own model struct, training registry and AdamW state
(built by the reference's src/wubu_train.c, oracle/_ref) handed to wubu_train_step_cuda of the shim
(wuburvc_b200/shim), which runs the step on this library and writes the weights back into the
reference's registry.  The result must equal the same step taken through this library's own API
(same kernels, same inputs, the loss gradient formed with the same float32 operations), exactly:
once with the reference step's spectral term switched off (WUBU_SPECTRAL_WEIGHT=0, dL/dy = the MSE
gradient) and once with it on (MSE gradient + the multi-scale STFT gradient rescaled by
sqrt(mse)).  The reference's OpenMP reductions run on one thread here so both sides sum alike."""
import ctypes
import os

import numpy as np
import pytest

from oracle import generator_ref as G
from oracle import ref_oracle
from wuburvc_b200 import Generator, flatten, model, unflatten
from wuburvc_b200._lib import lib

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "wuburvc_b200", "shim", "libwubu_train_b200.so")
vp = ctypes.c_void_p


def library_step(cfg, P, mel, wav, spectral):
    """The step through the library's API, dL/dy formed as the shim forms it (float32, in order)."""
    T = wav.shape[0]
    gen = Generator(cfg, 1, mel.shape[1], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2)
    gen.set_params(flatten(cfg, P))
    gen.upload(mel[None], dldy=np.zeros((1, T), np.float32))
    audio = gen.forward()[0]
    rl = ref_oracle.lib()
    rl.wubu_mse_loss.restype = ctypes.c_float
    rl.wubu_mse_loss.argtypes = [vp, vp, ctypes.c_int]
    mse = np.float32(rl.wubu_mse_loss(audio.ctypes.data_as(vp), wav.ctypes.data_as(vp), T))
    n = np.float32(T)
    d = np.float32(2) * (audio - wav) / n
    total = mse
    if spectral:
        ds = np.empty(T, np.float32)
        spec = np.zeros(1, np.float32)
        assert lib().wubu_b200_stft_loss_grad_host(audio.ctypes.data_as(vp), wav.ctypes.data_as(vp), 1, T, 3,
                                                   ds.ctypes.data_as(vp), spec.ctypes.data_as(vp)) == 0
        ss = np.cumsum(ds * ds, dtype=np.float32)[-1]
        rms = np.sqrt(ss / n, dtype=np.float32)
        k = np.float32(1.0) * np.float32(0.5) * (np.float32(2.0) / n) * np.sqrt(mse, dtype=np.float32) / rms
        d = d + ds * np.float32(k)
        total = mse + spec[0]
    gen.upload(mel[None], dldy=d.astype(np.float32)[None])
    gen.backward()
    gen.adamw()
    out = unflatten(cfg, gen.get_params())
    gen.close()
    return out, float(total)


@pytest.mark.skipif(not (os.path.exists(SHIM) and ref_oracle.available()), reason="shim / oracle/_ref not built")
@pytest.mark.parametrize("spectral", [False, True])
def test_reference_host_step_through_the_shim_equals_the_library_step(spectral, monkeypatch):
    monkeypatch.setenv("WUBU_SPECTRAL_WEIGHT", "1" if spectral else "0")
    cfg = model.decoder_only("40k")
    # the shim keeps one context per frame count (weights and AdamW state live on the device
    # between its calls), so each case uses its own frame count to start from these parameters
    F = 9 if spectral else 8
    T = F * model.hop(cfg)
    P = G.init_params_ref(cfg, 7)
    mel = G.counter_normal(13, 1, 192 * F).reshape(192, F).astype(np.float32)
    wav = (0.1 * G.counter_normal(13, 2, T)).astype(np.float32)
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    L = ref_oracle.lib()
    # one OpenMP thread: the reference's wubu_mse_loss (an OpenMP reduction) then sums in one order
    # in both runs, and the spectral scale sqrt(mse) agrees to the bit
    threads = L.refh_threads()
    L.refh_set_threads(1)
    shim = ctypes.CDLL(SHIM)
    shim.wubu_train_step_cuda.restype = ctypes.c_int
    shim.wubu_train_step_cuda.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    loss = ctypes.c_float(0.0)
    rc = shim.wubu_train_step_cuda(L.refh_model(ref.h), L.refh_registry(ref.h), L.refh_optimizer(ref.h),
                                   mel.ctypes.data_as(vp), F, wav.ctypes.data_as(vp), T, ctypes.byref(loss), 1)
    assert rc in (0, 1)
    after = ref.params()
    exp, total = library_step(cfg, P, mel, wav, spectral)
    L.refh_set_threads(threads)
    assert loss.value == np.float32(total)
    for name in ref.names:
        assert np.array_equal(after[name], exp[name].reshape(-1)), name
    ref.close()
