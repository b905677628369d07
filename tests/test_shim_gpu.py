"""The drop-in path end to end: the reference's own model struct, training registry and AdamW state
(built by the reference's src/wubu_train.c, oracle/_ref) handed to wubu_train_step_cuda of the shim
(wuburvc_b200/shim), which runs the step on this library and writes the weights back into the
reference's registry.  The result must equal the same step taken through this library's Python API
exactly (same kernels, same inputs), and the reported loss must be the reference's wubu_mse_loss."""
import ctypes
import os

import numpy as np
import pytest

from oracle import generator_ref as G
from oracle import ref_oracle
from wuburvc_b200 import Generator, flatten, model, unflatten

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "wuburvc_b200", "shim", "libwubu_train_b200.so")


@pytest.mark.skipif(not (os.path.exists(SHIM) and ref_oracle.available()), reason="shim / oracle/_ref not built")
def test_reference_host_step_through_the_shim_equals_the_library_step():
    cfg = model.decoder_only("40k")
    F = 8
    T = F * model.hop(cfg)
    P = G.init_params_ref(cfg, 7)
    mel = G.counter_normal(13, 1, 192 * F).reshape(192, F).astype(np.float32)
    wav = (0.1 * G.counter_normal(13, 2, T)).astype(np.float32)
    ref = ref_oracle.RefTrainer(P, cfg["upsample_rates"], cfg["upsample_kernels"])
    L = ref_oracle.lib()
    shim = ctypes.CDLL(SHIM)
    vp = ctypes.c_void_p
    shim.wubu_train_step_cuda.restype = ctypes.c_int
    shim.wubu_train_step_cuda.argtypes = [vp, vp, vp, vp, ctypes.c_int, vp, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    loss = ctypes.c_float(0.0)
    rc = shim.wubu_train_step_cuda(L.refh_model(ref.h), L.refh_registry(ref.h), L.refh_optimizer(ref.h),
                                   mel.ctypes.data_as(vp), F, wav.ctypes.data_as(vp), T, ctypes.byref(loss), 1)
    assert rc in (0, 1)
    after = ref.params()
    # the same step through the Python API
    gen = Generator(cfg, 1, F)
    gen.set_params(flatten(cfg, P))
    gen.upload(mel[None], dldy=np.zeros((1, T), np.float32))
    audio = gen.forward()[0]
    d = (2 * (audio - wav) / T).astype(np.float32)
    gen.upload(mel[None], dldy=d[None])
    gen.backward()
    gen.adamw()
    exp = unflatten(cfg, gen.get_params())
    gen.close()
    mse = float(np.mean((audio.astype(np.float64) - wav) ** 2))
    assert abs(loss.value - mse) <= 1e-5 * mse
    for name in ref.names:
        assert np.array_equal(after[name], exp[name].reshape(-1)), name
    ref.close()
