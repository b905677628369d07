"""Bounded waits end in an error, not a hang, and leave the device usable (failure detection without
a GPU fault: no trap, no bad address, no endless loop).

* wubu_b200_wait_selftest makes one warp wait, with the same bounded wait the tensor-core kernels
  use, on a barrier that nothing arrives on: after 1 ms it gives up, the call returns
  WUBU_B200_ERR_TIMEOUT, and a convolution right after gives the right result.
* A shorter limit set with wubu_b200_set_wait_limit_ns changes nothing in a normal step (no
  legitimate wait comes near it): the parameters after one step equal those of a context built with
  the default limit, bit for bit."""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import generator_ref as G
from wuburvc_b200 import Generator, flatten, model
from wuburvc_b200._lib import lib

pytestmark = pytest.mark.gpu


def test_wait_that_nothing_completes_times_out_and_the_device_stays_usable():
    assert lib().wubu_b200_wait_selftest(ctypes.c_ulonglong(1_000_000), None) == -4
    g = torch.Generator(device="cpu").manual_seed(7)
    B, Ci, T, Co, k, dil = 2, 64, 200, 64, 7, 3
    pad = dil * (k - 1) // 2
    x = torch.randn(B, T, Ci, generator=g).to("cuda").to(torch.bfloat16)
    w = (torch.randn(Co, Ci, k, generator=g) * 0.05).to("cuda").to(torch.bfloat16)
    wk = w.permute(2, 0, 1).contiguous()
    out = torch.empty(B, T, Co, device="cuda")
    assert lib().wubu_b200_conv1d(x.data_ptr(), None, wk.data_ptr(), None, None, out.data_ptr(), B, Ci, T, Co, k,
                                  dil, pad, 0, None) == 0
    ref = F.conv1d(x.double().transpose(1, 2), w.double(), padding=pad, dilation=dil)
    assert ((out.transpose(1, 2).double() - ref).norm() / ref.norm()).item() < 1e-5
    # and again: the wait's error word belonged to that call only
    assert lib().wubu_b200_wait_selftest(ctypes.c_ulonglong(1_000_000), None) == -4


def test_short_wait_limit_leaves_a_normal_step_unchanged():
    cfg = model.config("40k")
    B, F_ = 2, 8
    T = F_ * model.hop(cfg)
    P = flatten(cfg, G.init_params_ref(cfg, 5))
    z = G.counter_normal(3, 1, B * 192 * F_).reshape(B, 192, F_).astype(np.float32)
    g = G.counter_normal(3, 2, B * 256).reshape(B, 256).astype(np.float32)
    f0 = np.full((B, F_), 150.0, np.float32)
    dldy = G.counter_normal(3, 3, B * T).reshape(B, T).astype(np.float32)
    out = []
    for limit in (0, 200_000_000):  # default (2 s), then 200 ms
        assert lib().wubu_b200_set_wait_limit_ns(ctypes.c_ulonglong(limit)) == 0
        gen = Generator(cfg, B, F_)
        gen.set_params(P)
        gen.train_step(z, f0, g, None, dldy, noise_stream=2)
        out.append(gen.get_params())
        gen.close()
    assert lib().wubu_b200_set_wait_limit_ns(ctypes.c_ulonglong(0)) == 0
    assert np.array_equal(out[0], out[1])
