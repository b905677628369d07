"""The allocation-free weight-gradient entry point.

wubu_b200_conv1d_wgrad_noalloc serves callers that cannot call cudaMalloc: a host whose device
memory is owned by its own allocator (a framework's caching allocator that has reserved the HBM),
or a host that forbids allocation inside its processing callback (cudaMalloc / cudaFree take the
driver's locks and may synchronise the whole device).  It keeps its split-K scratch in a fixed
__device__ array shared by all calls.  Each of two calls in a row must match both the allocating
wubu_b200_conv1d_wgrad and the float64 weight gradient of the same bf16 inputs (rel-L2 <= 1e-5,
the weight-gradient tolerance of the kernel tests), so the second call is not disturbed by what the
first left in the shared scratch.  The cases cover 128-channel outputs, the tap-packed 64- and
32-channel outputs (two and four taps per 128-row accumulator) and a problem that needs more
scratch than the array holds (it runs with fewer splits).
This file is collected last on purpose.
"""
import pytest
import torch

from wuburvc_b200._lib import lib

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("case", [(2, 64, 500, 64, 11, 5), (1, 128, 300, 128, 7, 3),
                                  # 32 output channels: four taps per accumulator
                                  (2, 64, 400, 32, 7, 3), (1, 32, 257, 32, 11, 5),
                                  # needs more split-K scratch than the fixed array: runs with fewer splits
                                  (4, 128, 3200, 128, 11, 1)])
def test_wgrad_noalloc_matches_allocating_entry_point_and_fp64(case):
    B, Ci, T, Co, k, dil = case
    pad = dil * (k - 1) // 2
    for call in range(2):
        g = torch.Generator(device="cpu").manual_seed(100 + call)
        x = torch.randn(B, T, Ci, generator=g).to("cuda").to(torch.bfloat16)
        dy = torch.randn(B, T, Co, generator=g).to("cuda").to(torch.bfloat16)
        ref = torch.empty(Co, Ci, k, device="cuda")
        got = torch.full((Co, Ci, k), float("nan"), device="cuda")
        assert lib().wubu_b200_conv1d_wgrad(dy.data_ptr(), x.data_ptr(), ref.data_ptr(), B, Ci, T, Co, k, dil, pad,
                                            None) == 0
        assert lib().wubu_b200_conv1d_wgrad_noalloc(dy.data_ptr(), x.data_ptr(), got.data_ptr(), B, Ci, T, Co, k,
                                                    dil, pad, None) == 0
        assert torch.isfinite(got).all()
        assert rel(got, ref) <= 1e-5
        want = torch.nn.grad.conv1d_weight(x.double().transpose(1, 2), (Co, Ci, k), dy.double().transpose(1, 2),
                                           padding=pad, dilation=dil)
        assert rel(got, want) <= 1e-5
