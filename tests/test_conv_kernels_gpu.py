"""GPU numerics of the tcgen05 convolution primitives against a PyTorch fp64 reference.

Tolerances: split forward (operands as fp16 hi + fp16 lo/2048 pairs, three products) is
fp32-accurate -> rel-L2 <= 3e-6 against the fp64 convolution of the unsplit values; single-bf16
operands with fp32 accumulation, compared against the fp64 product of the same bf16 values -> 1e-5;
weight gradients (long fp32 sums) -> 1e-5.
"""
import pytest
import torch
import torch.nn.functional as F

from wuburvc_b200._lib import lib

pytestmark = pytest.mark.gpu

dev = "cuda"


def split(x):
    """The forward operand pair: x = hi + lo / 2048, both fp16."""
    hi = x.to(torch.float16)
    lo = ((x - hi.float()) * 2048).to(torch.float16)
    return hi.contiguous(), lo.contiguous()


def operands(x, splitmode):
    """(hi, lo) as the primitive takes them: the fp16 pair when split, else bf16 alone."""
    return split(x) if splitmode else (x.to(torch.bfloat16).contiguous(), None)


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def ptr(t):
    return t.data_ptr() if t is not None else None


CONV_CASES = [
    # B, C_in, T, C_out, k, dil
    (2, 32, 300, 32, 3, 1),
    (2, 32, 260, 32, 11, 5),
    (2, 64, 200, 64, 7, 3),
    (1, 128, 256, 128, 11, 1),
    (2, 256, 160, 256, 3, 5),
    (1, 192, 40, 512, 7, 1),
    # unequal channel counts and a single tap (the tap-packed weight gradient for 32 / 64 outputs)
    (1, 64, 333, 32, 5, 2),
    (2, 128, 190, 64, 9, 1),
    (1, 32, 129, 64, 1, 1),
]


@pytest.mark.parametrize("case", CONV_CASES)
@pytest.mark.parametrize("splitmode", [1, 0])
def test_conv1d(case, splitmode):
    B, Ci, T, Co, k, dil = case
    pad = dil * (k - 1) // 2
    g = torch.Generator(device="cpu").manual_seed(1)
    x = torch.randn(B, T, Ci, generator=g).to(dev)
    w = (torch.randn(Co, Ci, k, generator=g) * 0.05).to(dev)
    b = torch.randn(Co, generator=g).to(dev)
    xh, xl = operands(x, splitmode)
    wk = w.permute(2, 0, 1).contiguous()  # [k][Co][Ci]
    wh, wl = operands(wk, splitmode)
    out = torch.empty(B, T, Co, device=dev)
    rc = lib().wubu_b200_conv1d(ptr(xh), ptr(xl), ptr(wh), ptr(wl), ptr(b), ptr(out), B, Ci, T, Co, k, dil, pad,
                                splitmode, None)
    assert rc == 0
    if splitmode:
        ref = F.conv1d(x.double().transpose(1, 2), w.double(), b.double(), padding=pad, dilation=dil)
        tol = 3e-6
    else:
        wref = wh.double().permute(1, 2, 0)
        ref = F.conv1d(xh.double().transpose(1, 2), wref, b.double(), padding=pad, dilation=dil)
        tol = 1e-5
    assert rel(out.transpose(1, 2), ref) < tol


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv1d_wgrad(case):
    B, Ci, T, Co, k, dil = case
    pad = dil * (k - 1) // 2
    g = torch.Generator(device="cpu").manual_seed(2)
    x = torch.randn(B, T, Ci, generator=g).to(dev).to(torch.bfloat16)
    dy = torch.randn(B, T, Co, generator=g).to(dev).to(torch.bfloat16)
    dw = torch.empty(Co, Ci, k, device=dev)
    rc = lib().wubu_b200_conv1d_wgrad(ptr(dy), ptr(x), ptr(dw), B, Ci, T, Co, k, dil, pad, None)
    assert rc == 0
    xd = x.double().transpose(1, 2)
    ref = torch.nn.grad.conv1d_weight(xd, (Co, Ci, k), dy.double().transpose(1, 2), padding=pad, dilation=dil)
    assert rel(dw, ref) < 1e-5


CONVT_CASES = [
    # B, C_in, T_in, C_out, k, s
    (2, 512, 32, 256, 16, 10),
    (2, 256, 64, 128, 16, 10),
    (2, 128, 100, 64, 4, 2),
    (2, 64, 150, 32, 4, 2),
    (1, 256, 40, 128, 16, 8),
    (1, 512, 36, 256, 24, 12),
]


def phase_pack(W, s):
    """W [C_in][C_out][k] -> [k][C_out][C_in] with taps in phase order."""
    k = W.shape[2]
    order = [r + s * m for r in range(s) for m in range(k) if r + s * m < k]
    return W.permute(2, 1, 0)[order].contiguous()


@pytest.mark.parametrize("case", CONVT_CASES)
@pytest.mark.parametrize("splitmode", [1, 0])
def test_convT(case, splitmode):
    B, Ci, Ti, Co, k, s = case
    pad = (k - s) // 2
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(B, Ti, Ci, generator=g).to(dev)
    W = (torch.randn(Ci, Co, k, generator=g) * 0.05).to(dev)
    b = torch.randn(Co, generator=g).to(dev)
    xh, xl = operands(x, splitmode)
    wh, wl = operands(phase_pack(W, s), splitmode)
    out = torch.empty(B, Ti * s, Co, device=dev)
    rc = lib().wubu_b200_convT(ptr(xh), ptr(xl), ptr(wh), ptr(wl), ptr(b), ptr(out), B, Ci, Ti, Co, k, s, pad,
                               splitmode, None)
    assert rc == 0
    if splitmode:
        ref = F.conv_transpose1d(x.double().transpose(1, 2), W.double(), b.double(), stride=s, padding=pad)
        tol = 3e-6
    else:
        Wh = W.to(torch.bfloat16).double()
        ref = F.conv_transpose1d(xh.double().transpose(1, 2), Wh, b.double(), stride=s, padding=pad)
        tol = 1e-5
    assert rel(out.transpose(1, 2), ref) < tol


@pytest.mark.parametrize("case", CONVT_CASES)
def test_convT_dgrad(case):
    B, Ci, Ti, Co, k, s = case
    pad = (k - s) // 2
    g = torch.Generator(device="cpu").manual_seed(4)
    dy = torch.randn(B, Ti * s, Co, generator=g).to(dev).to(torch.bfloat16)
    W = (torch.randn(Ci, Co, k, generator=g) * 0.05).to(dev).to(torch.bfloat16)
    wd = W.permute(2, 0, 1).contiguous()  # [k][C_in][C_out]
    dx = torch.empty(B, Ti, Ci, device=dev)
    rc = lib().wubu_b200_convT_dgrad(ptr(dy), ptr(wd), ptr(dx), B, Ci, Ti, Co, k, s, pad, None)
    assert rc == 0
    ref = F.conv1d(dy.double().transpose(1, 2), W.double(), stride=s, padding=pad)
    assert rel(dx.transpose(1, 2), ref) < 1e-5


@pytest.mark.parametrize("case", CONVT_CASES)
def test_convT_wgrad(case):
    B, Ci, Ti, Co, k, s = case
    pad = (k - s) // 2
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(B, Ti, Ci, generator=g).to(dev).to(torch.bfloat16)
    dy = torch.randn(B, Ti * s, Co, generator=g).to(dev).to(torch.bfloat16)
    dw = torch.empty(Ci, Co, k, device=dev)
    rc = lib().wubu_b200_convT_wgrad(ptr(x), ptr(dy), ptr(dw), B, Ci, Ti, Co, k, s, pad, None)
    assert rc == 0
    Wd = torch.zeros(Ci, Co, k, dtype=torch.float64, device=dev, requires_grad=True)
    y = F.conv_transpose1d(x.double().transpose(1, 2), Wd, stride=s, padding=pad)
    (ref,) = torch.autograd.grad(y, Wd, dy.double().transpose(1, 2))
    assert rel(dw, ref) < 1e-5
