"""GPU spectral loss (wubu_b200_stft_loss_grad) against the float64 oracle (oracle/stft_ref.py) and
the reference's own outputs (tests/golden/stft_loss.npz).  The GPU evaluates the DFTs as float32
FFTs; tolerances: loss relative 2e-5, gradient relative L2 2e-4 against the oracle, 1e-3 against the
reference (whose direct DFT rounds its phases in float32)."""
import os

import numpy as np
import pytest
import torch

import wuburvc_b200 as wb
from oracle import stft_ref

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def signals(B, n, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n) / 40000.0
    f = rng.uniform(100, 400, size=(B, 1))
    a = 0.3 * np.sin(2 * np.pi * f * t) + 0.1 * rng.standard_normal((B, n))
    b = 0.3 * np.sin(2 * np.pi * (f * 1.05) * t) + 0.1 * rng.standard_normal((B, n))
    return a.astype(np.float32), b.astype(np.float32)


@pytest.mark.parametrize("B,n,scales", [(3, 12800, 3), (2, 3000, 2), (2, 300, 3), (1, 1000, 1), (2, 900, 5),
                                        (1, 700, 0)])
def test_stft_loss_grad_matches_oracle(B, n, scales):
    a, b = signals(B, n, B * 1000 + n + scales)
    loss, grad = wb.stft_loss_grad(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), scales)
    loss, grad = loss.cpu().numpy(), grad.cpu().numpy()
    for i in range(B):
        lo, go = stft_ref.loss_grad(a[i], b[i], scales)
        assert abs(loss[i] - lo) <= 2e-5 * abs(lo), (i, loss[i], lo)
        assert rel(grad[i], go) < 2e-4, i


def test_stft_loss_grad_matches_reference_golden():
    d = np.load(os.path.join(HERE, "golden", "stft_loss.npz"))
    for i in range(int(d["n_cases"])):
        a = torch.from_numpy(d[f"a{i}"]).cuda()
        b = torch.from_numpy(d[f"b{i}"]).cuda()
        loss, grad = wb.stft_loss_grad(a, b, 3)
        ref = float(d[f"loss{i}"])
        assert abs(float(loss) - ref) <= 2e-5 * abs(ref), i
        assert rel(grad.cpu().numpy(), d[f"grad{i}"].astype(np.float64)) < 1e-3, i


def test_stft_loss_grad_deterministic():
    a, b = signals(4, 5000, 7)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    l1, g1 = wb.stft_loss_grad(ta, tb)
    l2, g2 = wb.stft_loss_grad(ta, tb)
    assert torch.equal(l1, l2) and torch.equal(g1, g2)
