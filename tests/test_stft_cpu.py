"""The spectral-loss oracle (oracle/stft_ref.py) pinned to the reference's wubu_stft_loss_grad
(src/wubu_train.c:318-446): against the committed golden outputs of the reference itself
(tests/golden/stft_loss.npz, made by tests/golden/make_stft_golden.py), and against the reference
library directly where oracle/_ref is built.

The reference accumulates its direct DFT in float32 with phases rounded in float32; the oracle is
float64, so the loss agrees to ~1e-6 and the gradient to a few 1e-4 (relative L2)."""
import os

import numpy as np
import pytest

from oracle import stft_ref

HERE = os.path.dirname(os.path.abspath(__file__))


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_oracle_matches_reference_golden():
    d = np.load(os.path.join(HERE, "golden", "stft_loss.npz"))
    for i in range(int(d["n_cases"])):
        loss, grad = stft_ref.loss_grad(d[f"a{i}"], d[f"b{i}"], 3)
        ref_loss = float(d[f"loss{i}"])
        assert abs(loss - ref_loss) <= 5e-6 * abs(ref_loss), (i, loss, ref_loss)
        assert rel(d[f"grad{i}"], grad) < 1e-3, i


@pytest.mark.skipif(not stft_ref.reference_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("n,scales", [(2500, 3), (600, 2), (200, 1), (1000, 5), (900, 0)])
def test_oracle_matches_reference_library(n, scales):
    rng = np.random.default_rng(n + scales)
    a = (0.2 * rng.standard_normal(n)).astype(np.float32)
    b = (0.2 * rng.standard_normal(n)).astype(np.float32)
    loss, grad = stft_ref.loss_grad(a, b, scales)
    ref_loss, ref_grad = stft_ref.reference_loss_grad(a, b, scales)
    assert abs(loss - ref_loss) <= 5e-6 * abs(ref_loss)
    assert rel(ref_grad, grad) < 1e-3
