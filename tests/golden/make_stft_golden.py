"""Generates tests/golden/stft_loss.npz from the reference itself: ``wubu_stft_loss_grad``
(src/wubu_train.c:318-446, built unmodified by oracle/Makefile into oracle/_ref/libwubu_ref.so)
on seeded signal pairs, 3 scales.  Stored per case: the two signals, the reference loss and its
gradient with respect to the first signal.

  python tests/golden/make_stft_golden.py      (needs oracle/_ref built)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import stft_ref  # noqa: E402

# signal lengths: several frames at every scale, one frame at the largest scale only, and shorter
# than the largest window (zero-padded single frame)
CASES = (4000, 700, 300)


def main():
    rng = np.random.default_rng(20251)
    out = {}
    for i, n in enumerate(CASES):
        t = np.arange(n) / 40000.0
        # a harmonic signal against a noisy, detuned copy: realistic spectra with a few nulls
        a = (0.3 * np.sin(2 * np.pi * 220 * t) + 0.1 * rng.standard_normal(n)).astype(np.float32)
        b = (0.3 * np.sin(2 * np.pi * 233 * t) + 0.1 * rng.standard_normal(n)).astype(np.float32)
        loss, grad = stft_ref.reference_loss_grad(a, b, 3)
        out[f"a{i}"], out[f"b{i}"] = a, b
        out[f"loss{i}"] = np.float32(loss)
        out[f"grad{i}"] = grad
    np.savez_compressed(os.path.join(HERE, "stft_loss.npz"), n_cases=len(CASES), **out)
    print("wrote stft_loss.npz")


if __name__ == "__main__":
    main()
