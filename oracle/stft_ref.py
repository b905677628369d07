"""Multi-scale STFT spectral loss and its gradient — TEST INFRASTRUCTURE (the oracle).

Restates ``wubu_stft_loss_grad`` (``src/wubu_train.c:318-446``) in float64 numpy, vectorised over
frames and bins: for each scale w in (512, 256, 128)[:n_scales], hop w/4,
n_frames = max(1, (n - w) // hop + 1), a Hann window 0.5 - 0.5 cos(2 pi i / (w - 1)); per frame the
direct DFT X[k] = sum_t x[t] win[t] e^{-2 pi i k t / w} of both signals for k = 0..w/2, and for
k = 1..w/2 (DC skipped):

    loss  += 0.5 * (|ma - mb| + |log(ma + 1e-10) - log(mb + 1e-10)|) / nbins      (per frame)
    dm     = 0.5 * (sgn(ma - mb) + clamp(sgn(la - lb) / la, -10, 10)) / (nbins * n_frames * n_scales)
    dL/dx[start + t] += dm * (Re cos th + Im sin th) / ma * win[t]      (th = -2 pi k t / w, ma > 1e-12)

with sgn(0) = -1, la = ma + 1e-10, lb = mb + 1e-10, nbins = w/2 + 1; the frame losses are averaged
over frames, the scale losses summed and divided by n_scales (at most three scales are evaluated;
n_scales <= 0 means 3).  Samples past the end read as zero and receive no gradient.

Only ``tests/`` use this module.  ``reference_loss_grad`` calls the reference C function itself
(built from its sources by ``oracle/Makefile``) to pin the restatement.
"""
from __future__ import annotations

import ctypes

import numpy as np

WINDOWS = (512, 256, 128)


def loss_grad(a: np.ndarray, b: np.ndarray, n_scales: int = 3):
    """Loss (float) and dL/da (float64 [n]) of one pair of signals."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    n = a.shape[0]
    if n_scales <= 0:
        n_scales = 3
    # at most three scales are evaluated, but the reference divides by the count it was given
    grad = np.zeros(n)
    total = 0.0
    for si in range(min(n_scales, 3)):
        w = WINDOWS[si]
        hop = w // 4
        n_frames = max(1, (n - w) // hop + 1)
        nbins = w // 2 + 1
        win = 0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(w) / (w - 1))
        starts = np.arange(n_frames) * hop
        idx = starts[:, None] + np.arange(w)[None, :]
        inside = idx < n
        fa = np.where(inside, a[np.minimum(idx, n - 1)], 0.0) * win
        fb = np.where(inside, b[np.minimum(idx, n - 1)], 0.0) * win
        th = -2.0 * np.pi * np.outer(np.arange(nbins), np.arange(w)) / w  # [bins][t]
        c, s = np.cos(th), np.sin(th)
        ra, ia = fa @ c.T, fa @ s.T  # [frames][bins]
        rb, ib = fb @ c.T, fb @ s.T
        ma = np.sqrt(ra * ra + ia * ia)[:, 1:]
        mb = np.sqrt(rb * rb + ib * ib)[:, 1:]
        la, lb = ma + 1e-10, mb + 1e-10
        dsum = np.abs(ma - mb).sum(axis=1)
        dlog = np.abs(np.log(la) - np.log(lb)).sum(axis=1)
        total += float((0.5 * (dsum / nbins + dlog / nbins)).sum() / n_frames)
        dlog_g = np.clip(np.where(la > lb, 1.0, -1.0) / la, -10.0, 10.0)
        dm = 0.5 * (np.where(ma > mb, 1.0, -1.0) + dlog_g) / (nbins * n_frames * n_scales)
        safe = ma > 1e-12
        cr = np.where(safe, dm * ra[:, 1:] / np.where(safe, ma, 1.0), 0.0)
        ci = np.where(safe, dm * ia[:, 1:] / np.where(safe, ma, 1.0), 0.0)
        g_frames = (cr @ c[1:] + ci @ s[1:]) * win  # [frames][t]
        np.add.at(grad, idx[inside], g_frames[inside])
    return total / n_scales, grad


def reference_available() -> bool:
    from . import ref_oracle

    return ref_oracle.available()


def reference_loss_grad(a: np.ndarray, b: np.ndarray, n_scales: int = 3, sr: int = 40000):
    """The reference's own ``wubu_stft_loss_grad`` (float32, as built by oracle/Makefile)."""
    from . import ref_oracle

    h = ctypes.CDLL(ref_oracle.LIB)
    fp = ctypes.POINTER(ctypes.c_float)
    h.wubu_stft_loss_grad.restype = ctypes.c_float
    h.wubu_stft_loss_grad.argtypes = [fp, fp, ctypes.c_int, ctypes.c_int, fp, ctypes.c_int]
    a32 = np.ascontiguousarray(a, np.float32)
    b32 = np.ascontiguousarray(b, np.float32)
    g = np.zeros(a32.shape[0], np.float32)
    cp = lambda x: x.ctypes.data_as(fp)
    loss = h.wubu_stft_loss_grad(cp(a32), cp(b32), int(a32.shape[0]), int(sr), cp(g), int(n_scales))
    return float(loss), g

