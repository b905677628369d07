"""Generator configurations and the flat parameter table (host side).

The parameter table is defined once, in the native library
(``csrc/param_table.cpp``), and read back through the C-ABI; this module only
holds the named configurations the reference ships and small helpers.

Configurations follow ``knowledge/rvc_original/configs/v2/{32k,48k}.json`` and
``configs/v1/40k.json`` of the reference (upsample rates / kernels, 512 initial
channels, resblock kernels [3,7,11] x dilations [1,3,5], gin 256), and the
reference C trainer's decoder (``src/wubu_train.c:776-939``) for the
``decoder_only`` variant it trains (no cond, no sine source, no noise convs,
de-normalised weights trained directly).
"""
from __future__ import annotations

import copy
from typing import Dict

ACT_LRELU = 0
ACT_SNAKE = 1

_BASE = dict(
    in_channels=192,
    upsample_initial_channel=512,
    gin_channels=256,
    resblock_kernels=(3, 7, 11),
    resblock_dilations=((1, 3, 5), (1, 3, 5), (1, 3, 5)),
    harmonic_num=8,
    sine_amp=0.1,
    noise_std=0.003,
    activation="lrelu",
    lrelu_slope=0.1,
    final_slope=0.1,
    weight_norm=True,
    nsf=True,
)

CONFIGS: Dict[str, dict] = {
    "40k": dict(_BASE, sr=40000, upsample_rates=(10, 10, 2, 2), upsample_kernels=(16, 16, 4, 4)),
    "32k": dict(_BASE, sr=32000, upsample_rates=(10, 8, 2, 2), upsample_kernels=(20, 16, 4, 4)),
    "48k": dict(_BASE, sr=48000, upsample_rates=(12, 10, 2, 2), upsample_kernels=(24, 20, 4, 4)),
    "48k_snake": dict(_BASE, sr=48000, upsample_rates=(12, 10, 2, 2),
                      upsample_kernels=(24, 20, 4, 4), activation="snake"),
}


def config(name: str, **overrides) -> dict:
    c = copy.deepcopy(CONFIGS[name])
    c.update(overrides)
    return c


def decoder_only(name: str = "40k") -> dict:
    """The reference C trainer's decoder: conv_pre -> 4 x (lrelu, convT, MRF)
    -> lrelu -> conv_post -> tanh, trained on de-normalised weights."""
    return config(name, gin_channels=0, nsf=False, weight_norm=False)


def hop(cfg: dict) -> int:
    h = 1
    for r in cfg["upsample_rates"]:
        h *= r
    return h


def stage_lengths(cfg: dict, frames: int):
    out, n = [], frames
    for u, k in zip(cfg["upsample_rates"], cfg["upsample_kernels"]):
        p = (k - u) // 2
        n = (n - 1) * u - 2 * p + k
        out.append(n)
    return out


def stage_channels(cfg: dict):
    c0 = cfg["upsample_initial_channel"]
    return [c0 >> (L + 1) for L in range(len(cfg["upsample_rates"]))]


def train_flops_per_item(cfg: dict, frames: int) -> float:
    """Algorithmic conv FLOPs of one training item (2*MAC, forward x3 for
    forward + input-gradient + weight-gradient)."""
    T = stage_lengths(cfg, frames)
    C = stage_channels(cfg)
    c0 = cfg["upsample_initial_channel"]
    f = 2.0 * frames * c0 * cfg["in_channels"] * 7                     # conv_pre
    if cfg["gin_channels"]:
        f += 2.0 * c0 * cfg["gin_channels"]                            # cond (per item)
    cin = c0
    rates = cfg["upsample_rates"]
    for L, (u, k) in enumerate(zip(rates, cfg["upsample_kernels"])):
        n_in = T[L] // u
        f += 2.0 * n_in * cin * C[L] * k                                # convT
        if cfg["nsf"]:
            kn = 2 * (hop(cfg) // (T[L] // frames)) if L + 1 < len(rates) else 1
            f += 2.0 * T[L] * C[L] * kn                                 # noise conv
        for kk, dils in zip(cfg["resblock_kernels"], cfg["resblock_dilations"]):
            f += len(dils) * 2 * 2.0 * T[L] * C[L] * C[L] * kk          # MRF pairs
        cin = C[L]
    f += 2.0 * T[-1] * C[-1] * 7                                        # conv_post
    return 3.0 * f
