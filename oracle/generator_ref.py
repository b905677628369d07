"""CPU fp64 restatement of the generator training step — TEST INFRASTRUCTURE.

This module is the parity checker (oracle) for the CUDA library in
``wuburvc_b200``.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import it; the product never does.

It restates, in float64 torch on the CPU with autograd supplying the
gradients, the math of:

* the reference C trainer's decoder (``src/wubu_train.c``):
  conv1d ``:461-486``, convT1d ``:533-562``, lrelu ``:605-620`` (slope 0.1
  everywhere, including before conv_post), the MRF pair ``:634-648`` and the
  mean over stacks ``:854-897``, conv_post + tanh ``:913-936``;
* the upstream generator the reference mirrors
  (``knowledge/rvc_original/infer/module/models.py``): SineGen ``:267-343``
  with ``harmonic_num`` harmonics, SourceModuleHnNSF ``:346-400`` (l_linear +
  tanh; the sine itself is computed without gradient, ``:333``), the noise
  convs ``:445-457``/``:499-500``, cond(g) ``:470-471``/``:493-494`` and
  GeneratorNSF.forward ``:480-514``; ResBlock1 ``modules.py:227-322``;
* weight_norm (dim 0) ``W = g * v / ||v||`` (``src/wubu_rvc_weights.c:391-408``
  without the +1e-8, as torch.nn.utils.weight_norm);
* Snake ``x + sin^2(a x)/a`` (``src/wubu_rvc_real.c:676-680``) with a learnable
  per-channel ``a``;
* AdamW exactly as ``src/wubu_train.c:90-117`` (bias correction applied
  twice: ``lr_eff = lr*sqrt(b2c)/b1c`` and ``m/b1c``, ``sqrt(v/b2c)``).

Parity of this restatement is pinned against the reference's own C trainer
built from its sources (``oracle/_ref/libwubu_ref.so``, see
``oracle/ref_oracle.py``) on the decoder subset, and against the upstream
torch ``SineGen`` / ``SourceModuleHnNSF`` for the harmonic source
(``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np
import torch
import torch.nn.functional as F

LRELU = 0.1


# --------------------------------------------------------------------------
# counter-based noise (restates the product's device generator bit-for-bit on
# the integer side: splitmix64 finaliser over (seed, stream, index))
# --------------------------------------------------------------------------
_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _mix64(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.uint64)
    with np.errstate(over="ignore"):
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        x = x ^ (x >> np.uint64(31))
    return x


def counter_uniform_pair(seed: int, stream: int, idx: np.ndarray):
    """Two uniforms in (0,1] from 64-bit hashes of (seed, stream, idx)."""
    with np.errstate(over="ignore"):
        key = _mix64(np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)
                     + np.uint64(stream) * np.uint64(0xD1B54A32D192ED03))
        h = _mix64(key ^ (idx.astype(np.uint64) * np.uint64(0x9E3779B97F4A7C15)))
    hi = (h >> np.uint64(40)).astype(np.float64)                 # 24 bits
    lo = ((h >> np.uint64(8)) & np.uint64(0xFFFFFF)).astype(np.float64)
    u1 = (hi + 1.0) / 16777216.0
    u2 = (lo + 1.0) / 16777216.0
    return u1, u2


def counter_normal(seed: int, stream: int, n: int) -> np.ndarray:
    """Box-Muller normal deviates, index 0..n-1 (float64)."""
    u1, u2 = counter_uniform_pair(seed, stream, np.arange(n, dtype=np.uint64))
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)


def counter_rand_ini(seed: int, stream: int, dim: int) -> np.ndarray:
    """Initial harmonic phases in [0,1); harmonic 0 starts at phase 0."""
    u1, _ = counter_uniform_pair(seed, stream ^ 0x5A5A, np.arange(dim, dtype=np.uint64))
    r = u1 - 1.0 / 16777216.0
    r[0] = 0.0
    return r


def _name_stream(name: str) -> int:
    import zlib
    return zlib.crc32(name.encode()) + 7


def param_names(cfg):
    """Named parameter shapes of the generator in the reference layout."""
    out = {}
    C0 = cfg["upsample_initial_channel"]
    rates, kers = cfg["upsample_rates"], cfg["upsample_kernels"]
    snake = cfg["activation"] == "snake"
    wnorm = cfg["weight_norm"]
    out["dec.conv_pre.weight"] = (C0, cfg["in_channels"], 7)
    out["dec.conv_pre.bias"] = (C0,)
    if cfg["gin_channels"]:
        out["dec.cond.weight"] = (C0, cfg["gin_channels"], 1)
        out["dec.cond.bias"] = (C0,)
    if cfg["nsf"]:
        out["dec.m_source.l_linear.weight"] = (1, cfg["harmonic_num"] + 1)
        out["dec.m_source.l_linear.bias"] = (1,)
    nk = len(cfg["resblock_kernels"])
    for L in range(len(rates)):
        cin, c = C0 >> L, C0 >> (L + 1)
        if wnorm:
            out[f"dec.ups.{L}.weight_g"] = (cin, 1, 1)
            out[f"dec.ups.{L}.weight_v"] = (cin, c, kers[L])
        else:
            out[f"dec.ups.{L}.weight"] = (cin, c, kers[L])
        out[f"dec.ups.{L}.bias"] = (c,)
        if snake:
            out[f"dec.ups_act.{L}.alpha"] = (cin,)
        if cfg["nsf"]:
            k, s, p = noise_conv_geom(cfg, L)
            out[f"dec.noise_convs.{L}.weight"] = (c, 1, k)
            out[f"dec.noise_convs.{L}.bias"] = (c,)
        for j, kk in enumerate(cfg["resblock_kernels"]):
            R = L * nk + j
            for ct in (1, 2):
                for pi in range(len(cfg["resblock_dilations"][j])):
                    base = f"dec.resblocks.{R}.convs{ct}.{pi}"
                    if wnorm:
                        out[base + ".weight_g"] = (c, 1, 1)
                    out[base + ".weight_v"] = (c, c, kk)
                    out[base + ".bias"] = (c,)
                    if snake:
                        out[f"dec.resblocks.{R}.alpha{ct}.{pi}"] = (c,)
    if snake:
        out["dec.post_act.alpha"] = (C0 >> len(rates),)
    out["dec.conv_post.weight"] = (1, C0 >> len(rates), 7)
    return out


def init_params_ref(cfg, seed: int, w_std: float = 0.01, bias_std: float = 0.0):
    """Deterministic named parameters (reference layout): conv weights / v ~ N(0, w_std) from
    the counter generator (stream keyed by the tensor name), g = ||v|| per dim-0 row,
    biases N(0, bias_std), Snake alpha 1, l_linear weight U(-1/3, 1/3)."""
    P = {}
    shapes = param_names(cfg)
    for name, shp in shapes.items():
        n = int(np.prod(shp))
        st = _name_stream(name)
        if name.endswith(".alpha"):
            P[name] = np.ones(shp, np.float32)
        elif name.endswith("l_linear.weight"):
            u1, _ = counter_uniform_pair(seed, st, np.arange(n, dtype=np.uint64))
            P[name] = ((2 * u1 - 1) / 3).reshape(shp).astype(np.float32)
        elif name.endswith(".bias"):
            P[name] = (bias_std * counter_normal(seed, st, n)).reshape(shp).astype(np.float32)
        elif name.endswith(".weight_g"):
            continue
        else:
            P[name] = (w_std * counter_normal(seed, st, n)).reshape(shp).astype(np.float32)
    for name in shapes:
        if name.endswith(".weight_g"):
            v = P[name[:-1] + "v"]
            P[name] = np.linalg.norm(v.reshape(v.shape[0], -1).astype(np.float64), axis=1).reshape(
                shapes[name]).astype(np.float32)
    return P


# --------------------------------------------------------------------------
# building blocks
# --------------------------------------------------------------------------
def snake(x, alpha):
    a = alpha.view(1, -1, 1)
    return x + torch.sin(a * x) ** 2 / a


def act(x, cfg, alpha=None, slope=None):
    if cfg["activation"] == "snake":
        return snake(x, alpha)
    return F.leaky_relu(x, cfg.get("lrelu_slope", LRELU) if slope is None else slope)


def wn(g, v):
    """weight_norm over all dims but 0."""
    norm = v.reshape(v.shape[0], -1).norm(dim=1)
    return v * (g.reshape(-1) / norm).view(-1, *([1] * (v.dim() - 1)))


def sine_source(f0, cfg, lin_w, lin_b, noise, rand_ini):
    """SineGen + SourceModuleHnNSF (models.py:309-343, :388-400).

    f0 [B,F] (Hz, 0 = unvoiced); noise [B,T,dim] standard normal deviates;
    rand_ini [dim] initial phases.  Returns har_source [B,1,T]."""
    sr = cfg["sr"]
    upp = int(np.prod(cfg["upsample_rates"]))
    dim = cfg["harmonic_num"] + 1
    B, Fr = f0.shape
    with torch.no_grad():
        f0e = f0[:, :, None]
        rad = f0e / sr * torch.arange(1, upp + 1, dtype=f0.dtype)
        rad2 = torch.fmod(rad[..., -1:] + 0.5, 1.0) - 0.5
        rad_acc = rad2.cumsum(dim=1).fmod(1.0)
        rad = rad + F.pad(rad_acc, (0, 0, 1, -1))
        rad = rad.reshape(B, -1, 1) * torch.arange(1, dim + 1, dtype=f0.dtype).view(1, 1, -1)
        rad = rad + rand_ini.view(1, 1, -1)
        sine = torch.sin(2 * math.pi * rad) * cfg["sine_amp"]
        uv = (f0e > 0).to(f0.dtype)
        uv = uv.repeat_interleave(upp, dim=1)          # nearest upsample [B,T,1]
        noise_amp = uv * cfg["noise_std"] + (1 - uv) * cfg["sine_amp"] / 3
        sw = sine * uv + noise_amp * noise
    merge = torch.tanh(sw @ lin_w.reshape(1, dim).t() + lin_b.reshape(1))
    return merge.transpose(1, 2)


def ups_pads(cfg):
    return [(k - u) // 2 for u, k in zip(cfg["upsample_rates"], cfg["upsample_kernels"])]


def noise_conv_geom(cfg, L):
    rates = cfg["upsample_rates"]
    if L + 1 < len(rates):
        s = int(np.prod(rates[L + 1:]))
        return 2 * s, s, s // 2
    return 1, 1, 0


def weight_of(P, cfg, base):
    if cfg["weight_norm"]:
        return wn(P[base + ".weight_g"], P[base + ".weight_v"])
    key = base + ".weight_v" if base.startswith("dec.resblocks") else base + ".weight"
    return P[key]


def forward(P: Dict[str, torch.Tensor], cfg, z, f0=None, g=None, noise=None,
            rand_ini=None, keep=None):
    """Generator forward.  z [B,C_in,F] -> audio [B,1,T]."""
    rates, kers = cfg["upsample_rates"], cfg["upsample_kernels"]
    pads = ups_pads(cfg)
    nk = len(cfg["resblock_kernels"])
    x = F.conv1d(z, P["dec.conv_pre.weight"], P["dec.conv_pre.bias"], padding=3)
    if cfg["gin_channels"]:
        x = x + F.conv1d(g, P["dec.cond.weight"], P["dec.cond.bias"])
    har = None
    if cfg["nsf"]:
        har = sine_source(f0, cfg, P["dec.m_source.l_linear.weight"],
                          P["dec.m_source.l_linear.bias"], noise, rand_ini)
    for L in range(len(rates)):
        x = act(x, cfg, P.get(f"dec.ups_act.{L}.alpha"))
        x = F.conv_transpose1d(x, weight_of(P, cfg, f"dec.ups.{L}"), P[f"dec.ups.{L}.bias"],
                               stride=rates[L], padding=pads[L])
        if cfg["nsf"]:
            k, s, p = noise_conv_geom(cfg, L)
            x = x + F.conv1d(har, P[f"dec.noise_convs.{L}.weight"],
                             P[f"dec.noise_convs.{L}.bias"], stride=s, padding=p)
        xs = None
        for j, (kk, dils) in enumerate(zip(cfg["resblock_kernels"], cfg["resblock_dilations"])):
            R = L * nk + j
            y = x
            for P_i, d in enumerate(dils):
                base1 = f"dec.resblocks.{R}.convs1.{P_i}"
                base2 = f"dec.resblocks.{R}.convs2.{P_i}"
                t = act(y, cfg, P.get(f"dec.resblocks.{R}.alpha1.{P_i}"))
                t = F.conv1d(t, weight_of(P, cfg, base1), P[base1 + ".bias"],
                             dilation=d, padding=d * (kk - 1) // 2)
                t = act(t, cfg, P.get(f"dec.resblocks.{R}.alpha2.{P_i}"))
                t = F.conv1d(t, weight_of(P, cfg, base2), P[base2 + ".bias"],
                             padding=(kk - 1) // 2)
                y = t + y
            xs = y if xs is None else xs + y
        x = xs / nk
        if keep is not None:
            keep[f"stage{L}"] = x
    x = act(x, cfg, P.get("dec.post_act.alpha"), slope=cfg["final_slope"])
    x = F.conv1d(x, P["dec.conv_post.weight"], None, padding=3)
    return torch.tanh(x)


def train_grads(params_np: Dict[str, np.ndarray], cfg, z, f0, g, noise, rand_ini, dldy,
                dtype=torch.float64) -> Tuple[np.ndarray, Dict[str, np.ndarray]]:
    """Forward + backward with an explicit upstream gradient dL/dy.

    Returns (audio [B,1,T], {name: grad}) as float64 numpy arrays."""
    P = {k: torch.tensor(np.asarray(v), dtype=dtype, requires_grad=True)
         for k, v in params_np.items()}
    t = lambda a: None if a is None else torch.tensor(np.asarray(a), dtype=dtype)
    audio = forward(P, cfg, t(z), t(f0), t(g), t(noise), t(rand_ini))
    audio.backward(t(dldy))
    grads = {k: (v.grad.detach().numpy().astype(np.float64) if v.grad is not None
                 else np.zeros(v.shape)) for k, v in P.items()}
    return audio.detach().numpy().astype(np.float64), grads


def adamw_step(p, grad, m, v, t, lr, b1, b2, eps, wd):
    """One AdamW update in float32, restating src/wubu_train.c:90-117 (in place)."""
    f32 = np.float32
    bias1 = f32(1.0) - np.power(f32(b1), f32(t), dtype=np.float32)
    bias2 = f32(1.0) - np.power(f32(b2), f32(t), dtype=np.float32)
    bias1 = max(bias1, f32(1e-12))
    bias2 = max(bias2, f32(1e-12))
    lr_eff = f32(lr) * np.sqrt(bias2, dtype=np.float32) / bias1
    g = grad.astype(np.float32)
    m[...] = f32(b1) * m + (f32(1) - f32(b1)) * g
    v[...] = f32(b2) * v + (f32(1) - f32(b2)) * g * g
    denom = np.sqrt(v / bias2, dtype=np.float32) + f32(eps)
    p[...] = p - (lr_eff * (m / bias1) / denom + f32(lr) * f32(wd) * p)
