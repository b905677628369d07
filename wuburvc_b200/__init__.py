"""wuburvc_b200 — B200-native (sm_100a) NSF-HiFiGAN generator training step.

The product is the native library ``libwuburvc_b200.so`` (C ABI, ``include/wuburvc_b200.h``);
this package is the host-side mirror of the reference's training interface for Python callers
(tests, benchmarks).  It mirrors ``src/wubu_train.h`` of the reference: a registry of named
trainable tensors (``wubu_train_registry_build``), a forward, a backward that writes one gradient
per registry entry, and the AdamW update (``wubu_adamw_step``), with batched inputs added.

There is no CPU fallback: without the native library (or without a GPU) the calls raise.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import model
from ._lib import LibraryMissing, check, lib

__all__ = ["GenConfig", "param_table", "init_params", "Generator", "LibraryMissing", "model", "stft_loss_grad"]


class GenConfig(ctypes.Structure):
    _fields_ = [
        ("sample_rate", ctypes.c_int),
        ("n_ups", ctypes.c_int),
        ("upsample_rates", ctypes.c_int * 4),
        ("upsample_kernels", ctypes.c_int * 4),
        ("initial_channel", ctypes.c_int),
        ("in_channels", ctypes.c_int),
        ("gin_channels", ctypes.c_int),
        ("n_kernels", ctypes.c_int),
        ("resblock_kernels", ctypes.c_int * 3),
        ("n_dilations", ctypes.c_int),
        ("resblock_dilations", (ctypes.c_int * 3) * 3),
        ("harmonic_num", ctypes.c_int),
        ("sine_amp", ctypes.c_float),
        ("noise_std", ctypes.c_float),
        ("activation", ctypes.c_int),
        ("lrelu_slope", ctypes.c_float),
        ("final_slope", ctypes.c_float),
        ("weight_norm", ctypes.c_int),
        ("nsf", ctypes.c_int),
    ]

    @classmethod
    def from_dict(cls, c: dict) -> "GenConfig":
        s = cls()
        s.sample_rate = c["sr"]
        s.n_ups = len(c["upsample_rates"])
        for i, (u, k) in enumerate(zip(c["upsample_rates"], c["upsample_kernels"])):
            s.upsample_rates[i] = u
            s.upsample_kernels[i] = k
        s.initial_channel = c["upsample_initial_channel"]
        s.in_channels = c["in_channels"]
        s.gin_channels = c["gin_channels"]
        s.n_kernels = len(c["resblock_kernels"])
        for j, k in enumerate(c["resblock_kernels"]):
            s.resblock_kernels[j] = k
        s.n_dilations = len(c["resblock_dilations"][0])
        for j, ds in enumerate(c["resblock_dilations"]):
            for p, d in enumerate(ds):
                s.resblock_dilations[j][p] = d
        s.harmonic_num = c["harmonic_num"]
        s.sine_amp = c["sine_amp"]
        s.noise_std = c["noise_std"]
        s.activation = 1 if c["activation"] == "snake" else 0
        s.lrelu_slope = c["lrelu_slope"]
        s.final_slope = c["final_slope"]
        s.weight_norm = 1 if c["weight_norm"] else 0
        s.nsf = 1 if c["nsf"] else 0
        return s


class TrainOptions(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int),
        ("frames", ctypes.c_int),
        ("device", ctypes.c_int),
        ("lr", ctypes.c_float),
        ("beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("weight_decay", ctypes.c_float),
        ("seed", ctypes.c_ulonglong),
        ("precision", ctypes.c_int),
    ]

PRECISIONS = {"bf16": 0, "fp32": 1}


_SIGS = {
    "wubu_b200_gen_param_count": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_param_total": (ctypes.c_longlong, [ctypes.c_void_p]),
    "wubu_b200_gen_param_info": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_gen_init_params": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p]),
    "wubu_b200_gen_bucket_plan": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "wubu_b200_gen_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_gen_destroy": (None, [ctypes.c_void_p]),
    "wubu_b200_gen_set_params": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_gen_get_params": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_gen_get_grads": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_gen_get_opt_state": (ctypes.c_int, [ctypes.c_void_p] * 5),
    "wubu_b200_gen_set_opt_state": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                   ctypes.c_longlong, ctypes.c_ulonglong]),
    "wubu_b200_gen_samples": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_upload": (ctypes.c_int, [ctypes.c_void_p] * 6),
    "wubu_b200_gen_forward": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p]),
    "wubu_b200_gen_set_forward_only": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "wubu_b200_gen_backward": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_adamw": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_train_step": (ctypes.c_int, [ctypes.c_void_p] * 7 + [ctypes.c_ulonglong, ctypes.c_int]),
    "wubu_b200_gen_train_step_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_ulonglong]),
    "wubu_b200_gen_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "wubu_b200_gen_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_graph_kernels": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_kernel_bench": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_void_p, ctypes.c_void_p]),
    "wubu_b200_nccl_unique_id": (ctypes.c_int, [ctypes.c_void_p]),
    "wubu_b200_gen_attach_comm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "wubu_b200_gen_set_comm_timeout_ms": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
}

INPUTS_RESIDENT = 1
KINDS = ["conv_w", "convT_w", "wn_g", "wn_v", "bias", "alpha", "lin_w", "lin_b"]


def L():
    h = lib()
    if not getattr(h, "_gen_sigs", False):
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        h._gen_sigs = True
    return h


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def param_table(cfg: dict) -> List[Tuple[str, str, Tuple[int, int, int], int, int]]:
    """[(name, kind, shape3, offset, numel)] in flat-buffer order (host only)."""
    c = GenConfig.from_dict(cfg)
    n = L().wubu_b200_gen_param_count(ctypes.byref(c))
    if n < 0:
        raise ValueError("invalid generator config")
    out = []
    name = ctypes.create_string_buffer(160)
    shape = (ctypes.c_int * 3)()
    off, numel = ctypes.c_longlong(), ctypes.c_longlong()
    for i in range(n):
        kind = L().wubu_b200_gen_param_info(ctypes.byref(c), i, name, 160, shape, ctypes.byref(off),
                                            ctypes.byref(numel))
        out.append((name.value.decode(), KINDS[kind], tuple(shape), off.value, numel.value))
    return out


def param_total(cfg: dict) -> int:
    c = GenConfig.from_dict(cfg)
    return int(L().wubu_b200_gen_param_total(ctypes.byref(c)))


def bucket_plan(cfg: dict) -> List[Tuple[int, int]]:
    """Data-parallel all-reduce buckets [(start, end)] of the flat gradient buffer, in the order the
    backward finishes them (host only)."""
    c = GenConfig.from_dict(cfg)
    ends = (ctypes.c_longlong * 16)()
    n = L().wubu_b200_gen_bucket_plan(ctypes.byref(c), ends, 16)
    if n < 0:
        raise ValueError("invalid generator config")
    out, prev = [], 0
    for i in range(n):
        out.append((prev, int(ends[i])))
        prev = int(ends[i])
    return out


def stft_loss_grad(a, b, n_scales: int = 3):
    """Multi-scale STFT spectral loss (windows 512/256/128) of B signal pairs and its gradient with
    respect to ``a`` (the reference's wubu_stft_loss_grad, src/wubu_train.c:318-446, batched on the
    device).  ``a`` and ``b``: CUDA float32 tensors [B][n] (or [n]).  Returns (loss [B], grad)."""
    import torch

    if not (a.is_cuda and b.is_cuda) or a.shape != b.shape:
        raise ValueError("a and b: CUDA tensors of the same shape")
    squeeze = a.dim() == 1
    a2 = a.reshape(1, -1) if squeeze else a
    b2 = b.reshape(1, -1) if squeeze else b
    a2 = a2.to(torch.float32).contiguous()
    b2 = b2.to(torch.float32).contiguous()
    B, n = a2.shape
    grad = torch.empty_like(a2)
    loss = torch.empty(B, device=a2.device, dtype=torch.float32)
    stream = torch.cuda.current_stream(a2.device).cuda_stream
    check(lib().wubu_b200_stft_loss_grad(a2.data_ptr(), b2.data_ptr(), B, n, n_scales, grad.data_ptr(),
                                         loss.data_ptr(), stream), "stft_loss_grad")
    return (loss[0], grad[0]) if squeeze else (loss, grad)


def init_params(cfg: dict, seed: int = 0) -> np.ndarray:
    c = GenConfig.from_dict(cfg)
    flat = np.zeros(param_total(cfg), dtype=np.float32)
    check(L().wubu_b200_gen_init_params(ctypes.byref(c), seed, _ptr(flat)), "init_params")
    return flat


def unflatten(cfg: dict, flat: np.ndarray) -> Dict[str, np.ndarray]:
    """Named views of a flat buffer, shaped like the reference / torch tensors."""
    out = {}
    for name, kind, shape, off, n in param_table(cfg):
        a = flat[off:off + n]
        if kind in ("bias", "alpha") or name.endswith("l_linear.bias"):
            a = a.reshape(shape[0])
        elif kind == "lin_w":
            a = a.reshape(1, shape[1])
        else:
            a = a.reshape(shape)
        out[name] = a
    return out


def flatten(cfg: dict, named: Dict[str, np.ndarray]) -> np.ndarray:
    flat = np.zeros(param_total(cfg), dtype=np.float32)
    for name, kind, shape, off, n in param_table(cfg):
        flat[off:off + n] = np.asarray(named[name], dtype=np.float32).reshape(-1)
    return flat


class Generator:
    """One training context on one GPU (``batch`` items of ``frames`` frames)."""

    def __init__(self, cfg: dict, batch: int, frames: int, device: int = 0, lr: float = 1e-3,
                 betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-4, seed: int = 0,
                 precision: str = "bf16"):
        """precision: "bf16" (backward GEMMs on bf16 operands) or "fp32" (bf16 hi + lo pairs, three
        products: fp32-accurate gradients at about three times the backward's tensor work)."""
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.cfg = dict(cfg)
        self.B, self.F = batch, frames
        self.precision = precision
        self._c = GenConfig.from_dict(cfg)
        o = TrainOptions()
        o.batch, o.frames, o.device = batch, frames, device
        o.lr, o.beta1, o.beta2, o.eps, o.weight_decay = lr, betas[0], betas[1], eps, weight_decay
        o.seed = seed
        o.precision = PRECISIONS[precision]
        self._o = o
        self.h = L().wubu_b200_gen_create(ctypes.byref(self._c), ctypes.byref(o))
        if not self.h:
            raise RuntimeError("wubu_b200_gen_create failed (no sm_100 GPU, bad config or out of memory)")
        self.T = L().wubu_b200_gen_samples(self.h)
        self.table = param_table(cfg)
        self.total = param_total(cfg)

    def close(self):
        if getattr(self, "h", None):
            L().wubu_b200_gen_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- parameters ----
    def set_params(self, flat: np.ndarray):
        flat = _f32(flat)
        assert flat.size == self.total
        check(L().wubu_b200_gen_set_params(self.h, _ptr(flat)), "set_params")

    def get_params(self) -> np.ndarray:
        out = np.empty(self.total, dtype=np.float32)
        check(L().wubu_b200_gen_get_params(self.h, _ptr(out)), "get_params")
        return out

    def get_opt_state(self):
        """AdamW moments (flat, reference layout), step count and source-noise stream."""
        m = np.empty(self.total, dtype=np.float32)
        v = np.empty(self.total, dtype=np.float32)
        step, stream = ctypes.c_longlong(0), ctypes.c_ulonglong(0)
        check(L().wubu_b200_gen_get_opt_state(self.h, _ptr(m), _ptr(v), ctypes.byref(step), ctypes.byref(stream)),
              "get_opt_state")
        return m, v, int(step.value), int(stream.value)

    def set_opt_state(self, m: np.ndarray, v: np.ndarray, step: int, noise_stream: int = 0):
        """Restores the optimiser (after set_params, which restarts it)."""
        m, v = _f32(m), _f32(v)
        assert m.size == self.total and v.size == self.total
        check(L().wubu_b200_gen_set_opt_state(self.h, _ptr(m), _ptr(v), int(step), int(noise_stream)),
              "set_opt_state")

    def get_grads(self) -> np.ndarray:
        out = np.empty(self.total, dtype=np.float32)
        check(L().wubu_b200_gen_get_grads(self.h, _ptr(out)), "get_grads")
        return out

    # ---- step ----
    def upload(self, z, f0=None, g=None, noise=None, dldy=None):
        self._keep = [_f32(z), _f32(f0), _f32(g), _f32(noise), _f32(dldy)]
        check(L().wubu_b200_gen_upload(self.h, *[_ptr(a) for a in self._keep]), "upload")

    def forward(self, noise_stream: int = 0) -> np.ndarray:
        out = np.empty((self.B, self.T), dtype=np.float32)
        check(L().wubu_b200_gen_forward(self.h, noise_stream, _ptr(out)), "forward")
        return out

    def set_forward_only(self, on: bool = True, fast: bool = False):
        """Inference mode: the forward skips what only the backward reads (same waveform); with
        fast, single fp16 GEMM operands (forward rel-L2 ~4e-4 against fp64).  Backward and training
        steps raise while it is on."""
        check(L().wubu_b200_gen_set_forward_only(self.h, (2 if fast else 1) if on else 0), "set_forward_only")

    def backward(self):
        check(L().wubu_b200_gen_backward(self.h), "backward")

    def adamw(self):
        check(L().wubu_b200_gen_adamw(self.h), "adamw")

    def train_step(self, z=None, f0=None, g=None, noise=None, dldy=None, noise_stream: int = 0,
                   resident: bool = False, audio_out: Optional[np.ndarray] = None):
        arrs = [_f32(z), _f32(f0), _f32(g), _f32(noise), _f32(dldy)]
        rc = L().wubu_b200_gen_train_step(self.h, *[_ptr(a) for a in arrs], _ptr(audio_out), noise_stream,
                                          INPUTS_RESIDENT if resident else 0)
        check(rc, "train_step")
        return audio_out

    def train_step_raw(self, z_ptr, f0_ptr, g_ptr, dldy_ptr, audio_ptr, noise_stream: int = 0):
        """Step with caller-owned host buffers (raw addresses, e.g. pinned torch tensors)."""
        rc = L().wubu_b200_gen_train_step(self.h, z_ptr, f0_ptr, g_ptr, None, dldy_ptr, audio_ptr, noise_stream, 0)
        check(rc, "train_step")

    def step_async(self, noise_stream: int = 0):
        check(L().wubu_b200_gen_train_step_async(self.h, noise_stream), "train_step_async")

    def sync(self):
        check(L().wubu_b200_gen_sync(self.h), "sync")

    @property
    def stream(self) -> int:
        return L().wubu_b200_gen_stream(self.h) or 0

    def graph_kernels(self) -> int:
        return int(L().wubu_b200_gen_graph_kernels(self.h))

    def kernel_bench(self, which: int, stage: int, iters: int = 20):
        ms, fl = ctypes.c_float(), ctypes.c_double()
        check(L().wubu_b200_gen_kernel_bench(self.h, which, stage, iters, ctypes.byref(ms), ctypes.byref(fl)),
              "kernel_bench")
        return ms.value, fl.value

    # ---- data parallel ----
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(L().wubu_b200_nccl_unique_id(buf), "nccl_unique_id")
        return buf.raw

    def attach_comm(self, rank: int, world: int, uid: bytes):
        buf = ctypes.create_string_buffer(uid, 128)
        check(L().wubu_b200_gen_attach_comm(self.h, rank, world, buf), "attach_comm")

    def set_comm_timeout(self, seconds: float):
        """Deadline for a step's collectives; past it the communicator is aborted (WUBU_B200_ERR_COMM)."""
        check(L().wubu_b200_gen_set_comm_timeout_ms(self.h, max(1, int(seconds * 1000))), "set_comm_timeout")
