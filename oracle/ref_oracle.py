"""ctypes driver of the reference C trainer built by oracle/Makefile — TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` use this module
(as the parity checker and the timed CPU baseline).  It loads ``oracle/_ref/libwubu_ref.so``,
which is the reference's own ``src/wubu_train.c`` (decoder_forward ``:789``, decoder_backward
``:955``, wubu_adamw_step ``:90``) plus ``src/wubu_rvc_weights.c`` (wubu_rvc_find_tensor ``:377``)
compiled unmodified, and feeds it an in-memory model.

The reference trainer has no batch dimension, no harmonic source, no cond(g) and no noise convs
(``src/wubu_train_cuda.cu:8-10``); it trains de-normalised weights named like its registry
(``src/wubu_train.c:131-210``).  Tensors outside the registry (cond, l_linear, noise convs) may be
added to the model too: the reference's inference generator and the drop-in shim read them by name.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libwubu_ref.so")

_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        h = ctypes.CDLL(LIB)
        vp, ip, fp = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        h.refh_create.restype = vp
        h.refh_create.argtypes = [ip]
        h.refh_add_tensor.restype = ip
        h.refh_add_tensor.argtypes = [vp, ctypes.c_char_p, vp, ip, vp]
        h.refh_set_ups.restype = ip
        h.refh_set_ups.argtypes = [vp, ip, vp, ip, ip, ip]
        h.refh_finalize.restype = ip
        h.refh_finalize.argtypes = [vp, fp, fp, fp, fp, fp]
        h.refh_reg_count.restype = ip
        h.refh_reg_count.argtypes = [vp]
        h.refh_reg_name.restype = ctypes.c_char_p
        h.refh_reg_name.argtypes = [vp, ip]
        h.refh_reg_size.restype = ip
        h.refh_reg_size.argtypes = [vp, ip]
        h.refh_reg_gather.restype = ctypes.c_long
        h.refh_reg_gather.argtypes = [vp, ip, vp]
        h.refh_forward.restype = ip
        h.refh_forward.argtypes = [vp, vp, ip, vp, ip]
        h.refh_backward.restype = ip
        h.refh_backward.argtypes = [vp, vp, vp]
        h.refh_adamw.restype = ip
        h.refh_adamw.argtypes = [vp]
        h.refh_reg_set_grads.restype = ctypes.c_long
        h.refh_reg_set_grads.argtypes = [vp, vp]
        h.refh_set_sample_rate.restype = None
        h.refh_set_sample_rate.argtypes = [vp, ip]
        h.refh_threads.restype = ip
        h.refh_threads.argtypes = []
        h.refh_set_threads.restype = None
        h.refh_set_threads.argtypes = [ip]
        for f in ("refh_model", "refh_registry", "refh_optimizer"):
            getattr(h, f).restype = vp
            getattr(h, f).argtypes = [vp]
        h.refh_free.restype = None
        h.refh_free.argtypes = [vp]
        _lib = h
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class RefTrainer:
    """The reference decoder trainer on one item.

    params: named fp32 arrays in the reference layout (decoder-only names:
    dec.conv_pre.weight/bias, dec.ups.L.weight/bias, dec.resblocks.R.convsX.P.weight_v/bias,
    dec.conv_post.weight); rates / kernels: upsampling config."""

    def __init__(self, params: Dict[str, np.ndarray], rates, kernels, lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 wd=1e-4, sample_rate=0):
        L = lib()
        self.h = L.refh_create(320)
        if sample_rate:
            L.refh_set_sample_rate(self.h, sample_rate)
        self._keep = []
        for name, a in params.items():
            a = np.ascontiguousarray(a, dtype=np.float32)
            if name.startswith("dec.ups.") and name.endswith(".weight"):
                layer = int(name.split(".")[2])
                if L.refh_set_ups(self.h, layer, _p(a), a.size, rates[layer], kernels[layer]) != 0:
                    raise RuntimeError("refh_set_ups")
                continue
            dims = np.array(a.shape if a.ndim else (1,), dtype=np.int32)
            if L.refh_add_tensor(self.h, name.encode(), _p(a), dims.size, _p(dims)) < 0:
                raise RuntimeError("refh_add_tensor")
        n = L.refh_finalize(self.h, lr, betas[0], betas[1], eps, wd)
        if n <= 0:
            raise RuntimeError("reference registry is empty")
        self.names: List[str] = [L.refh_reg_name(self.h, i).decode() for i in range(n)]
        self.sizes: List[int] = [L.refh_reg_size(self.h, i) for i in range(n)]

    def close(self):
        if self.h:
            lib().refh_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, mel: np.ndarray) -> np.ndarray:
        """mel [C_in, F] -> audio [T]"""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        F = mel.shape[1]
        out = np.zeros(F * 480, dtype=np.float32)
        n = lib().refh_forward(self.h, _p(mel), F, _p(out), out.size)
        if n <= 0:
            raise RuntimeError("reference forward failed")
        self._mel = mel
        return out[:n].copy()

    def backward(self, d_audio: np.ndarray):
        d = np.ascontiguousarray(d_audio, dtype=np.float32)
        if lib().refh_backward(self.h, _p(self._mel), _p(d)) != 0:
            raise RuntimeError("reference backward failed")

    def _gather(self, which) -> Dict[str, np.ndarray]:
        flat = np.zeros(sum(self.sizes), dtype=np.float32)
        lib().refh_reg_gather(self.h, which, _p(flat))
        out, off = {}, 0
        for n, s in zip(self.names, self.sizes):
            out[n] = flat[off:off + s].copy()
            off += s
        return out

    def grads(self) -> Dict[str, np.ndarray]:
        return self._gather(1)

    def params(self) -> Dict[str, np.ndarray]:
        return self._gather(0)

    def adamw(self):
        lib().refh_adamw(self.h)

    def set_grads(self, named: Dict[str, np.ndarray]):
        """Registry gradients from named arrays (e.g. computed by the CUDA library)."""
        flat = np.concatenate([np.ascontiguousarray(named[n], dtype=np.float32).reshape(-1) for n in self.names])
        lib().refh_reg_set_grads(self.h, _p(flat))

    @staticmethod
    def threads() -> int:
        return lib().refh_threads()
