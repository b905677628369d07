"""ctypes binding of the native library ``libwuburvc_b200.so``.

There is no fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwuburvc_b200.so")

_lib = None

c_int, c_float, c_void_p, c_char_p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p
c_size_t, c_long = ctypes.c_size_t, ctypes.c_long
P = ctypes.POINTER

# name -> (restype, argtypes); every symbol declared in include/wuburvc_b200.h
SIGNATURES = {
    "wubu_b200_conv1d": (c_int, [c_void_p] * 4 + [c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]),
    "wubu_b200_conv1d_wgrad": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "wubu_b200_conv1d_wgrad_noalloc": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "wubu_b200_convT": (c_int, [c_void_p] * 4 + [c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]),
    "wubu_b200_convT_dgrad": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "wubu_b200_convT_wgrad": (c_int, [c_void_p, c_void_p, c_void_p] + [c_int] * 7 + [c_void_p]),
    "wubu_b200_stft_loss_grad": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "wubu_b200_stft_loss_grad_host": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "wubu_b200_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "wubu_b200_wait_selftest": (c_int, [ctypes.c_ulonglong, c_void_p]),
}


class LibraryMissing(RuntimeError):
    pass


def lib():
    """Loads (once) and returns the native library; raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(f"{LIB_PATH} not built (run python -m wuburvc_b200.build)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str = "call"):
    if rc != 0:
        raise RuntimeError(f"wuburvc_b200 {what} failed with code {rc}")
    return rc
