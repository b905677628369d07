"""The RVC GAN discriminators on the native library (wubu_b200_disc_* of include/wuburvc_b200.h).

Mirrors the upstream training step's discriminator side (knowledge/rvc_original/train/train.py:
500-525): ``Discriminator.step(y, y_hat)`` is ``net_d(wave, y_hat.detach())`` ->
``discriminator_loss`` -> backward -> ``optim_d.step()``; ``Discriminator.gen_loss(y, y_hat)`` is
``net_d(wave, y_hat)`` -> ``generator_loss + feature_loss`` -> the gradient with respect to y_hat,
which the generator's backward takes as its dL/dy.  Parameters are upstream's state_dict
(MultiPeriodDiscriminator, models.py:928-1094) flattened in order.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict

import numpy as np

from ._lib import lib

PERIODS_V1 = (2, 3, 5, 7, 11, 17)
PERIODS_V2 = (2, 3, 5, 7, 11, 17, 23, 37)
DEVICE = 1
NO_UPDATE = 2

_vp, _ip, _fp = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
_SIGS = {
    "wubu_b200_disc_param_count": (_ip, [_vp, _ip]),
    "wubu_b200_disc_param_total": (ctypes.c_longlong, [_vp, _ip]),
    "wubu_b200_disc_param_info": (_ip, [_vp, _ip, _ip, ctypes.c_char_p, _ip, _vp, _vp]),
    "wubu_b200_disc_create": (_vp, [_ip, _ip, _vp, _ip, _vp]),
    "wubu_b200_disc_destroy": (None, [_vp]),
    "wubu_b200_disc_n_params": (ctypes.c_longlong, [_vp]),
    "wubu_b200_disc_set_params": (_ip, [_vp, _vp]),
    "wubu_b200_disc_get_params": (_ip, [_vp, _vp]),
    "wubu_b200_disc_get_grads": (_ip, [_vp, _vp]),
    "wubu_b200_disc_set_adamw": (_ip, [_vp, _fp, _fp, _fp, _fp, _fp]),
    "wubu_b200_disc_step": (_ip, [_vp, _vp, _vp, _ip, _vp]),
    "wubu_b200_disc_gen_loss": (_ip, [_vp, _vp, _vp, _vp, _ip, _vp]),
    "wubu_b200_disc_stream": (_vp, [_vp]),
    "wubu_b200_disc_sync": (_ip, [_vp]),
    "wubu_b200_disc_launches": (_ip, [_vp]),
    "wubu_b200_disc_attach_comm": (_ip, [_vp, _ip, _ip, _vp]),
    "wubu_b200_disc_set_comm_timeout_ms": (_ip, [_vp, _ip]),
}
_bound = None


def L():
    global _bound
    if _bound is None:
        h = lib()
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _bound = h
    return _bound


def _periods(periods):
    arr = (ctypes.c_int * len(periods))(*periods)
    return arr, len(periods)


def _ptr(a):
    return a.ctypes.data_as(_vp)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"wuburvc_b200 {what} failed with code {rc}")


def param_table(periods=PERIODS_V1):
    """OrderedDict name -> (offset, shape) of the flat parameter buffer."""
    arr, n = _periods(periods)
    count = L().wubu_b200_disc_param_count(arr, n)
    if count < 0:
        raise ValueError(f"bad periods {periods}")
    out = OrderedDict()
    name = ctypes.create_string_buffer(128)
    shape = (ctypes.c_int * 3)()
    off = ctypes.c_longlong()
    for i in range(count):
        _check(L().wubu_b200_disc_param_info(arr, n, i, name, 128, shape, ctypes.byref(off)), "disc_param_info")
        shp = tuple(shape) if name.value.endswith(b"weight_v") else (shape[0],)
        out[name.value.decode()] = (off.value, shp)
    return out


def param_total(periods=PERIODS_V1):
    arr, n = _periods(periods)
    return int(L().wubu_b200_disc_param_total(arr, n))


def flatten(P, periods=PERIODS_V1):
    """Named tensors (upstream's state_dict names) -> the flat fp32 buffer."""
    out = np.zeros(param_total(periods), np.float32)
    for name, (off, shp) in param_table(periods).items():
        v = np.asarray(P[name], np.float32).reshape(-1)
        out[off:off + v.size] = v
    return out


def unflatten(flat, periods=PERIODS_V1):
    return OrderedDict((name, np.asarray(flat[off:off + int(np.prod(shp))]).reshape(shp))
                       for name, (off, shp) in param_table(periods).items())


class Discriminator:
    """MultiPeriodDiscriminator for batches of B items of T samples."""

    def __init__(self, B, T, periods=PERIODS_V1, stream=None):
        self.B, self.T, self.periods = int(B), int(T), tuple(periods)
        arr, n = _periods(self.periods)
        self.h = L().wubu_b200_disc_create(self.B, self.T, arr, n, stream)
        if not self.h:
            raise RuntimeError("wubu_b200_disc_create failed (no GPU, bad shape or out of memory)")
        self.n_params = int(L().wubu_b200_disc_n_params(self.h))

    def close(self):
        if self.h:
            L().wubu_b200_disc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_params(self, flat):
        flat = np.ascontiguousarray(flat, np.float32)
        assert flat.size == self.n_params
        _check(L().wubu_b200_disc_set_params(self.h, _ptr(flat)), "disc_set_params")

    def get_params(self):
        out = np.empty(self.n_params, np.float32)
        _check(L().wubu_b200_disc_get_params(self.h, _ptr(out)), "disc_get_params")
        return out

    def get_grads(self):
        out = np.empty(self.n_params, np.float32)
        _check(L().wubu_b200_disc_get_grads(self.h, _ptr(out)), "disc_get_grads")
        return out

    def set_adamw(self, lr=1e-4, betas=(0.8, 0.99), eps=1e-9, weight_decay=0.01):
        _check(L().wubu_b200_disc_set_adamw(self.h, lr, betas[0], betas[1], eps, weight_decay), "disc_set_adamw")

    def _inputs(self, y, y_hat):
        y = np.ascontiguousarray(y, np.float32).reshape(self.B, self.T)
        y_hat = np.ascontiguousarray(y_hat, np.float32).reshape(self.B, self.T)
        return y, y_hat

    def step(self, y, y_hat, update=True):
        """Discriminator loss on (y, y_hat), its gradients and (update) the AdamW step."""
        y, y_hat = self._inputs(y, y_hat)
        loss = np.zeros(1, np.float32)
        _check(L().wubu_b200_disc_step(self.h, _ptr(y), _ptr(y_hat), 0 if update else NO_UPDATE, _ptr(loss)),
               "disc_step")
        return float(loss[0])

    def gen_loss(self, y, y_hat):
        """(generator_loss, feature_loss, dL/dy_hat [B, T])."""
        y, y_hat = self._inputs(y, y_hat)
        dy = np.empty((self.B, self.T), np.float32)
        losses = np.zeros(2, np.float32)
        _check(L().wubu_b200_disc_gen_loss(self.h, _ptr(y), _ptr(y_hat), _ptr(dy), 0, _ptr(losses)),
               "disc_gen_loss")
        return float(losses[0]), float(losses[1]), dy

    def launches(self):
        return int(L().wubu_b200_disc_launches(self.h))

    def attach_comm(self, rank, world, id128, timeout_s=60):
        """Data parallelism: the gradient is all-reduced and averaged over the ranks before AdamW.
        id128: 128 bytes from ``wuburvc_b200.Generator.nccl_unique_id()`` on one rank."""
        buf = ctypes.create_string_buffer(bytes(id128), 128)
        _check(L().wubu_b200_disc_attach_comm(self.h, int(rank), int(world), buf), "disc_attach_comm")
        _check(L().wubu_b200_disc_set_comm_timeout_ms(self.h, int(timeout_s * 1000)), "disc_set_comm_timeout")
