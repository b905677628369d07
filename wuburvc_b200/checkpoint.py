"""Checkpoints: parameters in the reference's registry dump format, plus the optimiser state.

The reference's training demo saves its trained weights as a registry dump
(``src/tt_train_demo.c:86-106``): an int32 entry count, then per entry an int32 name length, the
name bytes, an int32 element count and that many float32 values, in registry order with the
registry's names (``src/wubu_train.c:131-210``).  ``write_registry_dump`` / ``read_registry_dump``
read and write exactly that layout, so a dump written here loads in the reference and the reverse.

``save_checkpoint`` writes one such file holding, after the parameters, the AdamW state as extra
entries a reader of parameters skips by name: ``adamw.m/<name>`` and ``adamw.v/<name>`` (the first
and second moments, shaped like the parameter), ``adamw.step`` and ``source.noise_stream`` (one
int64 each, stored as the raw bytes of two float32 values).  ``load_checkpoint`` restores all of it
into a ``Generator`` so training resumes exactly where it stopped.
"""
from __future__ import annotations

import struct
from typing import Dict

import numpy as np

M_PREFIX, V_PREFIX = "adamw.m/", "adamw.v/"
STEP_KEY, NOISE_KEY = "adamw.step", "source.noise_stream"


def write_registry_dump(path: str, entries: Dict[str, np.ndarray]) -> None:
    """Entries in insertion order, each flattened to float32."""
    with open(path, "wb") as f:
        f.write(struct.pack("<i", len(entries)))
        for name, a in entries.items():
            raw = name.encode("utf-8")
            data = np.ascontiguousarray(a, dtype="<f4").reshape(-1)
            f.write(struct.pack("<i", len(raw)))
            f.write(raw)
            f.write(struct.pack("<i", data.size))
            f.write(data.tobytes())


def read_registry_dump(path: str) -> Dict[str, np.ndarray]:
    """Name -> flat float32 array, in file order."""
    out: Dict[str, np.ndarray] = {}
    with open(path, "rb") as f:
        buf = f.read()
    (count,) = struct.unpack_from("<i", buf, 0)
    pos = 4
    for _ in range(count):
        (nlen,) = struct.unpack_from("<i", buf, pos)
        pos += 4
        name = buf[pos:pos + nlen].decode("utf-8")
        pos += nlen
        (n,) = struct.unpack_from("<i", buf, pos)
        pos += 4
        if n < 0 or pos + 4 * n > len(buf):
            raise ValueError(f"truncated registry dump at entry {name!r}")
        out[name] = np.frombuffer(buf, dtype="<f4", count=n, offset=pos).astype(np.float32)
        pos += 4 * n
    return out


def _i64_as_f32(x: int) -> np.ndarray:
    return np.array([x], dtype="<i8").view("<f4")


def _f32_as_i64(a: np.ndarray) -> int:
    return int(np.ascontiguousarray(a, dtype="<f4").view("<i8")[0])


def save_checkpoint(path: str, gen, cfg: dict) -> None:
    """Parameters (registry names and order), then the AdamW moments, step and noise stream."""
    from . import unflatten

    params = unflatten(cfg, gen.get_params())
    m, v, step, stream = gen.get_opt_state()
    mn, vn = unflatten(cfg, m), unflatten(cfg, v)
    entries: Dict[str, np.ndarray] = dict(params)
    for name in params:
        entries[M_PREFIX + name] = mn[name]
    for name in params:
        entries[V_PREFIX + name] = vn[name]
    entries[STEP_KEY] = _i64_as_f32(step)
    entries[NOISE_KEY] = _i64_as_f32(stream)
    write_registry_dump(path, entries)


def load_checkpoint(path: str, gen, cfg: dict) -> None:
    """Restores parameters and, when present, the optimiser state (else the optimiser restarts)."""
    from . import flatten, param_table

    d = read_registry_dump(path)
    names = [e[0] for e in param_table(cfg)]
    missing = [n for n in names if n not in d]
    if missing:
        raise KeyError(f"checkpoint lacks {len(missing)} parameters, e.g. {missing[0]}")
    shaped = lambda prefix: {n: d[prefix + n] for n in names}
    gen.set_params(flatten(cfg, _reshape(cfg, shaped(""))))
    if all(M_PREFIX + n in d and V_PREFIX + n in d for n in names) and STEP_KEY in d:
        m = flatten(cfg, _reshape(cfg, shaped(M_PREFIX)))
        v = flatten(cfg, _reshape(cfg, shaped(V_PREFIX)))
        stream = _f32_as_i64(d[NOISE_KEY]) if NOISE_KEY in d else 0
        gen.set_opt_state(m, v, _f32_as_i64(d[STEP_KEY]), stream)


def _reshape(cfg: dict, flat_named: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """Flat entries back to the shapes flatten() expects (those unflatten() gives)."""
    from . import param_total, unflatten

    views = unflatten(cfg, np.zeros(param_total(cfg), dtype=np.float32))
    out = {}
    for n, a in flat_named.items():
        if a.size != views[n].size:
            raise ValueError(f"{n}: {a.size} values, expected {views[n].size}")
        out[n] = a.reshape(views[n].shape)
    return out
