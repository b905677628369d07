"""Checkpoint files on the host: the reference's registry dump layout (src/tt_train_demo.c:86-106:
int32 count; per entry int32 name length, name, int32 element count, float32 data) read and
written byte for byte, and a parameter set surviving a round trip."""
import struct

import numpy as np

import wuburvc_b200 as wb
from wuburvc_b200 import checkpoint, model


def test_registry_dump_layout(tmp_path):
    a = np.arange(5, dtype=np.float32) * 0.5
    b = np.array([[1.0, -2.0], [3.0, 4.5]], dtype=np.float32)
    raw = struct.pack("<i", 2)
    for name, arr in (("dec.conv_pre.weight", a), ("x", b)):
        raw += struct.pack("<i", len(name)) + name.encode() + struct.pack("<i", arr.size) + arr.astype("<f4").tobytes()
    p = tmp_path / "ref_layout.bin"
    p.write_bytes(raw)
    d = checkpoint.read_registry_dump(str(p))
    assert list(d) == ["dec.conv_pre.weight", "x"]
    assert np.array_equal(d["dec.conv_pre.weight"], a) and np.array_equal(d["x"], b.reshape(-1))
    q = tmp_path / "ours.bin"
    checkpoint.write_registry_dump(str(q), {"dec.conv_pre.weight": a, "x": b})
    assert q.read_bytes() == raw


def test_parameter_dump_round_trip(tmp_path):
    cfg = model.config("40k")
    flat = wb.init_params(cfg, seed=3)
    named = wb.unflatten(cfg, flat)
    p = tmp_path / "params.bin"
    checkpoint.write_registry_dump(str(p), named)
    d = checkpoint.read_registry_dump(str(p))
    assert list(d) == [e[0] for e in wb.param_table(cfg)]
    back = wb.flatten(cfg, checkpoint._reshape(cfg, d))
    assert np.array_equal(back, flat)


def test_int64_entries_are_exact():
    for x in (0, 1, 123456789012, 2**62 + 5):
        assert checkpoint._f32_as_i64(checkpoint._i64_as_f32(x)) == x
