"""Checkpoint / resume on the GPU: a context restored from a checkpoint (registry dump of the
parameters plus the AdamW moments, step count and noise stream) continues training exactly like
the context that wrote it.  Every kernel of the step is deterministic, so the comparison is exact."""
import numpy as np
import pytest

from oracle import generator_ref as G
from wuburvc_b200 import Generator, checkpoint, flatten, model

pytestmark = pytest.mark.gpu


def inputs(cfg, B, F, seed):
    T = F * model.hop(cfg)
    z = G.counter_normal(seed, 1, B * 192 * F).reshape(B, 192, F).astype(np.float32)
    g = G.counter_normal(seed, 2, B * 256).reshape(B, 256).astype(np.float32)
    f0 = np.abs(G.counter_normal(seed, 3, B * F).reshape(B, F)).astype(np.float32) * 100 + 100
    noise = G.counter_normal(seed, 4, B * T * 9).reshape(B, T, 9).astype(np.float32)
    dldy = G.counter_normal(seed, 5, B * T).reshape(B, T).astype(np.float32)
    return z, f0, g, noise, dldy


def test_resume_from_checkpoint_continues_exactly(tmp_path):
    cfg = model.config("40k")
    B, F = 2, 4
    a = Generator(cfg, B, F)
    a.set_params(flatten(cfg, G.init_params_ref(cfg, 4)))
    for s in range(2):
        a.train_step(*inputs(cfg, B, F, 10 + s), noise_stream=s)
    path = tmp_path / "ckpt.bin"
    checkpoint.save_checkpoint(str(path), a, cfg)
    b = Generator(cfg, B, F)
    checkpoint.load_checkpoint(str(path), b, cfg)
    ma, va, sa, na = a.get_opt_state()
    mb, vb, sb, nb = b.get_opt_state()
    assert sa == sb == 2 and na == nb
    assert np.array_equal(ma, mb) and np.array_equal(va, vb)
    assert np.array_equal(a.get_params(), b.get_params())
    step = inputs(cfg, B, F, 20)
    a.train_step(*step, noise_stream=7)
    b.train_step(*step, noise_stream=7)
    assert np.array_equal(a.get_params(), b.get_params())
    a.close()
    b.close()
