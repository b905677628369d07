"""Long-clip inference (40 kHz, batch 1, 6000 frames = 2.4M samples, forward only) checked through a
size-independent property: with an unvoiced clip and an explicit noise input the generator is a
local (finite receptive field) map, so the interior of the long clip's audio must equal the audio
of a short clip cut from the same inputs.  Both runs use the same kernels; only the placement of
an output row inside its tile or warp differs, which reorders a few fp32 sums (conv_post's
warp transpose-reduction, for one) — measured 2.4e-6 relative, hence the rel-L2 bound of 1e-5."""
import numpy as np
import pytest

from oracle import generator_ref as G
from wuburvc_b200 import Generator, flatten, model

pytestmark = pytest.mark.gpu


def test_long_clip_interior_equals_short_clip():
    cfg = model.config("40k")
    hop = model.hop(cfg)
    F, s0, Fs, margin = 6000, 2980, 64, 20
    P = flatten(cfg, G.init_params_ref(cfg, 6))
    z = G.counter_normal(8, 1, 192 * F).reshape(1, 192, F).astype(np.float32)
    g = G.counter_normal(8, 2, 256).reshape(1, 256).astype(np.float32)
    f0 = np.zeros((1, F), np.float32)
    noise = G.counter_normal(8, 3, F * hop * 9).reshape(1, F * hop, 9).astype(np.float32)
    long_gen = Generator(cfg, 1, F)
    long_gen.set_params(P)
    long_gen.upload(z, f0, g, noise, None)
    audio = long_gen.forward()
    long_gen.close()
    assert np.isfinite(audio).all()
    short = Generator(cfg, 1, Fs)
    short.set_params(P)
    short.upload(np.ascontiguousarray(z[:, :, s0:s0 + Fs]), f0[:, s0:s0 + Fs], g,
                 np.ascontiguousarray(noise[:, s0 * hop:(s0 + Fs) * hop]), None)
    a_short = short.forward()
    short.close()
    lo, hi = margin * hop, (Fs - margin) * hop
    got = audio[0, s0 * hop + lo:s0 * hop + hi].astype(np.float64)
    want = a_short[0, lo:hi].astype(np.float64)
    assert np.linalg.norm(got - want) <= 1e-5 * np.linalg.norm(want)
