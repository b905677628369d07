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


def test_long_voiced_clip_matches_oracle_on_a_window():
    """Config 4 (40 kHz, batch 1, 6000 frames = 2.4M samples, f0 ~ U(80,400) Hz median-filtered over 5
    frames, 20 % unvoiced) forward on the GPU, compared with the fp64 oracle on a window cut from the
    clip.  The sine source carries its phase over every earlier frame (the parallel phase scan), so
    the window's oracle starts from that carry: harmonic h of the window starts at phase
    (acc0 * (h + 1) + rand_ini[h]) mod 1, acc0 = sum of the earlier frames' carries (fp64).  The
    generator is otherwise local, so the window's interior (a margin of 20 frames on each side) must
    match: forward rel-L2 <= 2e-3 (measured ~1e-6)."""
    import torch

    cfg = model.config("40k")
    hop, sr, dim = model.hop(cfg), cfg["sr"], cfg["harmonic_num"] + 1
    F, s0, Fs, margin, stream = 6000, 4711, 64, 20, 5
    P = G.init_params_ref(cfg, 12)
    z = G.counter_normal(9, 1, 192 * F).reshape(1, 192, F).astype(np.float32)
    g = G.counter_normal(9, 2, 256).reshape(1, 256).astype(np.float32)
    idx = np.arange(F, dtype=np.uint64)
    f0 = G.counter_uniform_pair(9, 3, idx)[0] * 320 + 80
    pad = np.pad(f0, 2, mode="edge")
    f0 = np.median(np.stack([pad[i:i + F] for i in range(5)]), axis=0)
    f0[G.counter_uniform_pair(9, 4, idx)[0] < 0.2] = 0.0
    f0 = f0.astype(np.float32)[None]
    noise = G.counter_normal(0, stream, F * hop * dim).reshape(1, F * hop, dim).astype(np.float32)
    gen = Generator(cfg, 1, F, seed=0)
    gen.set_params(flatten(cfg, P))
    gen.upload(z, f0, g, noise, None)
    audio = gen.forward(noise_stream=stream)[0]
    gen.close()
    assert np.isfinite(audio).all()

    # carry into frame s0 (fp64, as the source forms it), folded into the window's initial phases
    x = f0[0, :s0].astype(np.float64) / sr * hop + 0.5
    acc0 = np.fmod(np.sum(np.fmod(x, 1.0) - 0.5), 1.0)
    ri = G.counter_rand_ini(0, stream, dim)
    ri_w = np.mod(acc0 * np.arange(1, dim + 1) + ri, 1.0)
    w = slice(s0, s0 + Fs)
    t = lambda a: torch.tensor(np.asarray(a, np.float64))
    with torch.no_grad():
        a64 = G.forward({k: t(v) for k, v in P.items()}, cfg, t(z[:, :, w]), t(f0[:, w]), t(g[:, :, None]),
                        t(noise[:, s0 * hop:(s0 + Fs) * hop]), t(ri_w)).numpy()[0, 0]
    lo, hi = margin * hop, (Fs - margin) * hop
    got = audio[s0 * hop + lo:s0 * hop + hi].astype(np.float64)
    want = a64[lo:hi]
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    print(f"\n[long voiced clip] window rel-L2 {err:.2e}")
    assert err <= 2e-3
