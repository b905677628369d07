"""fp64 restatement of the RVC GAN losses — TEST INFRASTRUCTURE (the oracle of the discriminator
path).  Only tests/, the smoke check and bench.py's CPU baseline may import it; the product path
(wuburvc_b200/) never does.

What it restates (upstream RVC, knowledge/rvc_original/):
  * MultiPeriodDiscriminator (infer/module/models.py:928-951): DiscriminatorS followed by one
    DiscriminatorP per period [2, 3, 5, 7, 11, 17]; V2 (models.py:954-978) adds 23 and 37.
  * DiscriminatorS (models.py:981-1011): Conv1d 1->16 k15; grouped Conv1d k41 s4 (groups 4, 16,
    64, 256); Conv1d 1024->1024 k5; conv_post 1024->1 k3; LeakyReLU 0.1 after every conv but
    conv_post; every conv weight-normed (weight_norm, use_spectral_norm False).
  * DiscriminatorP (models.py:1014-1094): right reflect-pad to a multiple of the period, view
    [B, 1, T/p, p], Conv2d (5, 1) stride (3, 1) 1->32->128->512->1024, Conv2d (5, 1) stride 1
    1024->1024, conv_post (3, 1); a (k, 1) Conv2d is a Conv1d along time applied to each of the p
    columns on its own, which is how it is computed here.
  * discriminator_loss, generator_loss, feature_loss (train/losses.py:4-40).
  * the step order of train/train.py:500-525: the discriminator's loss on (real, generated
    detached), its AdamW step, then the generator's adversarial + feature-matching loss through
    the UPDATED discriminator, feature maps of the real half detached.
  * torch.optim.AdamW (train/train.py:230-235, default weight decay 0.01): decoupled decay, then
    the bias-corrected Adam update.

Pinned by tests/golden/gan_upstream.npz (tests/golden/make_gan_golden.py runs the upstream modules).
"""
from __future__ import annotations

from collections import OrderedDict

import numpy as np

from oracle.generator_ref import _name_stream, counter_normal, counter_uniform_pair

SLOPE = 0.1
PERIODS_V1 = (2, 3, 5, 7, 11, 17)
PERIODS_V2 = (2, 3, 5, 7, 11, 17, 23, 37)

# (C_in, C_out, k, stride, groups, pad) of DiscriminatorS's convs, then its conv_post
S_LAYERS = [(1, 16, 15, 1, 1, 7), (16, 64, 41, 4, 4, 20), (64, 256, 41, 4, 16, 20),
            (256, 1024, 41, 4, 64, 20), (1024, 1024, 41, 4, 256, 20), (1024, 1024, 5, 1, 1, 2),
            (1024, 1, 3, 1, 1, 1)]
# DiscriminatorP's (5, 1) convs (get_padding(5, 1) = 2), then its (3, 1) conv_post
P_LAYERS = [(1, 32, 5, 3, 1, 2), (32, 128, 5, 3, 1, 2), (128, 512, 5, 3, 1, 2), (512, 1024, 5, 3, 1, 2),
            (1024, 1024, 5, 1, 1, 2), (1024, 1, 3, 1, 1, 1)]


def discriminators(periods=PERIODS_V1):
    """[(period or 0 for DiscriminatorS, layers)] in upstream's order."""
    return [(0, S_LAYERS)] + [(p, P_LAYERS) for p in periods]


def layer_name(d, li, n_layers):
    return f"discriminators.{d}." + ("conv_post" if li == n_layers - 1 else f"convs.{li}")


def param_shapes(periods=PERIODS_V1):
    """Flat tensors in upstream's state_dict order: per conv bias [C_out], weight_g [C_out],
    weight_v [C_out, C_in/groups, k]."""
    S = OrderedDict()
    for d, (_, layers) in enumerate(discriminators(periods)):
        for li, (ci, co, k, _s, grp, _pad) in enumerate(layers):
            n = layer_name(d, li, len(layers))
            S[n + ".bias"] = (co,)
            S[n + ".weight_g"] = (co,)
            S[n + ".weight_v"] = (co, ci // grp, k)
    return S


def init_params(periods=PERIODS_V1, seed=3, bias_std=0.01):
    """v ~ N(0, 1/fan_in) per tensor (counter generator, stream keyed by the name); g = ||v|| per
    output channel times (1 + 0.2 u), u uniform in (-0.5, 0.5]; bias ~ N(0, bias_std)."""
    P = OrderedDict()
    for name, shp in param_shapes(periods).items():
        st = _name_stream(name)
        n = int(np.prod(shp))
        if name.endswith(".weight_v"):
            fan_in = shp[1] * shp[2]
            P[name] = (counter_normal(seed, st, n) / np.sqrt(fan_in)).reshape(shp).astype(np.float32)
        elif name.endswith(".bias"):
            P[name] = (bias_std * counter_normal(seed, st, n)).astype(np.float32)
    for name in list(param_shapes(periods)):
        if name.endswith(".weight_g"):
            v = P[name[:-1] + "v"].astype(np.float64)
            u, _ = counter_uniform_pair(seed, _name_stream(name), np.arange(v.shape[0], dtype=np.uint64))
            P[name] = (np.sqrt((v.reshape(v.shape[0], -1) ** 2).sum(1)) * (1 + 0.2 * (u - 0.5))).astype(np.float32)
    return OrderedDict((n, P[n]) for n in param_shapes(periods))


def _torch():
    import torch
    return torch


def _weight(P, n):
    torch = _torch()
    v = P[n + ".weight_v"]
    g = P[n + ".weight_g"]
    norm = torch.sqrt((v.reshape(v.shape[0], -1) ** 2).sum(1))
    return v * (g / norm).reshape(-1, 1, 1)


def disc_forward(P, x, period, layers, d):
    """One discriminator on x [B, T] -> (logits [B, n], fmaps).  fmaps of DiscriminatorP are
    [B, C, H, p] like upstream's Conv2d outputs."""
    torch = _torch()
    F = torch.nn.functional
    B, T = x.shape
    if period:
        if T % period:
            x = F.pad(x[:, None], (0, period - T % period), "reflect")[:, 0]
        H = x.shape[1] // period
        # column w of item b is the sequence x[b, w::p]; sequences ordered (b, w)
        h = x.reshape(B, H, period).permute(0, 2, 1).reshape(B * period, 1, H)
    else:
        h = x[:, None]
    fmaps = []
    for li, (_ci, _co, k, s, grp, pad) in enumerate(layers):
        n = layer_name(d, li, len(layers))
        h = F.conv1d(h, _weight(P, n), P[n + ".bias"], stride=s, padding=pad, groups=grp)
        if li < len(layers) - 1:
            h = F.leaky_relu(h, SLOPE)
        if period:
            C, L = h.shape[1], h.shape[2]
            fmaps.append(h.reshape(B, period, C, L).permute(0, 2, 3, 1))
        else:
            fmaps.append(h)
    out = fmaps[-1]
    return out.reshape(B, -1), fmaps


def mpd_forward(P, y, periods=PERIODS_V1):
    """MultiPeriodDiscriminator.forward on a batch: [(logits, fmaps)] per discriminator."""
    return [disc_forward(P, y, p, layers, d) for d, (p, layers) in enumerate(discriminators(periods))]


def discriminator_loss(dr, dg):
    return sum(((1 - a) ** 2).mean() + (b ** 2).mean() for a, b in zip(dr, dg))


def generator_loss(dg):
    return sum(((1 - b) ** 2).mean() for b in dg)


def feature_loss(fr, fg):
    return 2 * sum((a.detach() - b).abs().mean() for A, Bm in zip(fr, fg) for a, b in zip(A, Bm))


def _tensors(P, requires_grad=False, dtype=None):
    torch = _torch()
    dtype = dtype or torch.float64
    return OrderedDict((n, torch.tensor(np.asarray(v), dtype=dtype, requires_grad=requires_grad))
                       for n, v in P.items())


def d_step(P, y, y_hat, periods=PERIODS_V1, dtype=None):
    """The discriminator's loss on (real y, generated y_hat detached) and its gradient per
    parameter (flat float64 arrays).  dtype torch.float32 runs upstream's own fp32 arithmetic
    (the floor a fp32 implementation is measured against); the default is float64."""
    torch = _torch()
    dtype = dtype or torch.float64
    Pt = _tensors(P, True, dtype)
    yr = torch.tensor(np.asarray(y), dtype=dtype)
    yg = torch.tensor(np.asarray(y_hat), dtype=dtype)
    r = mpd_forward(Pt, yr, periods)
    g = mpd_forward(Pt, yg, periods)
    loss = discriminator_loss([a for a, _ in r], [a for a, _ in g])
    loss.backward()
    grads = OrderedDict((n, t.grad.double().numpy().reshape(-1).copy()) for n, t in Pt.items())
    logits = np.concatenate([a.detach().double().numpy().reshape(-1) for a, _ in r]
                            + [a.detach().double().numpy().reshape(-1) for a, _ in g])
    return float(loss.detach()), grads, logits


def g_step(P, y, y_hat, periods=PERIODS_V1, dtype=None):
    """generator_loss + feature_loss through the discriminator (real feature maps detached):
    (loss_gen, loss_fm, dL/dy_hat [B, T])."""
    torch = _torch()
    dtype = dtype or torch.float64
    Pt = _tensors(P, False, dtype)
    yr = torch.tensor(np.asarray(y), dtype=dtype)
    yg = torch.tensor(np.asarray(y_hat), dtype=dtype, requires_grad=True)
    r = mpd_forward(Pt, yr, periods)
    g = mpd_forward(Pt, yg, periods)
    lg = generator_loss([a for a, _ in g])
    lf = feature_loss([f for _, f in r], [f for _, f in g])
    (lg + lf).backward()
    return float(lg.detach()), float(lf.detach()), yg.grad.double().numpy().copy()


def adamw(P, grads, m, v, t, lr, betas, eps, wd):
    """torch.optim.AdamW (single tensor, amsgrad off) on flat float64 arrays; returns new P, m, v."""
    b1, b2 = betas
    out, mo, vo = OrderedDict(), OrderedDict(), OrderedDict()
    for n, p in P.items():
        p = np.asarray(p, np.float64).reshape(-1) * (1 - lr * wd)
        g = grads[n]
        mo[n] = b1 * m[n] + (1 - b1) * g
        vo[n] = b2 * v[n] + (1 - b2) * g * g
        bc1 = 1 - b1 ** t
        bc2 = 1 - b2 ** t
        denom = np.sqrt(vo[n]) / np.sqrt(bc2) + eps
        out[n] = (p - (lr / bc1) * mo[n] / denom).reshape(np.shape(P[n]))
    return out, mo, vo


def gan_step(P, y, y_hat, periods=PERIODS_V1, lr=1e-4, betas=(0.8, 0.99), eps=1e-9, wd=0.01):
    """One discriminator step then the generator-side gradient through the updated discriminator
    (train/train.py:500-525), from zero AdamW moments (t = 1)."""
    loss_d, grads, logits = d_step(P, y, y_hat, periods)
    zeros = OrderedDict((n, np.zeros(int(np.prod(np.shape(p))))) for n, p in P.items())
    P1, _, _ = adamw(P, grads, zeros, zeros, 1, lr, betas, eps, wd)
    loss_g, loss_fm, dy = g_step(P1, y, y_hat, periods)
    return dict(loss_d=loss_d, grads=grads, logits=logits, params_after=P1, loss_gen=loss_g,
                loss_fm=loss_fm, dldy_hat=dy)
