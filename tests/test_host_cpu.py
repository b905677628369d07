"""Host-side logic that needs no GPU: the native library loads and exports every symbol its
header declares, the parameter table matches the reference registry, init is deterministic."""
import os
import re

import numpy as np

from oracle import generator_ref as G
from wuburvc_b200 import flatten, init_params, model, param_table, param_total, unflatten
from wuburvc_b200._lib import LIB_PATH, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    txt = open(os.path.join(ROOT, "include", "wuburvc_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(wubu_b200_\w+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    assert os.path.exists(LIB_PATH)
    h = lib()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(h, n), n


def test_decoder_table_matches_reference_registry():
    """Same tensor set and sizes as wubu_train_registry_build (src/wubu_train.c:131-210):
    155 tensors / 14,327,424 floats for the 40 kHz decoder."""
    cfg = model.decoder_only("40k")
    t = param_table(cfg)
    assert len(t) == 155
    assert sum(x[4] for x in t) == 14327424
    ref = G.param_names(cfg)
    assert {x[0] for x in t} == set(ref)
    for name, kind, shape, off, n in t:
        assert n == int(np.prod(ref[name]))
        assert off % 64 == 0


def test_nsf_table_matches_upstream_generator():
    cfg = model.config("40k")
    t = param_table(cfg)
    assert sum(x[4] for x in t) == 14490890  # upstream GeneratorNSF with weight_norm, gin 256, 9 harmonics
    assert {x[0] for x in t} == set(G.param_names(cfg))
    snake = model.config("48k_snake")
    names = {x[0] for x in param_table(snake)}
    assert "dec.post_act.alpha" in names and "dec.resblocks.11.alpha2.2" in names


def test_table_order_is_backward_completion_order():
    cfg = model.config("40k")
    t = param_table(cfg)
    offs = {n: o for n, _, _, o, _ in t}
    assert offs["dec.conv_post.weight"] == 0
    assert offs["dec.ups.3.bias"] < offs["dec.resblocks.6.convs1.0.bias"] < offs["dec.ups.0.bias"]
    assert offs["dec.ups.0.bias"] < offs["dec.conv_pre.weight"] < offs["dec.m_source.l_linear.weight"]


def test_init_is_deterministic_and_weight_normed():
    cfg = model.config("40k")
    a = init_params(cfg, 0)
    b = init_params(cfg, 0)
    assert np.array_equal(a, b)
    named = unflatten(cfg, a)
    v = named["dec.resblocks.4.convs2.1.weight_v"]
    gg = named["dec.resblocks.4.convs2.1.weight_g"]
    np.testing.assert_allclose(gg.reshape(-1), np.linalg.norm(v.reshape(v.shape[0], -1), axis=1), rtol=1e-5)
    w = named["dec.conv_pre.weight"]
    assert abs(w.std() - 0.01) < 5e-4
    assert np.all(named["dec.ups.1.bias"] == 0)


def test_flatten_roundtrip():
    cfg = model.config("32k")
    P = G.init_params_ref(cfg, 3)
    flat = flatten(cfg, P)
    back = unflatten(cfg, flat)
    for k, v in P.items():
        np.testing.assert_array_equal(back[k].reshape(-1), v.reshape(-1))
    assert flat.size == param_total(cfg)


def test_training_flops_per_item():
    """Algorithmic FLOPs of one training item (forward + input and weight gradients of every
    convolution, 2 per multiply-add): 40 kHz at 32 frames, 32 kHz at 40, 48 kHz at 36."""
    assert abs(model.train_flops_per_item(model.config("40k"), 32) / 1e9 - 87.79) < 0.01
    assert abs(model.train_flops_per_item(model.config("32k"), 40) / 1e9 - 92.27) < 0.01
    assert abs(model.train_flops_per_item(model.config("48k"), 36) / 1e9 - 118.97) < 0.01


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks come before any device call (they run here, with no GPU)."""
    import ctypes

    from wuburvc_b200 import L

    h = lib()
    assert h.wubu_b200_stft_loss_grad(None, None, 1, 100, 3, None, None, None) == -1
    assert h.wubu_b200_stft_loss_grad(1, 1, 0, 100, 3, 1, 1, None) == -1
    g = L()
    assert g.wubu_b200_gen_set_opt_state(None, None, None, 0, 0) == -1
    m = (ctypes.c_float * 4)()
    assert g.wubu_b200_gen_get_opt_state(None, m, m, None, None) == -1


def test_primitives_reject_bad_arguments_before_touching_the_device():
    """Null operands and non-positive sizes return WUBU_B200_ERR_ARG (-1) before any CUDA call, so
    this runs without a GPU.  (A null operand would otherwise become a tensor map at address 0.)"""
    import ctypes

    h = lib()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    # split mode needs the lo halves
    assert h.wubu_b200_conv1d(p, None, p, None, None, p, 1, 32, 16, 32, 3, 1, 1, 1, None) == -1
    assert h.wubu_b200_conv1d(None, None, p, None, None, p, 1, 32, 16, 32, 3, 1, 1, 0, None) == -1
    assert h.wubu_b200_conv1d(p, None, p, None, None, p, 0, 32, 16, 32, 3, 1, 1, 0, None) == -1
    assert h.wubu_b200_conv1d_wgrad(p, None, p, 1, 32, 16, 32, 3, 1, 1, None) == -1
    assert h.wubu_b200_conv1d_wgrad_noalloc(p, p, None, 1, 32, 16, 32, 3, 1, 1, None) == -1
    assert h.wubu_b200_convT(p, p, p, None, None, p, 1, 64, 8, 32, 4, 2, 1, 1, None) == -1
    assert h.wubu_b200_convT_dgrad(p, p, p, 1, 64, 8, 32, 0, 2, 1, None) == -1
    assert h.wubu_b200_convT_wgrad(p, None, p, 1, 64, 8, 32, 4, 2, 1, None) == -1


def test_precision_option_is_checked_before_any_device_call():
    """The options struct carries the precision enum at the end (the header's layout), and both the
    Python constructor and wubu_b200_gen_create refuse an unknown value without touching a device."""
    import ctypes

    import pytest

    from wuburvc_b200 import PRECISIONS, GenConfig, Generator, L, TrainOptions

    assert PRECISIONS == {"bf16": 0, "fp32": 1}
    assert [f[0] for f in TrainOptions._fields_][-1] == "precision"
    hdr = open(os.path.join(ROOT, "include", "wuburvc_b200.h")).read()
    assert "WUBU_B200_PRECISION_BF16 = 0" in hdr and "WUBU_B200_PRECISION_FP32 = 1" in hdr
    with pytest.raises(ValueError):
        Generator(model.config("40k"), 1, 4, precision="tf32")
    c = GenConfig.from_dict(model.config("40k"))
    o = TrainOptions()
    o.batch, o.frames, o.precision = 1, 4, 7
    assert not L().wubu_b200_gen_create(ctypes.byref(c), ctypes.byref(o))


def test_discriminator_table_and_argument_checks_without_a_gpu():
    """The discriminators' parameter table is upstream's state_dict (MultiPeriodDiscriminator and
    V2, models.py:928-978) and every entry point checks its arguments before a device call."""
    import ctypes

    from oracle import gan_ref
    from wuburvc_b200 import gan

    for per in (gan.PERIODS_V1, gan.PERIODS_V2):
        t = gan.param_table(per)
        assert list(t) == list(gan_ref.param_shapes(per))
        assert all(tuple(s) == tuple(gan_ref.param_shapes(per)[n]) for n, (_, s) in t.items())
    assert gan.param_total() == 54968286
    h = gan.L()
    bad = (ctypes.c_int * 1)(1)
    assert h.wubu_b200_disc_param_count(bad, 1) == -1
    assert h.wubu_b200_disc_param_total(bad, 1) == -1
    assert h.wubu_b200_disc_param_info(None, 0, 129, None, 0, None, None) == -1
    assert not h.wubu_b200_disc_create(0, 12800, None, 0, None)
    assert not h.wubu_b200_disc_create(1, 64, None, 0, None)
    assert h.wubu_b200_disc_step(None, None, None, 0, None) == -1
    assert h.wubu_b200_disc_gen_loss(None, None, None, None, 0, None) == -1
    assert h.wubu_b200_disc_set_adamw(None, 1e-4, 0.8, 0.99, 1e-9, 0.01) == -1
    assert h.wubu_b200_disc_sync(None) == -1
    assert h.wubu_b200_disc_launches(None) == -1
    assert h.wubu_b200_disc_n_params(None) == -1
    assert h.wubu_b200_disc_attach_comm(None, 0, 2, None) == -1
    assert h.wubu_b200_disc_set_comm_timeout_ms(None, 1000) == -1
