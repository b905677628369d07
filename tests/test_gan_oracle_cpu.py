"""The GAN oracle (oracle/gan_ref.py, fp64) against the upstream golden (tests/golden/gan_upstream.npz,
made by tests/golden/make_gan_golden.py from knowledge/rvc_original/infer/module/models.py:928-1094
and train/losses.py).  Upstream casts every loss term to float32 (losses.py:8-9, 21-22, 34), so the
golden carries float32 rounding in the losses; the tolerances below are a few float32 ulps."""
import os

import numpy as np
import pytest

from oracle import gan_ref as D

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "gan_upstream.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def step(gold):
    P = D.init_params(D.PERIODS_V1, int(gold["seed"]))
    return D.gan_step(P, gold["y"], gold["y_hat"], D.PERIODS_V1, lr=float(gold["lr"]),
                      betas=tuple(gold["betas"]), eps=float(gold["eps"]), wd=float(gold["wd"]))


def test_parameter_table_matches_upstream(gold):
    assert list(D.param_shapes(D.PERIODS_V1)) == [str(n) for n in gold["names"]]
    assert sum(int(np.prod(s)) for s in D.param_shapes(D.PERIODS_V1).values()) == 54968286


def test_logits_and_losses(gold, step):
    np.testing.assert_allclose(step["logits"], gold["logits"], rtol=1e-9, atol=1e-12)
    assert step["loss_d"] == pytest.approx(float(gold["loss_d"]), rel=1e-6)
    assert step["loss_gen"] == pytest.approx(float(gold["loss_gen"]), rel=1e-6)
    assert step["loss_fm"] == pytest.approx(float(gold["loss_fm"]), rel=1e-6)


def test_discriminator_gradients_and_adamw(gold, step):
    names = [str(n) for n in gold["names"]]
    offs = gold["offs"]
    for i, n in enumerate(names):
        g = step["grads"][n]
        assert np.linalg.norm(g) == pytest.approx(gold["gnorm"][i], rel=1e-6), n
        ix = gold["idx"][offs[i]:offs[i + 1]]
        np.testing.assert_allclose(g[ix], gold["gval"][offs[i]:offs[i + 1]], rtol=1e-5,
                                   atol=1e-6 * gold["gnorm"][i], err_msg=n)
        p = np.asarray(step["params_after"][n], np.float64).reshape(-1)
        np.testing.assert_allclose(p[ix], gold["pval"][offs[i]:offs[i + 1]], rtol=1e-9, atol=1e-12, err_msg=n)


def test_generator_side_gradient(gold, step):
    want = gold["dldy_hat"]
    got = step["dldy_hat"]
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-6


def test_generator_side_gradient_moves_at_fp32_resolution(gold):
    """dL/dy_hat is discontinuous where a generated feature ties with the real one (the sign of
    feature_loss) or a LeakyReLU input sits at 0: a relative change of 1e-7 in y_hat (fp32 rounding
    size) moves the fp64 result by ~5e-4 at this shape.  This is why the GPU check of dL/dy_hat
    (fp32) is gated at a few times that rather than at the continuous gradients' 1e-4."""
    from oracle import generator_ref as G

    P = D.init_params(D.PERIODS_V1, int(gold["seed"]))
    y, y_hat = gold["y"], gold["y_hat"]
    _, _, d0 = D.g_step(P, y, y_hat)
    eps = 1e-7 * G.counter_normal(99, 0, y_hat.size).reshape(y_hat.shape)
    _, _, d1 = D.g_step(P, y, y_hat * (1 + eps))
    moved = np.linalg.norm(d1 - d0) / np.linalg.norm(d0)
    assert 1e-5 < moved < 1e-3
