"""The GAN discriminators on the GPU (wuburvc_b200/csrc/disc.cu through wuburvc_b200/gan.py)
against the fp64 oracle (oracle/gan_ref.py, pinned to upstream by tests/test_gan_oracle_cpu.py).

fp32 throughout, like upstream's training: the gates are fp32-level.  Every discriminator
parameter's gradient (129 tensors) by rel-L2 against fp64, printed beside the error of upstream's
own fp32 arithmetic on the same tensor (the oracle run in torch.float32).  The median must stay at
fp32 rounding (2e-6); each tensor within 5e-3, because of LeakyReLU kinks: at a 12800-sample
segment each discriminator's 1024-channel layers hold 10-40 pre-activations closer to 0 than the
rounding of their 5120-term fp32 sums, so which of them change side depends on the summation order
alone (torch's CPU order and this library's differ), and one change moves the gradients of the
layers below it by up to ~3e-3.  Also
the losses, dL/dy_hat through the updated discriminators, and the AdamW update by its rel-L2 (a
first Adam step moves each parameter by about lr sign(g), so an entry whose gradient is at the fp32
noise floor may take the other sign).  dL/dy_hat is checked at the GPU's own updated weights, so
the check isolates the kernels from those sign choices; feature_loss's gradient 2 sign(g - r) / n
is discontinuous where a generated feature equals the real one, so its gate is also relative to
the sensitivity of the fp64 result itself to fp32-size changes of its input."""
import numpy as np
import pytest
import torch

from oracle import gan_ref as D
from oracle import generator_ref as G
from wuburvc_b200 import gan

pytestmark = pytest.mark.gpu

GRAD_MEDIAN_TOL = 2e-6  # median over the tensors of the per-tensor rel-L2, fp32 against fp64
GRAD_TOL = 5e-3         # every tensor (LeakyReLU kink changes, see above)
LOSS_TOL = 1e-5      # relative
# rel-L2 of dL/dy_hat: the function is discontinuous at fp32 resolution (feature_loss's sign terms,
# the LeakyReLU kinks) -- a 1e-7 relative change of y_hat moves the fp64 result by up to ~5e-4
# (tests/test_gan_oracle_cpu.py measures it) -- so the gate is a few times that
DLDY_TOL = 2e-3


def rel(a, b):
    a, b = np.asarray(a, np.float64).reshape(-1), np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def inputs(B, T, seed=41):
    y = 0.3 * G.counter_normal(seed, 1, B * T).reshape(B, T)
    y_hat = 0.5 * y + 0.2 * G.counter_normal(seed, 2, B * T).reshape(B, T)
    return y.astype(np.float32), y_hat.astype(np.float32)


def check_step(B, T, periods, seed=3):
    P = D.init_params(periods, seed)
    y, y_hat = inputs(B, T)
    want = D.gan_step(P, y, y_hat, periods)
    d = gan.Discriminator(B, T, periods)
    d.set_params(gan.flatten(P, periods))
    # gradients without the update
    loss_d = d.step(y, y_hat, update=False)
    assert loss_d == pytest.approx(want["loss_d"], rel=LOSS_TOL)
    grads = gan.unflatten(d.get_grads(), periods)
    _, g32, _ = D.d_step(P, y, y_hat, periods, dtype=torch.float32)
    errs = {n: rel(grads[n], want["grads"][n]) for n in want["grads"]}
    floor = {n: rel(g32[n], want["grads"][n]) for n in want["grads"]}
    worst = max(errs, key=errs.get)
    print(f"B={B} T={T} periods={periods}: grad rel-L2 max {errs[worst]:.2e} ({worst}; upstream fp32 "
          f"{floor[worst]:.2e}), median {np.median(list(errs.values())):.2e} (upstream fp32 "
          f"{np.median(list(floor.values())):.2e})")
    assert np.median(list(errs.values())) <= GRAD_MEDIAN_TOL
    for n in errs:
        assert errs[n] <= GRAD_TOL, (n, errs[n], floor[n])
    # the step with AdamW, then the generator side through the updated discriminators
    before = d.get_params()
    d.step(y, y_hat, update=True)
    after = d.get_params()
    want_after = gan.flatten(want["params_after"], periods)
    upd = rel(after.astype(np.float64) - before, want_after.astype(np.float64) - before)
    print(f"AdamW update rel-L2 {upd:.2e}")
    assert upd <= 1e-2
    lg, lf, dy = d.gen_loss(y, y_hat)
    # the generator side at the GPU's own updated weights (fp64, and upstream's fp32 for the floor)
    Pa = gan.unflatten(after, periods)
    wg, wf, wdy = D.g_step(Pa, y, y_hat, periods)
    _, _, dy32 = D.g_step(Pa, y, y_hat, periods, dtype=torch.float32)
    assert lg == pytest.approx(wg, rel=LOSS_TOL)
    assert lf == pytest.approx(wf, rel=LOSS_TOL)
    e, fl = rel(dy, wdy), rel(dy32, wdy)
    print(f"dL/dy_hat rel-L2 {e:.2e} (upstream fp32 {fl:.2e}); loss_gen {lg:.6f} ({wg:.6f}) loss_fm {lf:.6f} "
          f"({wf:.6f}); launches {d.launches()}")
    assert e <= DLDY_TOL
    d.close()


def test_gan_step_matches_oracle_golden_shape():
    """B = 2, T = 2400 (the upstream golden's shape: reflect padding at periods 7, 11, 17)."""
    check_step(2, 2400, gan.PERIODS_V1)


def test_gan_step_matches_oracle_one_training_segment():
    """One 40 kHz training segment (12800 samples = 32 frames of hop 400), the shape of every item
    of the benchmarked batch: every layer has several position tiles and deep weight-gradient
    splits."""
    check_step(1, 12800, gan.PERIODS_V1)


def test_gan_step_v2_periods():
    """MultiPeriodDiscriminatorV2's periods (23 and 37 added), T not a multiple of either."""
    check_step(1, 4001, gan.PERIODS_V2)


def test_results_are_deterministic():
    B, T = 4, 12800
    P = D.init_params(gan.PERIODS_V1, 5)
    y, y_hat = inputs(B, T, seed=7)
    d = gan.Discriminator(B, T)
    d.set_params(gan.flatten(P))
    l1 = d.step(y, y_hat, update=False)
    g1 = d.get_grads()
    l2 = d.step(y, y_hat, update=False)
    g2 = d.get_grads()
    assert l1 == l2 and np.array_equal(g1, g2)
    a = d.gen_loss(y, y_hat)
    b = d.gen_loss(y, y_hat)
    assert a[0] == b[0] and a[1] == b[1] and np.array_equal(a[2], b[2])
    d.close()


def test_batch_items_are_independent():
    """Item b's dL/dy_hat does not depend on the other items, and each item's is the B = 1 result
    (the losses are batch means, so the B-item gradient is the single-item one divided by B)."""
    B, T = 3, 6000
    P = gan.flatten(D.init_params(gan.PERIODS_V1, 5))
    y, y_hat = inputs(B, T, seed=9)
    d = gan.Discriminator(B, T)
    d.set_params(P)
    _, _, dy = d.gen_loss(y, y_hat)
    d.close()
    one = gan.Discriminator(1, T)
    one.set_params(P)
    for b in range(B):
        _, _, dy1 = one.gen_loss(y[b:b + 1], y_hat[b:b + 1])
        assert rel(dy[b] * B, dy1[0]) < 1e-5
    one.close()
