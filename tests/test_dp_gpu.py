"""Data parallelism on two GPUs (skipped with fewer): one child process per GPU, the library's NCCL
gradient all-reduce inside the step, the host liveness rendezvous of wuburvc_b200.dp.

* The all-reduced gradients of a step over 2 x B items (B per rank) equal one GPU's gradients over
  the same 2B items (rel-L2 <= 1e-5 per tensor: only the fp32 summation order differs), and both
  ranks hold the same parameters after AdamW.
* A rank that leaves between steps (with none of its kernels or collectives in flight) makes the
  other rank's next step raise PeerLost on the host before it launches anything.
NVLS is switched off (NCCL_NVLS_ENABLE=0), as for every multi-GPU failure test on this pool."""
import os
import socket
import time

import numpy as np
import pytest
import torch

from oracle import generator_ref as G

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")
B, F = 2, 8


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(cfg):
    from wuburvc_b200 import model

    T = F * model.hop(cfg)
    n = 2 * B
    z = G.counter_normal(41, 1, n * 192 * F).reshape(n, 192, F).astype(np.float32)
    g = G.counter_normal(41, 2, n * 256).reshape(n, 256).astype(np.float32)
    f0 = (G.counter_uniform_pair(41, 3, np.arange(n * F, dtype=np.uint64))[0] * 320 + 80).reshape(n, F)
    f0 = f0.astype(np.float32)
    dldy = G.counter_normal(41, 4, n * T).reshape(n, T).astype(np.float32)
    noise = G.counter_normal(41, 5, n * T * 9).reshape(n, T, 9).astype(np.float32)
    return z, f0, g, dldy, noise


def _worker(rank, world, port, scenario, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from wuburvc_b200 import Generator, flatten, model
    from wuburvc_b200.dp import DataParallel, PeerLost

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    log = []
    gen = None
    try:
        cfg = model.config("40k")
        P = flatten(cfg, G.init_params_ref(cfg, 3))
        z, f0, g, dldy, noise = _inputs(cfg)
        sl = slice(rank * B, (rank + 1) * B)
        gen = Generator(cfg, B, F, device=rank)
        gen.set_params(P)
        dp = DataParallel(gen, timeout_s=20)
        dp.attach()
        gen.set_comm_timeout(30)
        if scenario == "equal":
            dp.step(z[sl], f0[sl], g[sl], noise[sl], dldy[sl], noise_stream=1)
            np.save(os.path.join(out_dir, f"grads{rank}.npy"), gen.get_grads())
            np.save(os.path.join(out_dir, f"params{rank}.npy"), gen.get_params())
            log.append("stepped")
        else:  # rank 1 leaves after the first step
            dp.step(z[sl], f0[sl], g[sl], noise[sl], dldy[sl], noise_stream=1)
            log.append("step0")
            if rank == 1:
                log.append("left")
                return
            t0 = time.monotonic()
            try:
                dp.step(z[sl], f0[sl], g[sl], noise[sl], dldy[sl], noise_stream=2)
                log.append("step1")
            except PeerLost:
                log.append(f"lost {time.monotonic() - t0:.1f}")
    finally:
        if gen is not None:
            gen.close()
        with open(os.path.join(out_dir, f"log{rank}"), "w") as f:
            f.write("\n".join(log))


def _run(tmp_path, scenario):
    import torch.multiprocessing as mp

    ctx = mp.start_processes(_worker, args=(2, _free_port(), scenario, str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    deadline = time.monotonic() + 300
    while not ctx.join(timeout=2):
        assert time.monotonic() < deadline, "ranks did not finish"
    return [(tmp_path / f"log{r}").read_text().splitlines() for r in range(2)]


@needs_two
def test_two_rank_step_equals_one_gpu_over_the_union_batch(tmp_path):
    from wuburvc_b200 import Generator, flatten, model, unflatten

    logs = _run(tmp_path, "equal")
    assert logs == [["stepped"], ["stepped"]]
    cfg = model.config("40k")
    P = flatten(cfg, G.init_params_ref(cfg, 3))
    z, f0, g, dldy, noise = _inputs(cfg)
    one = Generator(cfg, 2 * B, F, device=0)
    one.set_params(P)
    one.upload(z, f0, g, noise, dldy)
    one.forward(noise_stream=1)
    one.backward()
    want = unflatten(cfg, one.get_grads())
    one.close()
    g0 = unflatten(cfg, np.load(tmp_path / "grads0.npy"))
    g1 = np.load(tmp_path / "grads1.npy")
    assert np.array_equal(np.load(tmp_path / "grads0.npy"), g1)
    assert np.array_equal(np.load(tmp_path / "params0.npy"), np.load(tmp_path / "params1.npy"))
    worst = 0.0
    for n, w in want.items():
        if np.linalg.norm(w) == 0:
            continue
        e = np.linalg.norm(g0[n].astype(np.float64) - w) / np.linalg.norm(w)
        worst = max(worst, e)
        assert e <= 1e-5, (n, e)
    print(f"\n[dp2] all-reduced gradients vs one GPU over the union batch: worst rel-L2 {worst:.2e}")


@needs_two
def test_rank_leaving_between_steps_is_detected_before_the_next_launch(tmp_path):
    r0, r1 = _run(tmp_path, "leave")
    assert r1 == ["step0", "left"]
    assert r0[0] == "step0" and r0[1].startswith("lost")


def _disc_inputs():
    T = 2400
    y = (0.3 * G.counter_normal(43, 1, 4 * T).reshape(4, T)).astype(np.float32)
    y_hat = (0.5 * y + 0.2 * G.counter_normal(43, 2, 4 * T).reshape(4, T)).astype(np.float32)
    return y, y_hat


def _disc_worker(rank, world, port, out_dir):
    """One rank of the discriminators' data parallelism: 2 of the 4 items, gradient all-reduced and
    averaged before AdamW."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from oracle import gan_ref as D
    from wuburvc_b200 import Generator, gan

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    log = []
    d = None
    try:
        y, y_hat = _disc_inputs()
        sl = slice(2 * rank, 2 * rank + 2)
        d = gan.Discriminator(2, y.shape[1])
        d.set_params(gan.flatten(D.init_params(gan.PERIODS_V1, 3)))
        uid = [Generator.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        d.attach_comm(rank, world, uid[0], timeout_s=30)
        d.step(y[sl], y_hat[sl], update=False)
        np.save(os.path.join(out_dir, f"dgrads{rank}.npy"), d.get_grads())
        d.step(y[sl], y_hat[sl], update=True)
        np.save(os.path.join(out_dir, f"dparams{rank}.npy"), d.get_params())
        log.append("stepped")
    finally:
        if d is not None:
            d.close()
        with open(os.path.join(out_dir, f"dlog{rank}"), "w") as f:
            f.write("\n".join(log))


@needs_two
def test_discriminator_two_ranks_equal_one_gpu_over_the_union_batch(tmp_path):
    """The discriminators' averaged gradient over 2 ranks x 2 items equals one GPU's over the 4 items
    (each item's forward is computed identically, only the weight gradients' summation order
    differs: median rel-L2 <= 1e-6; per tensor <= 1e-4, as the weight-norm backward keeps only the
    part of dW orthogonal to v, which on the 5-entry rows of the first layers amplifies that
    rounding), and both ranks take the same AdamW step."""
    import torch.multiprocessing as mp

    from oracle import gan_ref as D
    from wuburvc_b200 import gan

    ctx = mp.start_processes(_disc_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    deadline = time.monotonic() + 300
    while not ctx.join(timeout=2):
        assert time.monotonic() < deadline, "ranks did not finish"
    logs = [(tmp_path / f"dlog{r}").read_text().splitlines() for r in range(2)]
    assert logs == [["stepped"], ["stepped"]]
    g0, g1 = np.load(tmp_path / "dgrads0.npy"), np.load(tmp_path / "dgrads1.npy")
    assert np.array_equal(g0, g1)
    assert np.array_equal(np.load(tmp_path / "dparams0.npy"), np.load(tmp_path / "dparams1.npy"))
    y, y_hat = _disc_inputs()
    one = gan.Discriminator(4, y.shape[1])
    one.set_params(gan.flatten(D.init_params(gan.PERIODS_V1, 3)))
    one.step(y, y_hat, update=False)
    want = gan.unflatten(one.get_grads())
    one.close()
    got = gan.unflatten(g0)
    errs = [float(np.linalg.norm(got[n].astype(np.float64) - w) / np.linalg.norm(w)) for n, w in want.items()]
    print(f"\n[dp2] discriminator gradients vs one GPU over the union batch: worst rel-L2 {max(errs):.2e}, "
          f"median {np.median(errs):.2e}")
    assert np.median(errs) <= 1e-6 and max(errs) <= 1e-4
