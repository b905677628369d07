"""Failure detection of the data-parallel host logic (wuburvc_b200/dp.py) on CPU gloo ranks: a rank
that leaves between steps, or arrives later than the deadline, makes the other ranks' next step
raise PeerLost within the deadline instead of blocking in the step's collective.  The step is a
stand-in whose collective is a gloo all-reduce (the GPU step's NCCL all-reduce waits the same way).
No GPU is involved: the failures are made on the host (a rank returns early, a rank sleeps)."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wuburvc_b200.dp import DataParallel, PeerLost

TIMEOUT = 2.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class FakeGen:
    """The step's collective without a GPU: every step all-reduces a small tensor."""

    def __init__(self):
        self.comm = None

    @staticmethod
    def nccl_unique_id():
        return bytes(range(128))

    def attach_comm(self, rank, world, uid):
        self.comm = (rank, world, uid)

    def train_step(self):
        t = torch.ones(4)
        dist.all_reduce(t)
        return float(t[0])


def _worker(rank, world, port, scenario, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = []
    try:
        gen = FakeGen()
        dp = DataParallel(gen, timeout_s=TIMEOUT)
        dp.attach()
        assert gen.comm == (rank, world, bytes(range(128)))
        for step in range(3):
            if rank == 1 and scenario == "leave" and step == 1:
                log.append("left")
                return
            if rank == 1 and scenario == "late" and step == 1:
                time.sleep(3 * TIMEOUT)
            t0 = time.monotonic()
            try:
                log.append(f"ok {dp.step()}")
            except PeerLost:
                log.append(f"lost {time.monotonic() - t0:.2f}")
                return
    finally:
        with open(os.path.join(out_dir, f"r{rank}"), "w") as f:
            f.write("\n".join(log))
        if scenario == "normal":
            dist.destroy_process_group()


def run(tmp_path, scenario):
    world = 2
    ctx = mp.start_processes(_worker, args=(world, _free_port(), scenario, str(tmp_path)), nprocs=world,
                             start_method="spawn", join=False)
    deadline = time.monotonic() + 60
    while not ctx.join(timeout=1):
        assert time.monotonic() < deadline, "ranks did not finish: a step blocked"
    return [(tmp_path / f"r{r}").read_text().splitlines() for r in range(world)]


def test_all_ranks_step_together(tmp_path):
    r0, r1 = run(tmp_path, "normal")
    assert r0 == r1 == ["ok 2.0"] * 3


def test_rank_that_leaves_between_steps(tmp_path):
    r0, r1 = run(tmp_path, "leave")
    assert r1 == ["ok 2.0", "left"]
    assert r0[0] == "ok 2.0" and r0[1].startswith("lost")
    assert float(r0[1].split()[1]) < TIMEOUT + 5  # within the deadline, not blocked in the collective


def test_rank_later_than_the_deadline(tmp_path):
    r0, r1 = run(tmp_path, "late")
    # rank 0 gives up waiting for rank 1's arrival; rank 1, arriving later, finds rank 0 never
    # committed the step and gives up too: neither enters the collective alone
    assert r0[0] == "ok 2.0" and r0[1].startswith("lost")
    assert r1[0] == "ok 2.0" and r1[1].startswith("lost")
