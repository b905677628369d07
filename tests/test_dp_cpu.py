"""Data-parallel host logic on CPU: two gloo ranks (world_size 2).

The GPU step all-reduces the flat gradient buffer in the buckets of ``bucket_plan`` as the backward
finishes each stage (NCCL on the device).  Here the same plan drives a bucketed gloo all-reduce of a
flat buffer on each rank, which must equal one all-reduce of the whole buffer; the ranks must agree
on the plan; and the 128-byte communicator id that rank 0 broadcasts must reach every rank intact.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import wuburvc_b200 as wb
from wuburvc_b200 import model


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, cfg_name, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = model.config(cfg_name)
        plan = wb.bucket_plan(cfg)
        total = wb.param_total(cfg)
        # every rank computes the same plan
        flat_plan = torch.tensor([e for _, e in plan], dtype=torch.int64)
        gathered = [torch.zeros_like(flat_plan) for _ in range(world)]
        dist.all_gather(gathered, flat_plan)
        for g in gathered:
            assert torch.equal(g, flat_plan)
        # buckets tile [0, total) in order
        prev = 0
        for a, b in plan:
            assert a == prev and b >= a
            prev = b
        assert prev == total
        # bucketed all-reduce == whole-buffer all-reduce
        gen = np.random.default_rng(1234 + rank)
        grads = torch.from_numpy(gen.standard_normal(total).astype(np.float32))
        whole = grads.clone()
        dist.all_reduce(whole)
        for a, b in plan:
            if b > a:
                view = grads[a:b]
                dist.all_reduce(view)
        assert torch.equal(grads, whole)
        # the averaged gradient the optimizer sees (grad_scale = 1 / world)
        ref = sum(torch.from_numpy(np.random.default_rng(1234 + r).standard_normal(total).astype(np.float32))
                  for r in range(world))
        assert torch.allclose(grads / world, ref / world, rtol=0, atol=1e-5)
        # the 128-byte communicator id broadcast from rank 0
        payload = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            payload = torch.from_numpy(np.frombuffer(os.urandom(128), dtype=np.uint8).copy())
        dist.broadcast(payload, 0)
        blobs = [torch.zeros(128, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(blobs, payload)
        for bl in blobs:
            assert torch.equal(bl, blobs[0])
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write(str(len(plan)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg_name", ["40k", "48k_snake"])
def test_bucketed_allreduce_two_ranks(tmp_path, cfg_name):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), cfg_name, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        assert (tmp_path / f"ok{r}").read_text() == "5"
