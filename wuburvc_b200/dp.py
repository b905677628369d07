"""Data parallelism, one process per GPU: the host side of the step.

The generator step all-reduces its gradients over NCCL inside the step (the library's communicator,
attached once).  A collective waits for every rank, so a rank that crashed or left between steps
would leave the others blocked in their next all-reduce.  ``DataParallel`` keeps that from
happening: before each step every rank announces the step in the process group's key-value store
and waits, for at most ``timeout_s``, until every peer has announced it too.  A peer that left, or
one later than the deadline, makes ``step`` raise ``PeerLost`` on the surviving ranks before any of
them launches the step, so no collective is ever entered without all ranks.  (The library's own
watchdog is the second line: a context with a communicator aborts it and returns
WUBU_B200_ERR_COMM when a step's collectives do not finish within its comm timeout.)

The communicator id travels over the same process group (rank 0 creates it).  The helper needs only
``torch.distributed`` for its store and one broadcast; the step itself is any object with
``attach_comm(rank, world, uid)`` and ``train_step(...)`` (``wuburvc_b200.Generator``).
"""
from __future__ import annotations

import datetime
from typing import Any, Callable, Optional

import torch.distributed as dist


class PeerLost(RuntimeError):
    """A rank did not reach a step within the deadline (it left, crashed or hangs)."""


def _default_store():
    # the store the default process group was created with (env:// or tcp:// rendezvous)
    from torch.distributed import distributed_c10d as c10d

    return c10d._get_default_store()


class DataParallel:
    def __init__(self, gen: Any, timeout_s: float = 60.0, store=None, group=None, prefix: str = "wubu_b200"):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed is not initialized")
        self.gen = gen
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.store = store if store is not None else _default_store()
        self.prefix = prefix
        self.steps = 0

    # ---- communicator ----
    def attach(self, unique_id: Optional[Callable[[], bytes]] = None):
        """Rank 0 creates the 128-byte NCCL id, every rank attaches it to its generator."""
        if self.world <= 1:
            return
        make = unique_id or type(self.gen).nccl_unique_id
        obj = [make() if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        self.gen.attach_comm(self.rank, self.world, obj[0])

    # ---- liveness ----
    def _key(self, phase: str, step: int, rank: int) -> str:
        return f"{self.prefix}/{phase}{step}/rank{rank}"

    def _announce_and_wait(self, phase: str):
        self.store.set(self._key(phase, self.steps, self.rank), b"1")
        peers = [self._key(phase, self.steps, r) for r in range(self.world) if r != self.rank]
        try:
            self.store.wait(peers, self.timeout)
        except Exception as e:  # the store reports a timeout (or a dead store) as an error
            missing = []
            for r in range(self.world):
                if r == self.rank:
                    continue
                try:
                    if not self.store.check([self._key(phase, self.steps, r)]):
                        missing.append(r)
                except Exception:
                    missing.append(r)
            raise PeerLost(f"rank(s) {missing or '?'} did not reach step {self.steps} ({phase}) within "
                           f"{self.timeout.total_seconds():.1f} s: {e}") from e

    def rendezvous(self):
        """Announces step `self.steps` and waits (bounded) until every peer has announced it, in two
        phases: a rank that gave up in the first ("arrive") never announces the second ("commit"),
        so a peer that arrived late cannot enter the step's collective alone."""
        if self.world <= 1:
            return
        self._announce_and_wait("arrive")
        self._announce_and_wait("commit")

    def step(self, *args, **kwargs):
        """The liveness rendezvous, then one training step (forward, backward, all-reduce, AdamW)."""
        self.rendezvous()
        out = self.gen.train_step(*args, **kwargs)
        self.steps += 1
        return out
