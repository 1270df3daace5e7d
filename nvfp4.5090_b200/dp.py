"""Data-parallel plumbing of the NVFP4 MLP training step.

The token dimension is sharded across ranks (one process per GPU); weights
are replicated and every rank re-quantizes the same bf16 weights, so the only
exchange is the bf16 weight-gradient all-reduce.  It runs over NCCL (NVLink /
NVSwitch) through torch.distributed, one bucket per MLP block, launched as
soon as that block's wgrad GEMMs are enqueued so the transfer overlaps the
backward of the blocks below.  The reference has no distributed code; this
module is new.
"""
from __future__ import annotations

import datetime
import os
from typing import Dict, Hashable, Optional

import torch
import torch.distributed as dist


def init_from_env(backend: str = "nccl", timeout_s: float = 300.0):
    """Initialise the default process group from RANK / WORLD_SIZE / MASTER_* (torchrun).

    Returns (world, rank, local_rank).  A short timeout makes ranks whose peer
    died end their next collective with an error instead of waiting forever."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local


class BucketAllReducer:
    """One asynchronous SUM all-reduce per gradient bucket.

    ``launch`` enqueues the collective after the work already on the current
    stream (torch's NCCL process group orders it after the producing kernels);
    ``wait`` makes the current stream wait for it (no host synchronisation)."""

    def __init__(self, process_group=None):
        self.pg = process_group
        self.world = dist.get_world_size(process_group) if (process_group is not None or dist.is_initialized()) else 1
        self.works: Dict[Hashable, object] = {}

    @property
    def active(self) -> bool:
        return self.world > 1

    def launch(self, key: Hashable, bucket: torch.Tensor) -> None:
        if not self.active:
            return
        if key in self.works:
            raise RuntimeError(f"bucket {key!r} already in flight")
        self.works[key] = dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=self.pg, async_op=True)

    def wait(self, key: Hashable, timeout_s: Optional[float] = None) -> None:
        """Wait for one bucket; with ``timeout_s`` the host blocks at most that
        long and a collective that cannot complete (a dead peer) raises."""
        w = self.works.pop(key, None)
        if w is None:
            return
        if timeout_s is None:
            w.wait()
        else:
            w.wait(timeout=datetime.timedelta(seconds=timeout_s))

    def wait_all(self) -> None:
        for k in list(self.works):
            self.wait(k)

    def grad_scale(self) -> float:
        """Factor that turns the summed gradient into the mean over ranks."""
        return 1.0 / self.world
