"""Data-parallel plumbing of the NVFP4 MLP training step.

The token dimension is sharded across ranks (one process per GPU).  The
weight gradients are exchanged over NCCL (NVLink / NVSwitch) through
torch.distributed with one bucket per MLP block, launched as soon as that
block's wgrad GEMMs are enqueued so the transfer overlaps the backward of
the blocks below.  Two schemes:

* ``BucketAllReducer``: SUM all-reduce of each gradient bucket; every rank
  then runs the full optimizer update.
* ``ShardedBucketOptimizer`` (ZeRO-1): reduce-scatter of each bucket, the
  optimizer update of this rank's 1/world shard only (optimizer state exists
  only for the shard), then an all-gather of the updated parameter shards.
  The per-step optimizer work and memory then fall as 1/world; the gathers
  are waited for lazily, right before a block's weights are next used.
  (``mlp.GatheredWeights`` goes one step further for the MLP trainer: each
  rank quantizes its shard's rows and the ranks all-gather NVFP4 weights
  instead of bf16 parameters.)

The reference has no distributed code; this module is new.
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


def shard_len(n: int, world: int, align: int = 16) -> int:
    """Per-rank shard length of an n-element flat bucket: buckets are padded to
    world * shard elements, shards are multiples of ``align`` elements (16
    elements keep every shard 32-byte aligned for bf16 and fp32 vectors)."""
    per = -(-n // world)
    return -(-per // align) * align


class ShardedBucketOptimizer:
    """ZeRO-1 over flat buckets (see the module docstring).

    ``sizes`` maps a bucket key to its element count.  Gradient and parameter
    buckets handed in must have ``padded_len(key)`` elements (the tail past
    the real size is padding that stays zero in the gradient).  ``update_fn(p,
    g, m, v)`` updates one shard in place: p is this rank's slice of the
    parameter bucket, g the reduce-scattered gradient sum, m/v the shard's
    optimizer state (fp32, zero-initialised).  With ``master_weights`` the
    shard also keeps an fp32 master copy of its parameters, taken from the
    parameter shard at the first update, and ``update_fn(p, g, m, v, w)``
    receives it as ``w``."""

    def __init__(self, process_group, sizes: Dict[Hashable, int], device, grad_dtype=torch.bfloat16,
                 master_weights: bool = False):
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.shard = {k: shard_len(n, self.world) for k, n in sizes.items()}
        self.grad_shard = {k: torch.zeros(s, device=device, dtype=grad_dtype) for k, s in self.shard.items()}
        self.m = {k: torch.zeros(s, device=device, dtype=torch.float32) for k, s in self.shard.items()}
        self.v = {k: torch.zeros(s, device=device, dtype=torch.float32) for k, s in self.shard.items()}
        self.master_weights = master_weights
        self.w: Dict[Hashable, torch.Tensor] = {}
        self.rs_works: Dict[Hashable, object] = {}
        self.ag_works: Dict[Hashable, object] = {}

    def padded_len(self, key: Hashable) -> int:
        return self.shard[key] * self.world

    def shard_slice(self, key: Hashable) -> slice:
        s = self.shard[key]
        return slice(self.rank * s, (self.rank + 1) * s)

    def reduce_scatter(self, key: Hashable, grad_full: torch.Tensor) -> None:
        if grad_full.numel() != self.padded_len(key):
            raise RuntimeError(f"bucket {key!r}: gradient has {grad_full.numel()} elements, "
                               f"expected the padded length {self.padded_len(key)}")
        if key in self.rs_works:
            raise RuntimeError(f"bucket {key!r} already in flight")
        self.rs_works[key] = dist.reduce_scatter_tensor(self.grad_shard[key], grad_full, op=dist.ReduceOp.SUM,
                                                        group=self.pg, async_op=True)

    def update(self, key: Hashable, param_full: torch.Tensor, update_fn, timeout_s: Optional[float] = None,
               gather: bool = True) -> None:
        """Wait for the bucket's reduce-scatter and update this rank's shard;
        with ``gather`` also start the all-gather of the updated parameters
        (otherwise call ``gather`` later, e.g. in the order the next forward
        needs the buckets)."""
        w = self.rs_works.pop(key, None)
        if w is None:
            raise RuntimeError(f"bucket {key!r}: no reduce-scatter in flight")
        if timeout_s is None:
            w.wait()
        else:
            w.wait(timeout=datetime.timedelta(seconds=timeout_s))
        if param_full.numel() != self.padded_len(key):
            raise RuntimeError(f"bucket {key!r}: parameters have {param_full.numel()} elements, "
                               f"expected the padded length {self.padded_len(key)}")
        p_shard = param_full[self.shard_slice(key)]
        if self.master_weights:
            w = self.w.get(key)
            if w is None:
                w = self.w[key] = p_shard.float()
            update_fn(p_shard, self.grad_shard[key], self.m[key], self.v[key], w)
        else:
            update_fn(p_shard, self.grad_shard[key], self.m[key], self.v[key])
        if gather:
            self.gather(key, param_full)

    def gather(self, key: Hashable, param_full: torch.Tensor) -> None:
        """Start the all-gather of every rank's updated shard into ``param_full``."""
        if key in self.ag_works:
            raise RuntimeError(f"bucket {key!r}: gather already in flight")
        p_shard = param_full[self.shard_slice(key)]
        self.ag_works[key] = dist.all_gather_into_tensor(param_full, p_shard, group=self.pg, async_op=True)

    def wait_params(self, key: Hashable, timeout_s: Optional[float] = None) -> None:
        """Make the current stream wait until the bucket's gathered parameters are in place."""
        w = self.ag_works.pop(key, None)
        if w is None:
            return
        if timeout_s is None:
            w.wait()
        else:
            w.wait(timeout=datetime.timedelta(seconds=timeout_s))

    def wait_all(self) -> None:
        for k in list(self.ag_works):
            self.wait_params(k)

    def grad_scale(self) -> float:
        """Factor that turns the summed gradient into the mean over ranks."""
        return 1.0 / self.world
