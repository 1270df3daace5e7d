"""Data-parallel MLP trainer on 2 GPUs (NCCL), skipped with fewer GPUs.

Two ranks each take half of a 512-token batch; the single-rank trainer runs
the same batch as two micro-batches of the same 256 tokens, so every global
scale of every GEMM operand is the same in both runs.  Checks:

* ZeRO-1 (reduce-scatter, sharded AdamW with fp32 masters, all-gather) and
  the all-reduce path give bit-identical parameters after two steps (a sum of
  two bf16 gradients does not depend on the collective; the AdamW update is
  element-wise);
* the all-reduced gradient bucket equals the single-rank gradient (fp32
  accumulation of the two micro-batches) within two bf16 roundings
  (relative Frobenius error <= 1e-2);
* the fp32 master weights after two steps move as the single-rank ones do:
  cosine similarity of the updates > 0.99 and the same sign on > 99% of the
  weights (AdamW's first steps are close to lr * sign(g), so the few
  gradients that the bf16 exchange rounds across zero flip their update).
"""
import datetime
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
T_LOCAL, D, F, BLOCKS = 256, 256, 512, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batch(world):
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(world * T_LOCAL, D, device="cuda", generator=g).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(world * T_LOCAL, D, device="cuda", generator=g)).to(torch.bfloat16)
    return x, dy


def _mlp():
    sys.path.insert(0, ROOT)
    import __graft_entry__
    __graft_entry__.import_package()
    import importlib
    return importlib.import_module("nvfp4_b200.mlp")


def _worker(rank, world, port, zero, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        mlp = _mlp()
        x, dy = _batch(world)
        lo, hi = rank * T_LOCAL, (rank + 1) * T_LOCAL
        tr = mlp.NVFP4MLPStackTrainer(BLOCKS, D, F, seed=7, micro_tokens=T_LOCAL, max_local_tokens=T_LOCAL,
                                      process_group=dist.group.WORLD, zero=zero)
        p0 = [b.param[:b.numel].clone() for b in tr.blocks]
        tr.step(x[lo:hi], dy[lo:hi])
        grads = None if zero else [b.grad[:b.numel].clone() for b in tr.blocks]   # summed over ranks
        tr.step(x[lo:hi], dy[lo:hi])
        tr.finish()
        torch.cuda.synchronize()
        masters = None
        if not zero:
            masters = [b.master[:b.numel].cpu() for b in tr.blocks]
        else:   # gather the fp32 master shards
            masters = []
            for i, b in enumerate(tr.blocks):
                w = tr.opt.w[i]
                full = torch.empty(w.numel() * world, device="cuda", dtype=torch.float32)
                dist.all_gather_into_tensor(full, w)
                masters.append(full[:b.numel].cpu())
        # the weight global scales of the next step (shard amaxes, max over ranks) are the weights' own
        for i, b in enumerate(tr.blocks):
            assert torch.equal(tr.w_g[i, 0:1], sys.modules["nvfp4_b200"].ops.global_scale(b.w_gu))
            assert torch.equal(tr.w_g[i, 1:2], sys.modules["nvfp4_b200"].ops.global_scale(b.w_down))
        if rank == 0:
            torch.save({"params": [b.param[:b.numel].cpu() for b in tr.blocks], "p0": [p.cpu() for p in p0],
                        "grads": None if grads is None else [g.cpu() for g in grads], "masters": masters,
                        "device_error": sys.modules["nvfp4_b200"].ops.device_error()}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_trainer_matches_single_rank(pkg, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    res = {}
    for zero in (True, False):
        path = str(tmp_path / f"zero{int(zero)}.pt")
        mp.spawn(_worker, args=(world, _free_port(), zero, path), nprocs=world, join=True)
        res[zero] = torch.load(path)
        assert res[zero]["device_error"] == 0
    for a, b in zip(res[True]["params"], res[False]["params"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    for a, b in zip(res[True]["masters"], res[False]["masters"]):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))

    mlp = _mlp()
    x, dy = _batch(world)
    single = mlp.NVFP4MLPStackTrainer(BLOCKS, D, F, seed=7, micro_tokens=T_LOCAL, max_local_tokens=world * T_LOCAL)
    for b, p0 in zip(single.blocks, res[False]["p0"]):
        assert torch.equal(b.param[:b.numel].cpu().view(torch.int16), p0.view(torch.int16))
    single.step(x, dy)
    # one rank with two micro-batches: the gradient is the fp32 accumulators
    g1 = [torch.cat([b.grad_gamma32, b.acc_gu.flatten(), b.acc_down.flatten()]).cpu() for b in single.blocks]
    single.step(x, dy)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    for gd, gs in zip(res[False]["grads"], g1):
        assert rel(gd, gs) < 1e-2
    for blk, md, p0 in zip(single.blocks, res[False]["masters"], res[False]["p0"]):
        ud = md - p0.float()
        us = blk.master[:blk.numel].cpu() - p0.float()
        cos = torch.nn.functional.cosine_similarity(ud, us, dim=0).item()
        assert cos > 0.99
        agree = (torch.sign(ud) == torch.sign(us)).float().mean().item()
        assert agree > 0.99
