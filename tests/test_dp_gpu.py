"""Data-parallel MLP trainer on 2 GPUs (NCCL), skipped with fewer GPUs.

Two ranks each take half of a 512-token batch; the single-rank trainer runs
the same batch as two micro-batches of the same 256 tokens, so every global
scale of every GEMM operand is the same in both runs.  Three exchanges run:
ZeRO-1 with sharded weight quantization (rank-major buckets, NVFP4 weights
gathered), ZeRO-1 gathering bf16 parameters, and all-reduce, each with one
micro-batch per rank (wgrads written into the bf16 bucket) and two (fp32
accumulators copied into it).  Checks:

* all three give bit-identical fp32 master weights after two steps (a sum of
  two bf16 gradients does not depend on the collective; the AdamW update is
  element-wise) and bit-identical NVFP4 weights for the next step (codes,
  swizzled scales and global scales of both orientations), whether every
  rank quantized all weights or only its rows before the gather;
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
MODES = ("zero_sq", "zero_flat", "allreduce")
RUNS = [(m, T_LOCAL) for m in MODES] + [("zero_sq", T_LOCAL // 2), ("allreduce", T_LOCAL // 2)]   # (mode, micro)
QFIELDS = ("g_gu", "g_down", "q_gu", "s_gu", "q_down", "s_down", "q_gu_t", "s_gu_t", "q_down_t", "s_down_t")


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


def _worker(rank, world, port, mode, micro, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        mlp = _mlp()
        ops = sys.modules["nvfp4_b200"].ops
        x, dy = _batch(world)
        lo, hi = rank * T_LOCAL, (rank + 1) * T_LOCAL
        sq = {"zero_sq": True, "zero_flat": False, "allreduce": None}[mode]
        tr = mlp.NVFP4MLPStackTrainer(BLOCKS, D, F, seed=7, micro_tokens=micro, max_local_tokens=T_LOCAL,
                                      process_group=dist.group.WORLD, zero=mode != "allreduce", shard_quant=sq)
        assert (tr.layout is not None) == (mode == "zero_sq")
        p0 = [tuple(t.cpu() for t in m) for m in tr.gather_masters()]
        tr.step(x[lo:hi], dy[lo:hi])
        grads = [b.grad[:b.numel].clone() for b in tr.blocks] if mode == "allreduce" else None   # summed over ranks
        tr.step(x[lo:hi], dy[lo:hi])
        tr.finish()
        torch.cuda.synchronize()
        masters = [tuple(t.cpu() for t in m) for m in tr.gather_masters()]
        qws = []
        for i, b in enumerate(tr.blocks):   # the NVFP4 weights the next step would use
            if tr.layout is not None:
                q = tr.gathered[i].qweights(tr.w_g[i, 0:1], tr.w_g[i, 1:2])
                tr.gathered[i].ensure_transposed()
            else:
                q = mlp.quantize_weights(b.w_gu, b.w_down, g_gu=tr.w_g[i, 0:1], g_down=tr.w_g[i, 1:2])
            qws.append({k: getattr(q, k).cpu() for k in QFIELDS})
        # the global scales of the next step (shard amaxes, max over ranks) are the weights' own
        for i, (_, wgu, wdn) in enumerate(masters):
            assert torch.equal(tr.w_g[i, 0:1], ops.global_scale(wgu.cuda().to(torch.bfloat16)))
            assert torch.equal(tr.w_g[i, 1:2], ops.global_scale(wdn.cuda().to(torch.bfloat16)))
        torch.cuda.synchronize()
        if rank == 0:
            torch.save({"p0": p0, "masters": masters, "qws": qws,
                        "grads": None if grads is None else [g.cpu() for g in grads],
                        "device_error": ops.device_error()}, out_path)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_trainer_matches_single_rank(pkg, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    res = {}
    for mode, micro in RUNS:
        path = str(tmp_path / f"{mode}_{micro}.pt")
        mp.spawn(_worker, args=(world, _free_port(), mode, micro, path), nprocs=world, join=True)
        res[mode, micro] = torch.load(path)
        assert res[mode, micro]["device_error"] == 0
    for (mode, micro) in RUNS:
        if mode == "allreduce":
            continue
        ref = res["allreduce", micro]
        for a, b in zip(res[mode, micro]["masters"], ref["masters"]):
            for x, y in zip(a, b):
                assert torch.equal(x.view(torch.int32), y.view(torch.int32)), (mode, micro)
        for qa, qb in zip(res[mode, micro]["qws"], ref["qws"]):
            for k in QFIELDS:
                assert torch.equal(qa[k], qb[k]), (mode, micro, k)
    ref = res["allreduce", T_LOCAL]

    mlp = _mlp()
    x, dy = _batch(world)
    single = mlp.NVFP4MLPStackTrainer(BLOCKS, D, F, seed=7, micro_tokens=T_LOCAL, max_local_tokens=world * T_LOCAL)
    for b, (gam, wgu, wdn) in zip(single.blocks, ref["p0"]):
        p = b.param[:b.numel].cpu().float()
        assert torch.equal(p, torch.cat([gam, wgu.flatten(), wdn.flatten()]))
    single.step(x, dy)
    # one rank with two micro-batches: the gradient is the fp32 accumulators
    g1 = [torch.cat([b.grad_gamma32, b.acc_gu.flatten(), b.acc_down.flatten()]).cpu() for b in single.blocks]
    single.step(x, dy)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    for gd, gs in zip(ref["grads"], g1):
        assert rel(gd, gs) < 1e-2
    for blk, md, p0 in zip(single.blocks, ref["masters"], ref["p0"]):
        ud = torch.cat([t.flatten() for t in md]) - torch.cat([t.flatten() for t in p0])
        us = blk.master[:blk.numel].cpu() - torch.cat([t.flatten() for t in p0])
        cos = torch.nn.functional.cosine_similarity(ud, us, dim=0).item()
        assert cos > 0.99
        agree = (torch.sign(ud) == torch.sign(us)).float().mean().item()
        assert agree > 0.99
