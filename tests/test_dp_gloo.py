"""Data-parallel host logic on CPU with gloo process groups of 2 and 4 ranks:
bucketed async all-reduce, mean-gradient scaling, the ZeRO-1 sharded
optimizer (reduce-scatter, shard update, all-gather) against the all-reduce
path, the gathers of sharded NVFP4 weights (GatheredWeights with the oracle
standing in for the GPU quantizer), and host-side failure detection (a rank
that dies before the collective)."""
import datetime
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _dp_module():
    sys.path.insert(0, ROOT)
    import __graft_entry__
    pkg = __graft_entry__.import_package()
    import importlib
    return importlib.import_module("nvfp4_b200.dp")


def _worker_reduce(rank, world, port, q):
    try:
        _init(rank, world, port, 30)
        dp = _dp_module()
        red = dp.BucketAllReducer(dist.group.WORLD)
        assert red.active and red.world == world
        buckets = {i: torch.full((1000 + i,), float(rank + 1) * (i + 1)) for i in range(4)}
        for i in reversed(range(4)):          # backward order: last block first
            red.launch(i, buckets[i])
        with pytest.raises(RuntimeError):
            red.launch(0, buckets[0])          # same bucket twice in flight
        for i in range(4):
            red.wait(i)
        expect = sum(r + 1 for r in range(world))
        for i in range(4):
            assert torch.allclose(buckets[i], torch.full_like(buckets[i], expect * (i + 1)))
            assert torch.allclose(buckets[i] * red.grad_scale(), torch.full_like(buckets[i], expect * (i + 1) / world))
        red.wait_all()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _adam_cpu(p, g, m, v, step=1, lr=1e-2, b1=0.9, b2=0.95, eps=1e-8, gscale=0.5):
    """Elementwise AdamW-like update on CPU tensors (p bf16, g bf16, m/v fp32), in place."""
    gf = g.float() * gscale
    m.mul_(b1).add_((1 - b1) * gf)
    v.mul_(b2).add_((1 - b2) * gf * gf)
    upd = (m / (1 - b1 ** step)) / ((v / (1 - b2 ** step)).sqrt() + eps)
    p.copy_((p.float() - lr * upd).to(p.dtype))


def _worker_sharded(rank, world, port, q):
    try:
        _init(rank, world, port, 30)
        dp = _dp_module()
        sizes = {0: 1001, 1: 37, 2: 4096}
        opt = dp.ShardedBucketOptimizer(dist.group.WORLD, sizes, "cpu")
        assert opt.world == world and opt.grad_scale() == 1.0 / world
        gen = torch.Generator().manual_seed(0)            # same initial parameters on every rank
        params = {k: torch.zeros(opt.padded_len(k), dtype=torch.bfloat16) for k in sizes}
        for k, n in sizes.items():
            params[k][:n] = torch.randn(n, generator=gen).to(torch.bfloat16)
        ref = {k: p.clone() for k, p in params.items()}
        ref_m = {k: torch.zeros(opt.padded_len(k)) for k in sizes}
        ref_v = {k: torch.zeros(opt.padded_len(k)) for k in sizes}
        for step in (1, 2):
            grads = {}
            for k, n in sizes.items():                   # rank-dependent gradients, zero padding
                gk = torch.zeros(opt.padded_len(k), dtype=torch.bfloat16)
                gk[:n] = (torch.arange(n, dtype=torch.float32) * 0.01 * (rank + 1) + step).to(torch.bfloat16)
                grads[k] = gk
            # reference: all-reduce the full bucket, update the full bucket
            for k in sizes:
                g_all = grads[k].clone()
                dist.all_reduce(g_all)
                _adam_cpu(ref[k], g_all, ref_m[k], ref_v[k], step=step)
            # sharded: reduce-scatter, shard update, all-gather (launched last block first)
            for k in reversed(list(sizes)):
                opt.reduce_scatter(k, grads[k])
            for k in reversed(list(sizes)):
                opt.update(k, params[k], lambda p, g, m, v: _adam_cpu(p, g, m, v, step=step))
            opt.wait_all()
            for k, n in sizes.items():
                assert torch.equal(params[k], ref[k]), (k, step)
                assert torch.all(params[k][n:] == 0)     # padding stays zero
        bad = torch.zeros(7, dtype=torch.bfloat16)
        try:
            opt.reduce_scatter(0, bad)
            raise AssertionError("wrong-length bucket accepted")
        except RuntimeError:
            pass
        opt.reduce_scatter(1, torch.zeros(opt.padded_len(1), dtype=torch.bfloat16))
        try:
            opt.reduce_scatter(1, torch.zeros(opt.padded_len(1), dtype=torch.bfloat16))
            raise AssertionError("second reduce-scatter of a bucket in flight accepted")
        except RuntimeError:
            pass
        opt.update(1, params[1], lambda p, g, m, v: None)
        opt.wait_all()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_gathered(rank, world, port, q):
    """Each rank quantizes its rows of a block's weights (rank-major bucket)
    through GatheredWeights.quantize, with the oracle in place of the GPU
    quantizer, and the real gathers assemble the full NVFP4 weights; every
    rank must then hold exactly the oracle's quantization of the whole
    matrices, in both orientations, and the whole gamma.  Two rounds with
    different weights check that the buffers and the permutation are redone."""
    try:
        _init(rank, world, port, 60)
        sys.path.insert(0, ROOT)
        import importlib

        import numpy as np

        import __graft_entry__
        from oracle import nvfp4_oracle as orc
        __graft_entry__.import_package()
        mlp = importlib.import_module("nvfp4_b200.mlp")

        def bits(t):
            return t.contiguous().view(torch.int16).numpy().view(np.uint16)

        def fake(transposed):
            def quantize(x, global_scale=None, out=None, **kw):
                assert not kw and out is not None
                xb = bits(x)
                qn, sn = orc.quant_nvfp4(np.ascontiguousarray(xb.T) if transposed else xb,
                                         np.float32(global_scale.item()))
                out[0].copy_(torch.from_numpy(qn))
                out[1].copy_(torch.from_numpy(sn).reshape(out[1].shape))
                return out
            return quantize

        mlp.ops.quantize, mlp.ops.quantize_t = fake(False), fake(True)
        d, f = {2: (256, 256), 3: (384, 192), 4: (512, 256)}[world]
        lay = mlp.ShardQuantLayout(d, f, world)
        gw = mlp.GatheredWeights(lay, "cpu")
        for rnd in range(2):
            gen = torch.Generator().manual_seed(11 + rnd)      # the same weights on every rank
            gamma = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16)
            w_gu = ((0.05 + rnd) * torch.randn(2 * f, d, generator=gen)).to(torch.bfloat16)
            w_down = ((0.05 + rnd) * torch.randn(d, f, generator=gen)).to(torch.bfloat16)
            full = torch.zeros(lay.shard * world, dtype=torch.bfloat16)
            lay.store(full, gamma, w_gu, w_down)
            param = torch.zeros_like(full)                     # only this rank's shard is present
            sl = slice(rank * lay.shard, (rank + 1) * lay.shard)
            param[sl] = full[sl]
            g_gu = orc.global_scale_of(orc.bf16_bits_to_f32(bits(w_gu)))
            g_dn = orc.global_scale_of(orc.bf16_bits_to_f32(bits(w_down)))
            tg_gu, tg_dn = torch.tensor([float(g_gu)]), torch.tensor([float(g_dn)])
            gw.quantize(rank, param, tg_gu, tg_dn)
            gw.gather_forward(rank, param, dist.group.WORLD)
            gw.gather_transposed(rank, dist.group.WORLD)
            qw = gw.qweights(tg_gu, tg_dn)
            assert torch.equal(gw.gamma, gamma), ("gamma", rnd)
            gw.ensure_transposed()
            for name, qq, ss, x, g in (("gu", qw.q_gu, qw.s_gu, bits(w_gu), g_gu),
                                       ("down", qw.q_down, qw.s_down, bits(w_down), g_dn),
                                       ("gu_t", qw.q_gu_t, qw.s_gu_t, np.ascontiguousarray(bits(w_gu).T), g_gu),
                                       ("down_t", qw.q_down_t, qw.s_down_t, np.ascontiguousarray(bits(w_down).T), g_dn)):
                oq, os_ = orc.quant_nvfp4(x, g)
                assert np.array_equal(qq.numpy(), oq), (name, rnd)
                assert np.array_equal(ss.numpy().reshape(-1), os_.reshape(-1)), (name, rnd)
            gw.wait()                                           # nothing left in flight
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _worker_failure(rank, world, port, q):
    try:
        _init(rank, world, port, 4)
        dp = _dp_module()
        red = dp.BucketAllReducer(dist.group.WORLD)
        if rank == 1:
            q.put((rank, "exiting"))
            q.close()
            q.join_thread()                  # flush the message before dying
            os._exit(3)                      # the failing rank dies between steps
        t = torch.ones(16)
        try:
            red.launch("blk", t)
            red.wait("blk", timeout_s=5)
            q.put((rank, "no error"))
        except Exception as e:               # detected on the host: connection closed / timeout
            q.put((rank, f"detected:{type(e).__name__}"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _run(target, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, msg = q.get(timeout=timeout)
        out[r] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_bucketed_allreduce(world):
    out = _run(_worker_reduce, world=world)
    assert out == {r: "ok" for r in range(world)}, out


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_optimizer_matches_allreduce(world):
    out = _run(_worker_sharded, world=world)
    assert out == {r: "ok" for r in range(world)}, out


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_nvfp4_weight_gathers(world):
    out = _run(_worker_gathered, world=world, timeout=120)
    assert out == {r: "ok" for r in range(world)}, out


def test_shard_len_pads_evenly():
    dp = _dp_module()
    for n in (1, 15, 16, 1001, 4096, 123457):
        for world in (1, 2, 3, 8):
            s = dp.shard_len(n, world)
            assert s % 16 == 0 and s * world >= n and (s - 16) * world < n


def test_rank_failure_is_detected_on_host():
    out = _run(_worker_failure)
    assert out[1] == "exiting"
    assert out[0].startswith("detected:"), out[0]


def test_single_process_reducer_is_noop():
    dp = _dp_module()
    red = dp.BucketAllReducer(None)
    assert not red.active and red.grad_scale() == 1.0
    t = torch.ones(4)
    red.launch(0, t)
    red.wait(0)
    assert torch.equal(t, torch.ones(4))
