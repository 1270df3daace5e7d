#!/usr/bin/env python3
"""Benchmark of the NVFP4 B200 hot path (one JSON line on rank 0).

Headline (``value``): the standalone block-scaled GEMM M=N=K=8192 on
pre-quantized NVFP4 operands (seed 1, N(0,1) bf16 quantized with per-tensor
global scales), in TFLOP/s = 2*M*N*K / device time, summed over ranks.  The
GEMM does not shard: at N GPUs each rank runs its own replica (weak scaling).

Also reported in the same line:
  quant      fused RMSNorm -> NVFP4 on x [32768 x 4096] (seed 2; row scale
             log-uniform [0.1, 10], gamma 1+0.1 N(0,1)), GB/s of algorithmic
             bytes, global-scale path (stats + quantize) and the single-pass
             reference-semantics kernel, plus the transposed quantizer;
  mlp_block  one RMSNorm+SwiGLU block training step, 16384 tokens, d=4096,
             ff=14336 (seed 3), tokens/s;
  mlp_stack  8 blocks, d=8192, ff=28672, 65536 global tokens split across
             ranks, NCCL bf16 wgrad all-reduce overlapped with backward
             (seed 4), tokens/s (strong scaling), device time max over ranks.

``--impl reference`` times the reference path's CPU emulation (quantize,
dequantize, fp32 matmul: the oracle restatement of float4utils.py) on the
host cores for the same GEMM metric, one output tile per step.  All inputs
are seeded synthetic data.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "NVFP4 GEMM TFLOPS (% FP4 peak); quant GB/s (% HBM); MLP step tokens/s 1–8 GPU"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FP4_PER_BF16 = 4.0          # dense FP4 : dense BF16 tensor throughput on B200 (9 : 2.25 PF)
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def load_traffic(name):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(name)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


class Flusher:
    def __init__(self):
        import torch
        self.buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def __call__(self):
        self.buf.fill_(1)


def timed_launches(fn, iters, flush, stream=None):
    """Per-launch device times (ms) with an L2 flush before each launch."""
    import torch
    times = []
    for _ in range(iters):
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


# ---------------------------------------------------------------------------
# GEMM headline
# ---------------------------------------------------------------------------

def gemm_operands(pkg, m, n, k, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    ga = pkg.ops.global_scale(a)
    gb = pkg.ops.global_scale(b)
    qa, sa = pkg.ops.quantize(a, global_scale=ga)
    qb, sb = pkg.ops.quantize(b, global_scale=gb)
    del a, b
    return qa, sa, qb, sb, ga, gb


def bench_gemm(pkg, args, world, rank, peaks):
    import torch
    m = n = k = 8192
    flops = 2.0 * m * n * k
    qa, sa, qb, sb, ga, gb = gemm_operands(pkg, m, n, k, seed=1)
    out = torch.empty((m, n), device="cuda", dtype=torch.bfloat16)
    flush = Flusher()
    run = lambda: pkg.ops.gemm(qa, sa, qb, sb, scale_a=ga, scale_b=gb, out=out)
    gpu_index = torch.cuda.current_device()
    with ClockSampler(gpu_index) as clk:
        for _ in range(max(args.warmup, 3)):
            run()
        barrier(world)
        times = timed_launches(run, args.steps, flush)
        barrier(world)
        # keep the same launch running for >= 1 s so the 200 ms clock samples see it under load
        t_end = time.perf_counter() + (0.0 if args.no_clock_hold else 1.0)
        while time.perf_counter() < t_end:
            for _ in range(50):
                run()
            torch.cuda.synchronize()
    total_ms = sum(times)
    ms_max = max_over_ranks(total_ms, world)
    value = world * flops * args.steps / (ms_max * 1e-3) / 1e12
    per_launch_ms = total_ms / args.steps
    achieved = flops / (per_launch_ms * 1e-3) / 1e12
    hbm, bf16, bf16_sus, src = peaks
    fp4_peak = bf16 * FP4_PER_BF16
    traffic = load_traffic("nvfp4_gemm_8192")
    clocks = clk.summary()
    clocks["window"] = "warmup + timed launches + 1 s sustained repeat of the same GEMM launch"
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "clocks": clocks,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp4_peak, "traffic": traffic,
                     "peak_source": f"4 x {src} dense bf16 ({bf16:.1f} TF/s burst, MEASURED_PEAKS.json); "
                                    "FP4:BF16 dense tensor ratio 9:2.25",
                     "kernel": "nvfp4b200::gemm::nvfp4_gemm_kernel", "launch_ms": per_launch_ms},
        "gpu_launches_per_step": 1,
    }
    # on-box Blackwell library baseline: cuBLASLt through torch scaled_mm (float4utils.py:427-436)
    if rank == 0 and not args.no_cublas:
        try:
            import torch.nn.functional as F
            from torch.nn.functional import ScalingType, SwizzleType
            a4 = qa.view(torch.float4_e2m1fn_x2)
            b4 = qb.view(torch.float4_e2m1fn_x2)
            s_a = sa.view(torch.float8_e4m3fn)
            s_b = sb.view(torch.float8_e4m3fn)
            cub = lambda: F.scaled_mm(a4, b4.mT, s_a, ScalingType.BlockWise1x16, s_b, ScalingType.BlockWise1x16,
                                      swizzle_a=SwizzleType.SWIZZLE_32_4_4, swizzle_b=SwizzleType.SWIZZLE_32_4_4,
                                      output_dtype=torch.bfloat16, contraction_dim=(1, 0))
            for _ in range(3):
                cub()
            ct = timed_launches(cub, args.steps, flush)
            res["cublaslt_scaled_mm_tflops"] = flops / (sum(ct) / len(ct) * 1e-3) / 1e12
        except Exception as e:  # keep the bench line even if the library path is unavailable
            res["cublaslt_scaled_mm_tflops"] = None
            res["cublaslt_error"] = f"{type(e).__name__}: {str(e)[:160]}"
    # MXFP4 GEMM (cutlass_mm_fp4.cu:71-165: UE8M0 scales per 1x32 block), same shape, outside the headline
    if rank == 0:
        gm = torch.Generator(device="cuda").manual_seed(6)
        mqa = torch.randint(0, 256, (m, k // 2), dtype=torch.uint8, device="cuda", generator=gm)
        mqb = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=gm)
        msa = torch.randint(120, 135, pkg.ops.mx_scale_shape(m, k), dtype=torch.uint8, device="cuda", generator=gm)
        msb = torch.randint(120, 135, pkg.ops.mx_scale_shape(n, k), dtype=torch.uint8, device="cuda", generator=gm)
        mrun = lambda: pkg.ops.mxfp4_mm(mqa, msa, mqb, msb)
        for _ in range(3):
            mrun()
        mt = timed_launches(mrun, args.steps, flush)
        mtf = flops / (sum(mt) / len(mt) * 1e-3) / 1e12
        mx = {"tflops": mtf, "frac": mtf / fp4_peak, "unit": "TFLOP/s",
              "workload": "MXFP4 GEMM M=N=K=8192 (random E2M1, UE8M0 scales 2^-7..2^7, seed 6), L2 flushed"}
        if not args.no_cublas:
            try:
                import torch.nn.functional as F
                from torch.nn.functional import ScalingType, SwizzleType
                ma4, mb4 = mqa.view(torch.float4_e2m1fn_x2), mqb.view(torch.float4_e2m1fn_x2)
                ms_a, ms_b = msa.view(torch.float8_e8m0fnu), msb.view(torch.float8_e8m0fnu)
                mcub = lambda: F.scaled_mm(ma4, mb4.mT, ms_a, ScalingType.BlockWise1x32, ms_b,
                                           ScalingType.BlockWise1x32, swizzle_a=SwizzleType.SWIZZLE_32_4_4,
                                           swizzle_b=SwizzleType.SWIZZLE_32_4_4, output_dtype=torch.bfloat16,
                                           contraction_dim=(1, 0))
                for _ in range(3):
                    mcub()
                mct = timed_launches(mcub, args.steps, flush)
                mx["cublaslt_scaled_mm_tflops"] = flops / (sum(mct) / len(mct) * 1e-3) / 1e12
            except Exception as e:
                mx["cublaslt_scaled_mm_tflops"] = None
                mx["cublaslt_error"] = f"{type(e).__name__}: {str(e)[:160]}"
        res["mxfp4"] = mx
        del mqa, mqb, msa, msb
    # e2e through the reference-shaped C-ABI op with host buffers (pinned), H2D + D2H in the timed region
    hqa = qa.cpu().pin_memory()
    hqb = qb.cpu().pin_memory()
    hsa = sa.cpu().pin_memory()
    hsb = sb.cpu().pin_memory()
    # two device slots: step i + 1's inputs upload while step i computes and step i - 1's result downloads
    hout = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev = [(torch.empty_like(qa), torch.empty_like(qb), torch.empty_like(sa), torch.empty_like(sb),
            torch.empty((m, n), device="cuda", dtype=torch.bfloat16)) for _ in range(2)]
    scale = (ga * gb).reshape(())

    def upload(i, b):
        dqa, dqb, dsa, dsb, _ = dev[b]
        dqa.copy_(hqa, non_blocking=True)
        dqb.copy_(hqb, non_blocking=True)
        dsa.copy_(hsa, non_blocking=True)
        dsb.copy_(hsb, non_blocking=True)

    def compute(i, b):
        dqa, dqb, dsa, dsb, dout = dev[b]
        pkg.ops._lib.call("nvfp4b200_nvfp4_mm", dqa.data_ptr(), dqb.data_ptr(), dsa.data_ptr(), dsb.data_ptr(),
                          scale.data_ptr(), None, dout.data_ptr(), m, n, k,
                          torch.cuda.current_stream().cuda_stream)

    def download(i, b):
        hout[b].copy_(dev[b][4], non_blocking=True)

    pipelined_e2e(2, upload, compute, download)   # warm-up
    barrier(world)
    e2e_ms = max_over_ranks(pipelined_e2e(args.steps, upload, compute, download), world)
    out = dev[(args.steps - 1) % 2][4]
    h2d = qa.numel() + qb.numel() + sa.numel() + sb.numel()
    d2h = out.numel() * 2
    bw_in, bw_out = pcie_bandwidth(hout[0], dev[0][4])
    # with both directions overlapped, a step cannot be shorter than the slower direction's copy
    pcie_ms = max(h2d / (bw_in * 1e9), d2h / (bw_out * 1e9)) * 1e3
    # ... and both directions at once share the link and the host memory: one step's copies timed together
    both_ms = pcie_concurrent_ms([(hqa, dev[0][0]), (hqb, dev[0][1]), (hsa, dev[0][2]), (hsb, dev[0][3])],
                                 [(dev[1][4], hout[1])])
    res["e2e"] = {"value": world * flops * args.steps / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                  "path": "nvfp4b200_nvfp4_mm C ABI (gn_kernels::cutlass_sm120a_nvfp4_mm contract)",
                  "pipeline": PIPELINE_NOTE,
                  "pcie": {"h2d_gbps": bw_in, "d2h_gbps": bw_out, "bound_ms_per_step": pcie_ms,
                           "bound_tflops": world * flops / (pcie_ms * 1e-3) / 1e12,
                           "both_directions_ms_per_step": both_ms,
                           "both_directions_bound_tflops": world * flops / (both_ms * 1e-3) / 1e12,
                           "note": "pinned-copy bandwidth measured here, each direction alone (bound_*) and one "
                                   "step's uploads and download in flight together (both_directions_*), the "
                                   "ceiling of the pipelined e2e"}}
    # correctness spot check against float64 (a few elements)
    res["spot_check_max_rel_err"] = gemm_spot_check(qa, sa, qb, sb, out, ga, gb)
    # M sweep at N = K = 8192 (same B operand), ours and cuBLASLt, L2 flushed per launch
    if rank == 0 and not args.no_sweep:
        res["m_sweep"] = gemm_m_sweep(pkg, args, qb, sb, gb, flush, with_cublas=not args.no_cublas)
    return res


def gemm_m_sweep(pkg, args, qb, sb, gb, flush, with_cublas=True):
    import torch
    out = {}
    n, k = qb.shape[0], 2 * qb.shape[1]
    for m in (128, 1024, 16384):
        g = torch.Generator(device="cuda").manual_seed(100 + m)
        a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        ga = pkg.ops.global_scale(a)
        qa, sa = pkg.ops.quantize(a, global_scale=ga)
        del a
        d = torch.empty((m, n), device="cuda", dtype=torch.bfloat16)
        run = lambda: pkg.ops.gemm(qa, sa, qb, sb, scale_a=ga, scale_b=gb, out=d)
        for _ in range(3):
            run()
        t = timed_launches(run, max(args.steps, 5), flush)
        ms = sum(t) / len(t)
        row = {"M": m, "N": n, "K": k, "ms": ms, "tflops": 2.0 * m * n * k / (ms * 1e-3) / 1e12}
        if with_cublas:
            try:
                import torch.nn.functional as F
                from torch.nn.functional import ScalingType, SwizzleType
                cub = lambda: F.scaled_mm(qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2).mT,
                                          sa.view(torch.float8_e4m3fn), ScalingType.BlockWise1x16,
                                          sb.view(torch.float8_e4m3fn), ScalingType.BlockWise1x16,
                                          swizzle_a=SwizzleType.SWIZZLE_32_4_4, swizzle_b=SwizzleType.SWIZZLE_32_4_4,
                                          output_dtype=torch.bfloat16, contraction_dim=(1, 0))
                for _ in range(3):
                    cub()
                ct = timed_launches(cub, max(args.steps, 5), flush)
                row["cublaslt_tflops"] = 2.0 * m * n * k / (sum(ct) / len(ct) * 1e-3) / 1e12
            except Exception as e:  # keep the sweep even if the library path is unavailable
                row["cublaslt_error"] = f"{type(e).__name__}: {str(e)[:120]}"
        out[str(m)] = row
        del qa, sa, d
    return out


def gemm_spot_check(qa, sa, qb, sb, out, ga, gb):
    import numpy as np
    import torch
    from oracle import nvfp4_oracle as orc
    m, kh = qa.shape
    n = qb.shape[0]
    k = 2 * kh
    rows = torch.tensor([0, 1, m // 2, m - 1], device="cuda")
    cols = torch.tensor([0, 7, n // 3, n - 1], device="cuda")
    ca = orc.unswizzle_scales(sa.cpu().numpy(), m, k)[rows.cpu().numpy()]
    cb = orc.unswizzle_scales(sb.cpu().numpy(), n, k)[cols.cpu().numpy()]
    va = orc.e2m1_decode(orc.unpack_nibbles(qa[rows].cpu().numpy())).reshape(4, -1, 16) * orc.e4m3_decode(ca)[..., None]
    vb = orc.e2m1_decode(orc.unpack_nibbles(qb[cols].cpu().numpy())).reshape(4, -1, 16) * orc.e4m3_decode(cb)[..., None]
    ref = (va.reshape(4, k).astype(np.float64) @ vb.reshape(4, k).astype(np.float64).T) * float(ga.item() * gb.item())
    got = out[rows][:, cols].float().cpu().numpy()
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + 1e-3 * np.abs(ref).max())))


# ---------------------------------------------------------------------------
# quantizer (RMSNorm -> NVFP4) workload
# ---------------------------------------------------------------------------

def bench_quant(pkg, args, peaks):
    import torch
    from oracle.nvfp4_oracle import bytes_nvfp4_quant
    r, k = 32768, 4096
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(r, k, device="cuda", generator=g)
    rs = torch.exp(torch.empty(r, 1, device="cuda").uniform_(math.log(0.1), math.log(10.0), generator=g))
    x = (x * rs).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).to(torch.bfloat16)
    flush = Flusher()
    hbm = peaks[0]
    base = bytes_nvfp4_quant(r, k)                 # float4utils.py:534-538
    alg = base + k * 2 + r * 4                     # + gamma read + inv_rms write
    out = {}

    def timeit(fn):
        for _ in range(3):
            fn()
        t = timed_launches(fn, max(args.steps, 5), flush)
        return sum(t) / len(t)

    st = timeit(lambda: pkg.ops.rmsnorm_stats(x, 1e-6, gamma=gamma))
    inv, gs = pkg.ops.rmsnorm_stats(x, 1e-6, gamma=gamma)
    qt = timeit(lambda: pkg.ops.quantize(x, global_scale=gs, row_scale=inv, gamma=gamma))
    fused = timeit(lambda: pkg.ops.rmsnorm_quantize(x, 1e-6, gamma=gamma))
    plain = timeit(lambda: pkg.ops.quantize(x))
    trans = timeit(lambda: pkg.ops.quantize_t(x, global_scale=gs, row_scale=inv, gamma=gamma))
    gb = lambda nbytes, ms: nbytes / (ms * 1e-3) / 1e9
    # the global scale must be known before any block is encoded, so this path reads x twice:
    # its own HBM bound is hbm * alg / (alg + R*K*2)
    two_pass = hbm * alg / (alg + r * k * 2)
    out["rmsnorm_quant_global_scale"] = {
        "gbps": gb(alg, st + qt), "ms": st + qt, "stats_ms": st, "quant_ms": qt,
        "quant_kernel_gbps": gb(alg, qt), "frac_hbm": gb(alg, st + qt) / hbm,
        "two_pass_bound_gbps": two_pass, "frac_of_two_pass_bound": gb(alg, st + qt) / two_pass,
        "note": "algorithmic bytes R*K*2 + R*K/2 + scales + gamma + inv_rms; stats pass (inv_rms + amax) reads x once more"}
    out["rmsnorm_quant_single_pass"] = {"gbps": gb(alg, fused), "ms": fused, "frac_hbm": gb(alg, fused) / hbm,
                                        "roofline": {"bound": "hbm", "achieved": gb(alg, fused), "peak": hbm,
                                                     "unit": "GB/s", "frac": gb(alg, fused) / hbm,
                                                     "traffic": load_traffic("rmsnorm_quant_32768x4096")}}
    out["quant_plain"] = {"gbps": gb(base, plain), "ms": plain, "frac_hbm": gb(base, plain) / hbm}
    out["quant_transposed"] = {"gbps": gb(alg, trans), "ms": trans, "frac_hbm": gb(alg, trans) / hbm}
    out["workload"] = "x bf16 [32768 x 4096], gamma, eps 1e-6 (seed 2)"
    return out


# ---------------------------------------------------------------------------
# MLP training steps
# ---------------------------------------------------------------------------

def bench_mlp(pkg, args, world, rank, n_blocks, d, f, global_tokens, seed, pg=None, micro_tokens=16384,
              e2e_steps=None):
    import torch
    from nvfp4_b200.mlp import NVFP4MLPStackTrainer
    t_local = global_tokens // world
    trainer = NVFP4MLPStackTrainer(n_blocks, d, f, device="cuda", seed=seed, micro_tokens=micro_tokens,
                                   process_group=pg, max_local_tokens=t_local,
                                   comm_sms=getattr(args, "comm_sms", 0), zero=not getattr(args, "allreduce", False),
                                   shard_quant=False if getattr(args, "bf16_gather", False) else None)
    g = torch.Generator(device="cuda").manual_seed(seed * 1000 + rank)
    x = torch.randn(t_local, d, device="cuda", generator=g).to(torch.bfloat16)
    dy = (torch.randn(t_local, d, device="cuda", generator=g) * 1e-3).to(torch.bfloat16)
    for _ in range(max(args.warmup, 3)):
        trainer.step(x, dy)
    barrier(world)
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            r = trainer.step(x, dy)
        trainer.finish()   # the last step's parameter gathers (ZeRO-1 at N > 1)
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world) / args.steps
    flops = trainer.flops_per_step(global_tokens)
    res = {"tokens_per_s": global_tokens / (ms * 1e-3), "ms_per_step": ms, "tflops": flops / (ms * 1e-3) / 1e12,
           "flops_per_step": flops, "n_gpus": world, "tokens_global": global_tokens, "tokens_per_rank": t_local,
           "micro_tokens": micro_tokens, "clocks": clk.summary(), "finite": bool(torch.isfinite(r).all().item())}
    if world > 1:
        # under the power cap each GPU settles at its own clock; the step runs at the slowest
        own = res["clocks"].get("sm_mhz") or 0.0
        res["clocks"]["sm_mhz_min_over_ranks"] = -max_over_ranks(-float(own), world)
        res["clocks"]["sm_mhz_max_over_ranks"] = max_over_ranks(float(own), world)
        if trainer.layout is not None:
            res["exchange"] = ("ZeRO-1: reduce-scatter + sharded AdamW, each rank quantizes its rows of the "
                               "updated weights, all-gather of NVFP4 weights")
        elif trainer.opt is not None:
            res["exchange"] = "ZeRO-1: reduce-scatter + sharded AdamW + all-gather of bf16 parameters"
        else:
            res["exchange"] = "all-reduce + replicated AdamW"
        res["comm_sms"] = trainer.comm_sms
    # e2e through the public API: pinned host tokens + upstream grad copied in, step result read back
    hx = x.cpu().pin_memory()
    hdy = dy.cpu().pin_memory()
    hres = [torch.empty(1, dtype=torch.float32).pin_memory() for _ in range(2)]
    slots = [(torch.empty_like(x), torch.empty_like(dy)) for _ in range(2)]
    results = []   # step results stay referenced until the run ends (read on the download stream)

    def upload(i, b):
        slots[b][0].copy_(hx, non_blocking=True)
        slots[b][1].copy_(hdy, non_blocking=True)

    def compute(i, b):
        results.append(trainer.step(slots[b][0], slots[b][1]))

    def download(i, b):
        hres[b].copy_(results[i], non_blocking=True)

    n_e2e = max(2, e2e_steps if e2e_steps is not None else args.steps // 2)
    barrier(world)
    e2e_ms = max_over_ranks(pipelined_e2e(n_e2e, upload, compute, download, finish=trainer.finish), world) / n_e2e
    del results[:]
    res["e2e"] = {"value": global_tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                  "h2d_bytes_per_step": 2 * x.numel() * 2 * world, "d2h_bytes_per_step": 4 * world,
                  "pipeline": PIPELINE_NOTE}
    if getattr(args, "breakdown", False):   # every rank runs the profiled step (it holds collectives)
        # rank-major buckets with one micro-batch: each wgrad GEMM is one launch per rank's row block
        splits = world if (trainer.layout is not None and t_local <= micro_tokens) else 1
        bd = step_breakdown(trainer, x, dy, n_blocks, d, f, min(micro_tokens, t_local), wgrad_splits=splits)
        if world > 1:
            bd["exposed_comm_ms_max_over_ranks"] = max_over_ranks(bd.get("exposed_comm_ms", 0.0), world)
            # rank imbalance: a rank whose kernels finish early waits inside the next collective
            cb = bd.get("compute_busy_ms", 0.0)
            bd["compute_busy_ms_max_over_ranks"] = max_over_ranks(cb, world)
            bd["compute_busy_ms_min_over_ranks"] = -max_over_ranks(-cb, world)
        res["kernel_breakdown"] = bd
    del trainer
    torch.cuda.empty_cache()
    return res


def pcie_bandwidth(host_buf, dev_buf, reps: int = 5):
    """Pinned host <-> device copy bandwidth (GB/s, best of `reps`) for
    buffers of this size, H2D and D2H each alone."""
    import torch
    res = []
    for fn in (lambda: dev_buf.copy_(host_buf, non_blocking=True), lambda: host_buf.copy_(dev_buf, non_blocking=True)):
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        res.append(host_buf.numel() * host_buf.element_size() / (best * 1e-3) / 1e9)
    return res[0], res[1]


def pcie_concurrent_ms(h2d_pairs, d2h_pairs, reps: int = 5):
    """Device time (ms, best of `reps`) of one step's copies with both
    directions in flight at once: every (host, device) pair of h2d_pairs goes
    up on one stream while every (device, host) pair of d2h_pairs goes down
    on another, as in the pipelined e2e runs."""
    import torch
    cur = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        s_in.wait_event(e0)
        s_out.wait_event(e0)
        with torch.cuda.stream(s_in):
            for h, d in h2d_pairs:
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s_out):
            for d, h in d2h_pairs:
                h.copy_(d, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        e1.record(cur)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


PIPELINE_NOTE = ("every step uploads its inputs from pinned host memory and downloads its result inside the "
                 "timed region; step i + 1's upload and step i's download overlap step i's compute (two device "
                 "slots, one copy stream per direction, ordered by events)")


def pipelined_e2e(steps, upload, compute, download, finish=None):
    """Time `steps` end-to-end steps: upload(i, slot) copies step i's inputs
    host -> device on an upload stream, compute(i, slot) runs the step on the
    current stream, download(i, slot) copies its result device -> host on a
    download stream.  Two slots: step i + 1's upload overlaps step i's compute,
    and step i's download overlaps step i + 1.  Returns the device time (ms)
    from before the first upload to after the last download."""
    import torch
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_event(e0)

    def up(i):
        b = i % 2
        if i >= 2:
            s_in.wait_event(ev_comp[b])      # step i - 2 has finished with slot b
        with torch.cuda.stream(s_in):
            upload(i, b)
        ev_in[b].record(s_in)

    up(0)
    for i in range(steps):
        b = i % 2
        if i + 1 < steps:
            up(i + 1)
        comp.wait_event(ev_in[b])
        if i >= 2:
            comp.wait_event(ev_out[b])       # step i - 2's result has been read out of slot b
        compute(i, b)
        ev_comp[b].record(comp)
        s_out.wait_event(ev_comp[b])
        with torch.cuda.stream(s_out):
            download(i, b)
        ev_out[b].record(s_out)
    if finish is not None:
        finish()
    comp.wait_stream(s_out)
    comp.wait_stream(s_in)
    e1.record(comp)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def step_breakdown(trainer, x, dy, n_blocks, d, f, micro, wgrad_splits=1):
    """One extra training step under torch.profiler (CUPTI kernel records, the
    real overlap, outside every timed region): device time per kernel, and each
    NVFP4 GEMM launch attributed to its role by its place in the step's fixed
    launch order (per micro-batch: gate/up and down per block forward, then dh,
    dW_down, dxn and dW_gu per block backward).  With a process group the
    NCCL kernels are separated out.  The profiled step ends with ``finish()``,
    which waits for the parameter all-gathers of the next step; in a stream of
    steps those overlap the next forward, except the first bucket's, which
    block 0 waits for.  So: ``exposed_in_step_ms`` is the time between the
    first and the last compute kernel in which no compute kernel runs,
    ``trailing_nccl_ms`` the collectives after the last compute kernel, and
    ``exposed_comm_ms`` = exposed_in_step_ms + the first of those gathers
    (the steady-state exposure per step)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.step(x, dy)
        trainer.finish()
        torch.cuda.synchronize()
    ks = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                if e.device_type == torch.autograd.DeviceType.CUDA)
    return summarize_kernels(ks, n_blocks, d, f, micro, wgrad_splits)


def summarize_kernels(ks, n_blocks, d, f, micro, wgrad_splits=1):
    """step_breakdown's summary of one step's kernel records ``ks`` = sorted
    (start_us, end_us, name) tuples; each wgrad GEMM is ``wgrad_splits``
    launches (row blocks), whose times are summed per role occurrence."""
    import collections
    if not ks:
        return {"error": "no kernel records"}
    agg = collections.defaultdict(lambda: [0, 0.0])
    for a, b, n in ks:
        key = n.split("(")[0]
        agg[key][0] += 1
        agg[key][1] += (b - a) / 1e3
    gem = [(b - a) / 1e3 for a, b, n in ks if "nvfp4_gemm_kernel" in n]
    t = micro
    flop = {"fwd_gate_up_swiglu": 2 * t * 2 * f * d, "fwd_down": 2 * t * d * f, "bwd_dh_swiglu": 2 * t * f * d,
            "wgrad_down": 2 * d * f * t, "bwd_dxn": 2 * t * d * 2 * f, "wgrad_gate_up": 2 * 2 * f * d * t}
    # the step's fixed GEMM launch order per micro-batch: gate/up and down per
    # block forward, then dh, dW_down, dxn, dW_gu per block backward
    sp = max(1, int(wgrad_splits))
    order = ["fwd_gate_up_swiglu", "fwd_down"] * n_blocks + (
        ["bwd_dh_swiglu"] + ["wgrad_down"] * sp + ["bwd_dxn"] + ["wgrad_gate_up"] * sp) * n_blocks
    roles = collections.defaultdict(list)
    prev = None
    for i, ms in enumerate(gem):
        j = i % len(order)
        r = order[j]
        if sp > 1 and r.startswith("wgrad") and prev is not None and prev[0] == r and prev[1] == j - 1:
            roles[r][-1] += ms          # another row block of the same wgrad GEMM
        else:
            roles[r].append(ms)
        prev = (r, j)
    busy = sum(v[1] for v in agg.values())
    span = (ks[-1][1] - ks[0][0]) / 1e3
    # collectives: time during which only NCCL kernels (or nothing) run, i.e. the
    # span minus the union of all compute-kernel intervals
    comp = sorted((a, b) for a, b, n in ks if "nccl" not in n.lower())
    union, cur = 0.0, None
    for a, b in comp:
        if cur is None or a > cur[1]:
            if cur is not None:
                union += cur[1] - cur[0]
            cur = [a, b]
        else:
            cur[1] = max(cur[1], b)
    if cur is not None:
        union += cur[1] - cur[0]
    nccl_ms = sum((b - a) / 1e3 for a, b, n in ks if "nccl" in n.lower())
    c_first = comp[0][0] if comp else ks[0][0]
    c_last = max(b for a, b in comp) if comp else ks[-1][1]
    in_step = (c_last - c_first) / 1e3 - union / 1e3
    trailing = sorted((a, b, n) for a, b, n in ks if "nccl" in n.lower() and a >= c_last)
    trailing_ms = sum((b - a) / 1e3 for a, b, n in trailing)
    first_gather = next(((b - a) / 1e3 for a, b, n in trailing if "allgather" in n.lower()), 0.0)
    # the largest gaps between compute kernels: where the step waits, and for what
    t0 = ks[0][0]
    comp_named = sorted((a, b, n) for a, b, n in ks if "nccl" not in n.lower())
    gaps = []
    end_prev = comp_named[0][1] if comp_named else 0.0
    for a1, b1, n1 in comp_named[1:]:
        if a1 - end_prev > 200.0:   # > 0.2 ms without compute
            during = sorted({n.split("(")[0].split("<")[0] for a, b, n in ks if "nccl" in n.lower() and a < a1 and b > end_prev})
            gaps.append({"at_ms": round((end_prev - t0) / 1e3, 3), "ms": round((a1 - end_prev) / 1e3, 3),
                         "next_kernel": n1.split("(")[0][:60], "nccl_running": during})
        end_prev = max(end_prev, b1)
    gaps.sort(key=lambda g: -g["ms"])
    return {
        "span_ms": span, "kernel_busy_ms": busy, "launches": len(ks), "compute_busy_ms": union / 1e3,
        "nccl_kernel_ms": nccl_ms, "exposed_in_step_ms": in_step, "trailing_nccl_ms": trailing_ms,
        "first_trailing_gather_ms": first_gather, "exposed_comm_ms": in_step + first_gather,
        "span_minus_compute_ms": span - union / 1e3, "largest_gaps": gaps[:8],
        "kernels": [{"name": k, "launches": c, "ms": round(ms, 3), "share": round(ms / busy, 4)}
                    for k, (c, ms) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:16]],
        "gemm_roles": {r: {"launches": len(v), "mean_ms": round(sum(v) / len(v), 4),
                           "tflops": round(flop[r] / (sum(v) / len(v) * 1e-3) / 1e12, 1)} for r, v in roles.items()},
        "note": "one step under torch.profiler (CUPTI), after the timed steps; per-kernel device time with real overlap",
    }


# ---------------------------------------------------------------------------
# reference arm: CPU emulation on the host cores
# ---------------------------------------------------------------------------

CPU_GEMM_ROWS, CPU_GEMM_COLS = 256, 2048


def _cpu_pool(threads=None):
    """Thread pool over all host cores for the oracle's numpy passes (its
    large ufuncs release the GIL) and torch's CPU matmuls."""
    import concurrent.futures
    import torch
    cores = threads or os.cpu_count() or 1
    torch.set_num_threads(cores)
    return cores, concurrent.futures.ThreadPoolExecutor(cores)


def _qdq_rows(x_f32, g, pool, chunk=512):
    """Oracle quantize (along the last dim, global scale g) then dequantize,
    in row chunks on the pool; float32 result (exact dequantised values * g)."""
    import numpy as np
    from oracle import nvfp4_oracle as orc
    x_f32 = np.ascontiguousarray(x_f32, dtype=np.float32)
    r, k = x_f32.shape

    def one(lo):
        c = x_f32[lo:lo + chunk]
        q, s = orc.quant_nvfp4_f32(c, g)
        out = orc.dequant_nvfp4(q, s, c.shape[0], k)
        return out if g is None else out * np.float32(g)

    return np.concatenate(list(pool.map(one, range(0, r, chunk))), axis=0)


def cpu_gemm_sample(rows: int = CPU_GEMM_ROWS, cols: int = CPU_GEMM_COLS, k: int = 8192, threads=None):
    """Reference-path CPU emulation of a [rows x cols] output tile of the
    8192^3 GEMM (quantize both operands with per-tensor global scales,
    dequantize, fp32 torch matmul, bf16 result), all inside the timed region.
    Returns (TFLOP/s of the tile's 2*rows*cols*k flop, cores, seconds, tile)."""
    import numpy as np
    import torch
    from oracle import nvfp4_oracle as orc
    cores, pool = _cpu_pool(threads)
    g = torch.Generator().manual_seed(1)
    a = torch.randn(rows, k, generator=g).to(torch.bfloat16).float().numpy()
    b = torch.randn(cols, k, generator=g).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()
    da = _qdq_rows(a, orc.global_scale_of(a), pool)
    db = _qdq_rows(b, orc.global_scale_of(b), pool)
    d = (torch.from_numpy(da) @ torch.from_numpy(db).T).to(torch.bfloat16)
    dt = time.perf_counter() - t0
    pool.shutdown()
    return 2.0 * rows * cols * k / dt / 1e12, cores, dt, d


def cpu_quant_sample(rows: int = 2048, k: int = 4096, threads=None):
    """Reference-path CPU RMSNorm -> NVFP4 (the oracle restatement of
    float4utils.py:169-295 with gamma and a global scale: 1/RMS, amax of the
    normalised rows, quantize) on `rows` rows of the 32768 x 4096 workload.
    Returns (GB/s of algorithmic bytes, cores, seconds)."""
    import numpy as np
    import torch
    from oracle import nvfp4_oracle as orc
    cores, pool = _cpu_pool(threads)
    g = torch.Generator().manual_seed(2)
    rs = torch.exp(torch.empty(rows, 1).uniform_(math.log(0.1), math.log(10.0), generator=g))
    x = (torch.randn(rows, k, generator=g) * rs).to(torch.bfloat16).float().numpy()
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).float().numpy()
    t0 = time.perf_counter()

    def stats(lo):
        c = x[lo:lo + 512].astype(np.float64)
        inv = (1.0 / np.sqrt(np.mean(c * c, axis=1) + 1e-6)).astype(np.float32)
        y = (x[lo:lo + 512] * inv[:, None]).astype(np.float32) * gamma[None, :]
        return inv, y.astype(np.float32)

    parts = list(pool.map(stats, range(0, rows, 512)))
    y = np.concatenate([p[1] for p in parts])
    gs = orc.global_scale_of(y)
    list(pool.map(lambda lo: orc.quant_nvfp4_f32(y[lo:lo + 512], gs), range(0, rows, 512)))
    dt = time.perf_counter() - t0
    pool.shutdown()
    nbytes = orc.bytes_nvfp4_quant(rows, k) + k * 2 + rows * 4
    return nbytes / dt / 1e9, cores, dt


def cpu_mlp_sample(tokens: int = 128, d: int = 4096, f: int = 14336, threads=None):
    """Reference-path CPU emulation of one NVFP4 SwiGLU MLP block training step
    (the single-block workload at a reduced token count): every GEMM operand
    quantized with its global scale along its contraction dimension and
    dequantized (oracle), fp32 torch matmuls, bf16 rounding where the CUDA
    step stores bf16, RMSNorm backward, and fp32 AdamW with master weights on
    all 3*d*f + d parameters.  Returns (tokens/s, cores, seconds)."""
    import numpy as np
    import torch
    from oracle import nvfp4_oracle as orc
    cores, pool = _cpu_pool(threads)
    g = torch.Generator().manual_seed(3)
    bf = lambda t: t.to(torch.bfloat16).float()
    x = bf(torch.randn(tokens, d, generator=g))
    w_gu = bf(0.02 * torch.randn(2 * f, d, generator=g))
    w_down = bf(0.02 * torch.randn(d, f, generator=g))
    dy = bf(1e-3 * torch.randn(tokens, d, generator=g))
    params = [w_gu, w_down]
    master = [p.clone() for p in params]
    mom = [(torch.zeros_like(p), torch.zeros_like(p)) for p in params]
    gsc = lambda t: orc.global_scale_of(t.numpy())
    qdq = lambda t, gg: torch.from_numpy(_qdq_rows(t.contiguous().numpy(), gg, pool))
    t0 = time.perf_counter()
    g_gu, g_d = gsc(w_gu), gsc(w_down)
    wgu_q, wd_q = qdq(w_gu, g_gu), qdq(w_down, g_d)
    wgu_tq, wd_tq = qdq(w_gu.T, g_gu), qdq(w_down.T, g_d)
    inv = torch.rsqrt((x.double() ** 2).mean(1) + 1e-6).float()
    xn = x * inv[:, None]
    g_xn = gsc(xn)
    gu = bf(qdq(xn, g_xn) @ wgu_q.T)
    gate, up = gu[:, :f], gu[:, f:]
    sg = torch.sigmoid(gate)
    h = bf(gate * sg * up)
    g_h = gsc(h)
    y = bf(qdq(h, g_h) @ wd_q.T + x)
    g_dy = gsc(dy)
    dh = bf(qdq(dy, g_dy) @ wd_tq.T)
    dgu = torch.cat([bf(dh * up * (sg * (1 + gate * (1 - sg)))), bf(dh * gate * sg)], dim=1)
    g_dgu = gsc(dgu)
    dxn = bf(qdq(dgu, g_dgu) @ wgu_tq.T)
    d_down = qdq(dy.T, g_dy) @ qdq(h.T, g_h).T
    d_gu = qdq(dgu.T, g_dgu) @ qdq(xn.T, g_xn).T
    mean = (dxn * xn).sum(1, keepdim=True) / d
    dx = bf(inv[:, None] * (dxn - xn * mean) + dy)
    for p, w, (m, v), gr in zip(params, master, mom, (d_gu, d_down)):   # AdamW, torch.optim.AdamW order
        w.mul_(1.0)
        m.lerp_(gr, 0.1)
        v.mul_(0.95).addcmul_(gr, gr, value=0.05)
        w.addcdiv_(m, v.sqrt().div_(math.sqrt(0.05)).add_(1e-8), value=-1e-4 / 0.1)
        p.copy_(bf(w))
    dt = time.perf_counter() - t0
    pool.shutdown()
    assert torch.isfinite(y).all() and torch.isfinite(dx).all()
    return tokens / dt, cores, dt


def reference_arm(args, world, rank):
    """The reference's own CPU path restated (the oracle: quantize,
    dequantize, fp32 matmul; float4utils.py:79-148 and the emulation of
    cutlass_mm_fp4.cu:182-184) on the host cores, one [256 x 2048] tile of the
    8192^3 GEMM per step.  Rank 0 only."""
    if world > 1 and rank != 0:
        return None
    for _ in range(args.warmup):
        cpu_gemm_sample()
    vals, secs = [], []
    cores = 1
    for _ in range(args.steps):
        v, cores, dt, _ = cpu_gemm_sample()
        vals.append(v)
        secs.append(dt)
    val = statistics.median(vals)
    flops_tile = 2.0 * CPU_GEMM_ROWS * CPU_GEMM_COLS * 8192
    sample = (f"{CPU_GEMM_ROWS} x {CPU_GEMM_COLS} output tile of the 8192^3 GEMM per step ({flops_tile:.3g} flop): "
              f"oracle quantize (global scales) + dequantize of both operand slices + torch fp32 matmul on {cores} "
              "host threads")
    return {"impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(secs) * 1e3,
            "ms_per_full_8192_cubed_extrapolated": 2.0 * 8192 ** 3 / (val * 1e12) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "NVFP4 block-scaled GEMM M=N=K=8192 (seed 1), CPU emulation of one "
                                   f"{CPU_GEMM_ROWS} x {CPU_GEMM_COLS} output tile per step",
                       "global_batch": 8192, "seq_len": 1, "parallelism": "rank0 host cores"},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip", default="", help="comma list of sub-benchmarks to skip: quant,mlp_block,mlp_stack,cpu")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the GEMM M sweep")
    ap.add_argument("--no-clock-hold", action="store_true", help="skip the 1 s sustained clock window (profiling)")
    ap.add_argument("--comm-sms", type=int, default=0,
                    help="MLP stack at N > 1: SMs left free of GEMMs for the NCCL kernels (0 = none)")
    ap.add_argument("--allreduce", action="store_true",
                    help="MLP stack at N > 1: plain all-reduce + replicated AdamW instead of ZeRO-1")
    ap.add_argument("--bf16-gather", action="store_true",
                    help="MLP stack at N > 1 (ZeRO-1): gather bf16 parameters and quantize all weights on every "
                         "rank instead of gathering each rank's quantized rows")
    ap.add_argument("--breakdown", action="store_true",
                    help="after the timed MLP steps, one more step under torch.profiler: per-kernel device time")
    ap.add_argument("--only", choices=["gemm", "gemm_sweep", "quant", "mlp_block", "mlp_stack"], default=None,
                    help="run one section and print its result (profiling runs)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    skip = set(s for s in args.skip.split(",") if s)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    import torch
    import __graft_entry__
    pkg = __graft_entry__.import_package()
    pkg.load_library()
    world, rank, local = dist_setup(args.gpus)
    peaks = load_peaks()
    pg = None
    if world > 1:
        import torch.distributed as dist
        pg = dist.group.WORLD

    if args.only is not None:
        if args.only == "gemm":
            res = bench_gemm(pkg, args, world, rank, peaks)
        elif args.only == "gemm_sweep":   # the M sweep alone (N = K = 8192), e.g. to profile one size
            _, _, qb, sb, _, gb = gemm_operands(pkg, 8, 8192, 8192, seed=1)
            res = gemm_m_sweep(pkg, args, qb, sb, gb, Flusher(), with_cublas=not args.no_cublas)
        elif args.only == "quant":
            res = bench_quant(pkg, args, peaks)
        elif args.only == "mlp_block":
            res = bench_mlp(pkg, args, world, rank, 1, 4096, 14336, 16384, seed=3, e2e_steps=args.steps)
        else:
            res = bench_mlp(pkg, args, world, rank, 8, 8192, 28672, 65536, seed=4, pg=pg)
        if rank == 0:
            print(json.dumps({"only": args.only, "result": res}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return 0

    gemm = bench_gemm(pkg, args, world, rank, peaks)
    line = {"metric": METRIC, "value": gemm["value"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": gemm["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e4m3, fp32 accumulate) -> bf16",
            "data": "synthetic (seeded N(0,1) bf16, pre-quantized NVFP4)",
            "config": {"workload": "NVFP4 block-scaled GEMM M=N=K=8192, seed 1, per-rank replica",
                       "M": 8192, "N": 8192, "K": 8192, "global_batch": 8192 * world, "seq_len": 1,
                       "parallelism": f"replicas x{world}", "l2": "flushed (256 MB write) before every timed launch"},
            "roofline": gemm["roofline"], "clocks": gemm["clocks"], "e2e": gemm["e2e"],
            "gpu_launches": args.steps * gemm["gpu_launches_per_step"],
            "cublaslt_scaled_mm_tflops": gemm.get("cublaslt_scaled_mm_tflops"),
            "spot_check_max_rel_err": gemm["spot_check_max_rel_err"]}
    if "m_sweep" in gemm:
        line["gemm_m_sweep"] = gemm["m_sweep"]
    if "mxfp4" in gemm:
        line["mxfp4_gemm_8192"] = gemm["mxfp4"]
    if "cublaslt_error" in gemm:
        line["cublaslt_error"] = gemm["cublaslt_error"]
    cpu = rank == 0 and world == 1 and "cpu" not in skip
    if cpu:
        v, cores, dt, _ = cpu_gemm_sample()
        line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                "sample": f"{CPU_GEMM_ROWS} x {CPU_GEMM_COLS} output tile of the 8192^3 GEMM: oracle "
                                          "quantize + dequantize of both operand slices + torch fp32 matmul on "
                                          f"{cores} host threads ({dt:.2f} s)"}
    if world == 1 and "quant" not in skip:
        line["quant"] = bench_quant(pkg, args, peaks)
        if cpu:
            v, cores, dt = cpu_quant_sample()
            line["quant"]["cpu_baseline"] = {
                "value": v, "unit": "GB/s", "cores": cores, "kind": "port",
                "sample": f"2048 of 32768 rows: oracle 1/RMS, amax of (x*inv_rms)*gamma and NVFP4 quantize on "
                          f"{cores} host threads ({dt:.2f} s), GB/s of the rows' algorithmic bytes"}
    if world == 1 and "mlp_block" not in skip:
        line["mlp_block"] = bench_mlp(pkg, args, world, rank, 1, 4096, 14336, 16384, seed=3, e2e_steps=args.steps)
        line["mlp_block"]["workload"] = "1 RMSNorm+SwiGLU block, 16384 tokens, d=4096, ff=14336, AdamW fp32"
        if cpu:
            v, cores, dt = cpu_mlp_sample()
            line["mlp_block"]["cpu_baseline"] = {
                "value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                "sample": f"one block step at 128 tokens (d 4096, ff 14336): oracle quantize/dequantize of every "
                          f"GEMM operand incl. both weight orientations, torch fp32 matmuls, AdamW on {cores} host "
                          f"threads ({dt:.2f} s); tokens/s = 128 / that time (the per-step weight work does not "
                          "shrink with tokens, so this understates the CPU rate at 16384 tokens)"}
    if "mlp_stack" not in skip:
        line["mlp_stack"] = bench_mlp(pkg, args, world, rank, 8, 8192, 28672, 65536, seed=4, pg=pg)
        line["mlp_stack"]["workload"] = ("8 RMSNorm+SwiGLU blocks, d=8192, ff=28672, 65536 global tokens split "
                                         "across ranks; at N > 1 ZeRO-1: bf16 wgrad reduce-scatter (NCCL) overlapped "
                                         "with backward, AdamW on each rank's 1/N shard, each rank quantizes its "
                                         "rows of the updated weights, NVFP4 weight all-gather overlapped with the "
                                         "next step's forward")
        line["mlp_stack"]["scaling"] = "strong"
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
