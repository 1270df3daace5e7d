"""CPU tests of bench.py's host logic: the clock record that decides whether a
run is kept (median SM clock and the throttle reasons seen), the reference
arm's rank handling under torchrun (ranks other than 0 exit without work),
the CPU baseline samples (the reference arm's GEMM tile is the oracle's NVFP4
product of its operands), and the per-kernel step summaries."""
import numpy as np
import pytest
import torch

import bench
from oracle import nvfp4_oracle as orc


def _sampler(lines):
    s = bench.ClockSampler(0)
    s.lines = lines
    return s.summary()


def test_clock_summary_median_and_power_cap():
    lines = [
        "0, 1470, 1965, 998.1, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1455, 1965, 1001.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 420.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    s = _sampler(lines)
    assert s["sm_mhz"] == 1470 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_reports_rejecting_reasons():
    lines = [
        "0, 1200, 1965, 700.0, 0x48, Active, Not Active, Not Active, Not Active",
        "0, 1100, 1965, 690.0, 0x20, Not Active, Not Active, Active, Not Active",
        "0, 1000, 1965, 650.0, 0x40, Not Active, Active, Not Active, Not Active",
    ]
    s = _sampler(lines)
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_clock_summary_skips_malformed_lines():
    s = _sampler(["garbage", "0, [N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
                  "0, 1500, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active"])
    assert s["sm_mhz"] == 1500 and s["samples"] == 1 and s["reasons"] == []
    assert _sampler([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_reference_arm_other_ranks_exit_without_work(monkeypatch, capsys):
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setattr(bench, "cpu_gemm_sample", lambda: (_ for _ in ()).throw(AssertionError("ran work")))
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3"]) == 0
    assert capsys.readouterr().out == ""


def test_kernel_summary_exposed_comm():
    """summarize_kernels on a synthetic step: compute kernels with one gap
    covered by a reduce-scatter, then the next step's two all-gathers after
    the last compute kernel.  Steady-state exposure = the in-step gap + the
    first trailing gather; the trailing gathers are reported apart."""
    ks = sorted([
        (0.0, 1000.0, "nvfp4b200::gemm::nvfp4_gemm_kernel(...)"),
        (1000.0, 1500.0, "quant_tile_kernel"),
        (1400.0, 2600.0, "ncclDevKernel_ReduceScatter_Sum_bf16_RING_LL"),
        (2000.0, 3000.0, "nvfp4b200::gemm::nvfp4_gemm_kernel(...)"),   # gap 1500..2000 under the RS
        (3000.0, 3400.0, "ncclDevKernel_AllGather_RING_LL"),
        (3400.0, 3900.0, "ncclDevKernel_AllGather_RING_LL"),
    ])
    r = bench.summarize_kernels(ks, n_blocks=1, d=64, f=128, micro=16)
    assert abs(r["compute_busy_ms"] - 2.5) < 1e-9
    assert abs(r["exposed_in_step_ms"] - 0.5) < 1e-9
    assert abs(r["trailing_nccl_ms"] - 0.9) < 1e-9
    assert abs(r["first_trailing_gather_ms"] - 0.4) < 1e-9
    assert abs(r["exposed_comm_ms"] - 0.9) < 1e-9
    assert abs(r["span_minus_compute_ms"] - 1.4) < 1e-9
    assert r["largest_gaps"][0]["ms"] == 0.5 and r["largest_gaps"][0]["nccl_running"] == ["ncclDevKernel_ReduceScatter_Sum_bf16_RING_LL"]


def test_kernel_summary_wgrad_splits():
    """With rank-major buckets each wgrad GEMM is several launches: the role
    time sums a GEMM's row blocks, and the other roles keep their place."""
    g = "nvfp4b200::gemm::nvfp4_gemm_kernel"
    dur = {"fwd_gate_up_swiglu": 300.0, "fwd_down": 200.0, "bwd_dh_swiglu": 250.0, "wgrad_down": 50.0,
           "bwd_dxn": 400.0, "wgrad_gate_up": 100.0}
    seq = ["fwd_gate_up_swiglu", "fwd_down"] * 2 + (["bwd_dh_swiglu"] + ["wgrad_down"] * 4 + ["bwd_dxn"]
                                                    + ["wgrad_gate_up"] * 4) * 2
    ks, t = [], 0.0
    for r in seq:
        ks.append((t, t + dur[r], g))
        t += dur[r]
    out = bench.summarize_kernels(ks, n_blocks=2, d=64, f=128, micro=16, wgrad_splits=4)["gemm_roles"]
    assert out["wgrad_down"]["launches"] == 2 and abs(out["wgrad_down"]["mean_ms"] - 0.2) < 1e-9
    assert out["wgrad_gate_up"]["launches"] == 2 and abs(out["wgrad_gate_up"]["mean_ms"] - 0.4) < 1e-9
    assert out["bwd_dxn"]["launches"] == 2 and abs(out["bwd_dxn"]["mean_ms"] - 0.4) < 1e-9
    assert out["fwd_down"]["launches"] == 2 and abs(out["fwd_down"]["mean_ms"] - 0.2) < 1e-9


@pytest.fixture
def keep_torch_threads():
    n = torch.get_num_threads()
    yield
    torch.set_num_threads(n)


def test_cpu_gemm_sample_computes_its_tile(keep_torch_threads):
    """The reference arm's tile (quantize both operands with their global
    scales, dequantize, fp32 matmul, bf16) at a small size, against the
    oracle's float64 emulation of the same NVFP4 GEMM: every element within
    the GEMM parity bound 2^-8 |ref| + 2^-20 sum |terms|."""
    rows, cols, k = 128, 64, 512
    tflops, cores, secs, d = bench.cpu_gemm_sample(rows, cols, k, threads=2)
    assert tflops > 0 and cores == 2 and secs > 0
    assert d.shape == (rows, cols) and d.dtype == torch.bfloat16
    g = torch.Generator().manual_seed(1)                  # the sample's own operands
    a = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    b = torch.randn(cols, k, generator=g).to(torch.bfloat16)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)
    ga = orc.global_scale_of(a.float().numpy())
    gb = orc.global_scale_of(b.float().numpy())
    qa, sa = orc.quant_nvfp4(bits(a), ga)
    qb, sb = orc.quant_nvfp4(bits(b), gb)
    ref = orc.gemm_emulation_f64(qa, sa, qb, sb, rows, cols, k, output_scale=np.float32(ga) * np.float32(gb))
    terms = (np.abs(orc.dequant_nvfp4(qa, sa, rows, k, ga)).astype(np.float64)
             @ np.abs(orc.dequant_nvfp4(qb, sb, cols, k, gb)).astype(np.float64).T)
    err = np.abs(d.float().numpy().astype(np.float64) - ref)
    assert np.all(err <= 2.0 ** -8 * np.abs(ref) + 2.0 ** -20 * terms)
    assert orc.rel_frobenius(d.float().numpy(), ref) < 1e-2


def test_cpu_quant_and_mlp_samples_run_small(keep_torch_threads):
    gbs, cores, secs = bench.cpu_quant_sample(rows=512, k=256, threads=2)
    assert gbs > 0 and cores == 2 and secs > 0
    tok_s, cores, secs = bench.cpu_mlp_sample(tokens=16, d=128, f=256, threads=2)
    assert tok_s > 0 and cores == 2 and secs > 0
