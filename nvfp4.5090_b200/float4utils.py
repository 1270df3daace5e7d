"""B200 drop-in for the reference's ``float4utils.py`` API.

Same names, signatures, shapes, dtypes and error behaviour as the reference
module (xTimeCrystal/NVFP4.5090 ``float4utils.py``), backed by the sm_100a
CUDA library of this package instead of CuPy/NVRTC kernels and the SM120-only
CUTLASS op.  Additions are keyword-only and default to the reference
behaviour:

* ``global_scale`` on the quantizers (a 1-element float32 CUDA tensor; the
  default ``None`` means g = 1, bit-identical to the reference);
* ``use_global_scale`` on the GEMM wrappers (computes per-tensor scales
  g = amax/(6*448) and folds g_A*g_B into the GEMM's output scale);
* ``nvfp4_backward`` on ``NVFP4Linear`` (NVFP4 dgrad/wgrad instead of the
  reference's bf16 backward, float4utils.py:653-683).

Benchmarks are timed with CUDA events (no Triton): ``bench_quant_gbps`` and
``bench_gemm_tflops`` keep the reference's sweep points and ``.run()``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import ops
from .gn_kernels import cutlass_nvfp4_mm, cutlass_nvfp4_mm_relu, cutlass_nvfp4_mm_relu_2


# -----------------------------
# Helpers & Checks (float4utils.py:43-48)
# -----------------------------
def round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m


def require(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


# -----------------------------
# DType checks (float4utils.py:53-56)
# -----------------------------
require(hasattr(torch, "float4_e2m1fn_x2"), "Your torch build lacks torch.float4_e2m1fn_x2.")
require(hasattr(torch, "float8_e4m3fn"), "Your torch build lacks torch.float8_e4m3fn.")
FP4_DTYPE = torch.float4_e2m1fn_x2
FP8_SCALE_DTYPE = torch.float8_e4m3fn


def _flatten(x: torch.Tensor):
    shape = x.shape
    k = shape[-1]
    batch = shape[:-1]
    r = math.prod(batch) if batch else 1
    return x.reshape(r, k), batch, r, k


# ============================================================
# Quantizers (float4utils.py:327-401)
# ============================================================

def quant_nvfp4_fused(x_bf16: torch.Tensor, *, global_scale: Optional[torch.Tensor] = None
                      ) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [..., K] -> (q float4_e2m1fn_x2 [..., K/2], s float8_e4m3fn [round_up(R,128), round_up(K/16,4)])."""
    require(x_bf16.is_cuda and x_bf16.dtype == torch.bfloat16,
            "quant_nvfp4_fused expects a CUDA BF16 tensor.")
    x = x_bf16.contiguous()
    x2, batch, r, k = _flatten(x)
    require(k % 16 == 0, "K must be divisible by 16 for NVFP4 1x16 scaling.")
    q, s = ops.quantize(x2, global_scale=global_scale)
    return q.view(FP4_DTYPE).reshape(*batch, k // 2), s.view(FP8_SCALE_DTYPE)


def rmsnorm_quant_nvfp4_fused(x_bf16: torch.Tensor, epsilon: float = 1e-6, *,
                              gamma: Optional[torch.Tensor] = None,
                              global_scale: Optional[torch.Tensor] = None
                              ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """RMSNorm along K then NVFP4 -> (q, s, inv_rms float32 [...])."""
    require(x_bf16.is_cuda and x_bf16.dtype == torch.bfloat16,
            "rmsnorm_quant_nvfp4_fused expects a CUDA BF16 tensor.")
    x = x_bf16.contiguous()
    x2, batch, r, k = _flatten(x)
    require(k % 16 == 0, "K must be divisible by 16 for NVFP4 1x16 scaling.")
    q, s, inv = ops.rmsnorm_quantize(x2, float(epsilon), gamma=gamma, global_scale=global_scale)
    return (q.view(FP4_DTYPE).reshape(*batch, k // 2), s.view(FP8_SCALE_DTYPE),
            inv.reshape(batch if batch else (1,)))


# ============================================================
# NVFP4 matmul (float4utils.py:407-515)
# ============================================================

def _quant_operands(A_bf16, B_bf16, apply_rmsnorm_lhs, rms_eps, use_global_scale):
    a2, batch, _, k = _flatten(A_bf16.contiguous())
    b2 = B_bf16.contiguous()
    require(b2.dim() == 2, "B must be a 2-D [N, K] tensor")
    ga = gb = None
    inv = None
    if use_global_scale:
        gb = ops.global_scale(b2)
        if apply_rmsnorm_lhs:
            inv, ga = ops.rmsnorm_stats(a2, rms_eps)
            qa, sa = ops.quantize(a2, global_scale=ga, row_scale=inv)
        else:
            ga = ops.global_scale(a2)
            qa, sa = ops.quantize(a2, global_scale=ga)
    else:
        if apply_rmsnorm_lhs:
            qa, sa, inv = ops.rmsnorm_quantize(a2, rms_eps)
        else:
            qa, sa = ops.quantize(a2)
    qb, sb = ops.quantize(b2, global_scale=gb)
    return qa, sa, qb, sb, ga, gb, inv, batch


def _nvfp4mm_impl(A_bf16, B_bf16, out_dtype, apply_rmsnorm_lhs, rms_eps, use_global_scale, epilogue):
    require(A_bf16.is_cuda and B_bf16.is_cuda, "nvfp4mm requires CUDA tensors.")
    require(A_bf16.dtype == torch.bfloat16 and B_bf16.dtype == torch.bfloat16, "nvfp4mm expects BF16 inputs.")
    qa, sa, qb, sb, ga, gb, inv, batch = _quant_operands(A_bf16, B_bf16, apply_rmsnorm_lhs, rms_eps,
                                                         use_global_scale)
    od = out_dtype if out_dtype in (torch.bfloat16, torch.float32) else torch.bfloat16
    c = ops.gemm(qa, sa, qb, sb, scale_a=ga, scale_b=gb, out_dtype=od, epilogue=epilogue)
    c = c.reshape(*batch, c.shape[-1])
    if apply_rmsnorm_lhs:
        return c, inv.reshape(batch if batch else (1,))
    return c


@torch.no_grad()
def nvfp4mm_torch(A_bf16: torch.Tensor, B_bf16: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
                  apply_rmsnorm_lhs: bool = False, rms_eps: float = 1e-6) -> torch.Tensor:
    """Fully dynamic NVFP4 GEMM: C = A @ B^T through torch's ``scaled_mm`` (cuBLASLt), as the
    reference's float4utils.py:407-437 does; the quantizers are this library's."""
    import torch.nn.functional as F
    from torch.nn.functional import ScalingType, SwizzleType
    require(A_bf16.is_cuda and B_bf16.is_cuda, "nvfp4mm requires CUDA tensors.")
    if apply_rmsnorm_lhs:
        a_fp4, s_a_swz, _ = rmsnorm_quant_nvfp4_fused(A_bf16, epsilon=rms_eps)
    else:
        a_fp4, s_a_swz = quant_nvfp4_fused(A_bf16)
    b_fp4, s_b_swz = quant_nvfp4_fused(B_bf16)
    return F.scaled_mm(a_fp4, b_fp4.mT, s_a_swz, ScalingType.BlockWise1x16, s_b_swz, ScalingType.BlockWise1x16,
                       swizzle_a=SwizzleType.SWIZZLE_32_4_4, swizzle_b=SwizzleType.SWIZZLE_32_4_4,
                       output_dtype=out_dtype, contraction_dim=(1, 0))


@torch.no_grad()
@torch._dynamo.disable
def nvfp4mm(A_bf16: torch.Tensor, B_bf16: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
            apply_rmsnorm_lhs: bool = False, rms_eps: float = 1e-6, use_global_scale: bool = False):
    """Fully dynamic NVFP4 GEMM: C = A @ B^T (returns (C, inv_rms) with apply_rmsnorm_lhs)."""
    return _nvfp4mm_impl(A_bf16, B_bf16, out_dtype, apply_rmsnorm_lhs, rms_eps, use_global_scale, ops.EPI_NONE)


@torch.no_grad()
@torch._dynamo.disable
def nvfp4mm_relu(A_bf16: torch.Tensor, B_bf16: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
                 apply_rmsnorm_lhs: bool = False, rms_eps: float = 1e-6, use_global_scale: bool = False):
    """Fully dynamic NVFP4 GEMM: C = Relu(A @ B^T)."""
    return _nvfp4mm_impl(A_bf16, B_bf16, out_dtype, apply_rmsnorm_lhs, rms_eps, use_global_scale, ops.EPI_RELU)


@torch.no_grad()
@torch._dynamo.disable
def nvfp4mm_relu_2(A_bf16: torch.Tensor, B_bf16: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
                   apply_rmsnorm_lhs: bool = False, rms_eps: float = 1e-6, use_global_scale: bool = False):
    """Fully dynamic NVFP4 GEMM: C = Relu^2(A @ B^T)."""
    return _nvfp4mm_impl(A_bf16, B_bf16, out_dtype, apply_rmsnorm_lhs, rms_eps, use_global_scale, ops.EPI_RELU2)


# ============================================================
# Accuracy + Benchmarks (float4utils.py:521-617)
# ============================================================

@torch.no_grad()
def test_accuracy(M=1024, N=2048, K=4096):
    print(f"\n--- NVFP4 Accuracy (M={M}, N={N}, K={K}) ---")
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    C_ref = A @ B.t()
    C = nvfp4mm(A, B, out_dtype=torch.bfloat16, apply_rmsnorm_lhs=False)
    diff = (C_ref - C).float().abs()
    mse = (diff ** 2).mean().item()
    mx = diff.max().item()
    rel = (diff.mean() / C_ref.float().abs().mean()).item()
    print(f"MSE:    {mse:.6e}")
    print(f"Max Abs:  {mx:.6e}")
    print(f"Mean Rel: {rel:.6%}")
    return {"mse": mse, "max_abs": mx, "mean_rel": rel}


def _bytes_nvfp4_quant_fused(R: int, K: int) -> float:
    pad_R = round_up(R, 128)
    pad_cols = round_up(K // 16, 4)
    # Traffic: Read bf16(2), Write fp4(0.5), Write scales(1)
    return (R * K * 2.0) + (R * K * 0.5) + (pad_R * pad_cols * 1.0)


def _time_ms(fn, warmup: int = 5, iters: int = 20) -> Tuple[float, float, float]:
    """Median, 20th and 80th percentile of per-call CUDA-event times (ms)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    pick = lambda q: times[min(len(times) - 1, int(q * len(times)))]
    return pick(0.5), pick(0.2), pick(0.8)


class _Sweep:
    """Minimal stand-in for the reference's triton ``perf_report`` objects."""

    def __init__(self, fn, x_name, x_vals, providers, args):
        self.fn, self.x_name, self.x_vals, self.providers, self.args = fn, x_name, x_vals, providers, args

    def __call__(self, **kw):
        return self.fn(**kw)

    def run(self, print_data: bool = True, save_path: Optional[str] = None):
        rows = []
        for x in self.x_vals:
            row = {self.x_name: x}
            for prov in self.providers:
                row[prov] = self.fn(**{**self.args, self.x_name: x, "provider": prov})[0]
            rows.append(row)
            if print_data:
                print(row)
        if save_path:
            import csv
            import os
            with open(os.path.join(save_path, f"{self.fn.__name__}.csv"), "w", newline="") as f:
                w = csv.DictWriter(f, fieldnames=list(rows[0]))
                w.writeheader()
                w.writerows(rows)
        return rows


def _bench_quant_gbps(M, N, K, provider):
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16).contiguous()
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16).contiguous()
    if provider == "quant_A":
        fn, rows = (lambda: quant_nvfp4_fused(A)), M
    elif provider == "quant_B":
        fn, rows = (lambda: quant_nvfp4_fused(B)), N
    else:
        fn, rows = (lambda: rmsnorm_quant_nvfp4_fused(A)), M
    ms, lo, hi = _time_ms(fn)
    gbps = lambda t: _bytes_nvfp4_quant_fused(rows, K) / (t * 1e-3) / 1e9
    return gbps(ms), gbps(hi), gbps(lo)


def _bench_gemm_tflops(M, N, K, provider):
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16).contiguous()
    B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16).contiguous()
    ones = torch.tensor(1.0, device="cuda")
    if provider == "static":
        a_fp4, s_a = quant_nvfp4_fused(A)
        b_fp4, s_b = quant_nvfp4_fused(B)
        fn = lambda: cutlass_nvfp4_mm(a_fp4, b_fp4.mT, s_a, s_b, ones)
    elif provider == "dynamic":
        def fn():
            a, sa = quant_nvfp4_fused(A)
            b, sb = quant_nvfp4_fused(B)
            return cutlass_nvfp4_mm(a, b.mT, sa, sb, ones)
    else:
        def fn():
            a, sa, _ = rmsnorm_quant_nvfp4_fused(A)
            b, sb = quant_nvfp4_fused(B)
            return cutlass_nvfp4_mm(a, b.mT, sa, sb, ones)
    ms, lo, hi = _time_ms(fn)
    tflops = lambda t_ms: (2.0 * M * N * K) / (t_ms * 1e-3) / 1e12
    return tflops(ms), tflops(hi), tflops(lo)


bench_quant_gbps = _Sweep(_bench_quant_gbps, "K", [1024 * i for i in range(4, 33, 4)],
                          ["quant_A", "quant_B", "rmsnorm_quant_A"], {"M": 4096, "N": 8192})
bench_gemm_tflops = _Sweep(_bench_gemm_tflops, "K", [128, 256] + [512 * i for i in range(1, 33)],
                           ["static", "dynamic", "dynamic_rms"], {"M": 4096, "N": 8192})


# ============================================================
# Autograd linear (float4utils.py:619-714)
# ============================================================

class NVFP4LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, input: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                nvfp4_backward: bool = False):
        """Forward pass: X @ W^T with fully dynamic NVFP4 quantization."""
        ctx.save_for_backward(input, weight)
        ctx.has_bias = bias is not None
        ctx.nvfp4_backward = nvfp4_backward
        input_shape = input.shape
        x_2d = input.view(-1, input_shape[-1]) if input.dim() > 2 else input
        out_2d = nvfp4mm(x_2d, weight, out_dtype=input.dtype, use_global_scale=nvfp4_backward)
        out = out_2d.view(*input_shape[:-1], weight.shape[0]) if input.dim() > 2 else out_2d
        if bias is not None:
            out += bias
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        """bf16 backward as in the reference (float4utils.py:653-683), or NVFP4
        dgrad/wgrad (each operand requantized along its contraction dim)."""
        input, weight = ctx.saved_tensors
        grad_input = grad_weight = grad_bias = None
        if input.dim() > 2:
            grad_output_2d = grad_output.reshape(-1, grad_output.shape[-1])
            input_2d = input.reshape(-1, input.shape[-1])
        else:
            grad_output_2d = grad_output
            input_2d = input
        if not ctx.nvfp4_backward:
            if ctx.needs_input_grad[0]:
                grad_input = grad_output_2d.matmul(weight).view_as(input)
            if ctx.needs_input_grad[1]:
                grad_weight = grad_output_2d.t().matmul(input_2d)
        else:
            dy = grad_output_2d.contiguous().to(torch.bfloat16)
            if ctx.needs_input_grad[0]:
                gd = ops.global_scale(dy)
                gw = ops.global_scale(weight)
                qd, sd = ops.quantize(dy, global_scale=gd)
                qwt, swt = ops.quantize_t(weight.contiguous(), global_scale=gw)
                grad_input = ops.gemm(qd, sd, qwt, swt, scale_a=gd, scale_b=gw).view_as(input)
            if ctx.needs_input_grad[1]:
                gd = ops.global_scale(dy)
                gx = ops.global_scale(input_2d)
                qdt, sdt = ops.quantize_t(dy, global_scale=gd)
                qxt, sxt = ops.quantize_t(input_2d.contiguous(), global_scale=gx)
                grad_weight = ops.gemm(qdt, sdt, qxt, sxt, scale_a=gd, scale_b=gx)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            grad_bias = grad_output_2d.sum(dim=0)
        return grad_input, grad_weight, grad_bias, None


class NVFP4Linear(nn.Module):
    """Drop-in replacement for torch.nn.Linear using NVFP4 for the forward pass
    (and, with ``nvfp4_backward=True``, for dgrad and wgrad)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 device=None, dtype=torch.bfloat16, *, nvfp4_backward: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.nvfp4_backward = nvfp4_backward
        self.weight = nn.Parameter(torch.empty((out_features, in_features), device=device, dtype=dtype))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, device=device, dtype=dtype))
        else:
            self.register_parameter('bias', None)
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        return NVFP4LinearFunction.apply(input, self.weight, self.bias, self.nvfp4_backward)


__all__ = ["round_up", "require", "FP4_DTYPE", "FP8_SCALE_DTYPE", "quant_nvfp4_fused",
           "rmsnorm_quant_nvfp4_fused", "nvfp4mm_torch", "nvfp4mm", "nvfp4mm_relu", "nvfp4mm_relu_2",
           "test_accuracy", "_bytes_nvfp4_quant_fused", "bench_quant_gbps", "bench_gemm_tflops",
           "NVFP4LinearFunction", "NVFP4Linear", "cutlass_nvfp4_mm", "cutlass_nvfp4_mm_relu",
           "cutlass_nvfp4_mm_relu_2"]
