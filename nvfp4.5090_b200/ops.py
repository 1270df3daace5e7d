"""Torch-tensor wrappers over the C ABI: allocation, validation, stream.

Every function enqueues on the current CUDA stream of the input's device
(the reference's GEMM op does the same, cutlass_mm_fp4.cu:266; unlike the
reference's CuPy quantizer launches, nothing here runs on a second stream
system).  Packed E2M1 tensors are returned as ``uint8``; the
``float4utils``-compatible layer re-views them as ``torch.float4_e2m1fn_x2``
/ ``torch.float8_e4m3fn``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib

EPI_NONE, EPI_RELU, EPI_RELU2 = 0, 1, 2
_DT_BF16, _DT_F32 = 0, 1


def round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m


def scale_shape(rows: int, k: int) -> Tuple[int, int]:
    """Shape of the swizzled scale tensor for a [rows, k] operand (float4utils.py:343-344)."""
    return round_up(rows, 128), round_up(k // 16, 4)


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_bf16(x: torch.Tensor, what: str) -> None:
    _require(x.is_cuda and x.dtype == torch.bfloat16, f"{what} expects a CUDA BF16 tensor.")


def _scalar_f32(g: Optional[torch.Tensor], device) -> Optional[torch.Tensor]:
    if g is None:
        return None
    _require(isinstance(g, torch.Tensor) and g.is_cuda and g.dtype == torch.float32 and g.numel() == 1,
             "global scales are 1-element float32 CUDA tensors")
    _require(g.device == device, "global scale on a different device")
    return g


_WS = {}


def workspace(device: torch.device) -> torch.Tensor:
    """Zeroed 2-word workspace for the amax reductions, one per (device, stream).

    The kernels leave it zero after every call; calls on one stream never
    overlap, so one workspace per stream is race-free."""
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    ws = _WS.get(key)
    if ws is None:
        ws = torch.zeros(2, dtype=torch.int32, device=device)
        _WS[key] = ws
    return ws


# ----------------------------------------------------------------------------
# quantizers
# ----------------------------------------------------------------------------


def _outputs(out, q_shape, s_shape, device):
    """(q, s) to write: new tensors, or the caller's ``out`` pair checked for
    shape, dtype, device and contiguity (e.g. slots of a gather buffer)."""
    if out is None:
        return (torch.empty(q_shape, device=device, dtype=torch.uint8),
                torch.empty(s_shape, device=device, dtype=torch.uint8))
    q, s = out
    for t, shape, name in ((q, q_shape, "q"), (s, s_shape, "s")):
        _require(t.dtype == torch.uint8 and tuple(t.shape) == tuple(shape) and t.is_contiguous()
                 and t.device == device, f"out {name} must be a contiguous uint8 {tuple(shape)} tensor on {device}")
    return q, s


def quantize(x: torch.Tensor, global_scale: Optional[torch.Tensor] = None,
             row_scale: Optional[torch.Tensor] = None, gamma: Optional[torch.Tensor] = None, out=None):
    """Quantize a bf16 [R, K] matrix along K -> (q u8 [R, K/2], s u8 swizzled);
    ``out=(q, s)`` writes into given tensors of those shapes."""
    _check_bf16(x, "quantize")
    _require(x.dim() == 2, "quantize expects a 2-D tensor")
    x = x.contiguous()
    r, k = x.shape
    _require(k % 16 == 0, "K must be divisible by 16 for NVFP4 1x16 scaling.")
    q, s = _outputs(out, (r, k // 2), scale_shape(r, k), x.device)
    g = _scalar_f32(global_scale, x.device)
    if row_scale is not None:
        _require(row_scale.dtype == torch.float32 and row_scale.numel() == r, "row_scale is float32 [R]")
        row_scale = row_scale.contiguous()
    if gamma is not None:
        _check_bf16(gamma, "gamma")
        _require(gamma.numel() == k, "gamma is bf16 [K]")
        gamma = gamma.contiguous()
    if row_scale is None and gamma is None:
        _lib.call("nvfp4b200_quant_nvfp4", x.data_ptr(), q.data_ptr(), s.data_ptr(), r, k, _ptr(g), _stream(x))
    else:
        _lib.call("nvfp4b200_scaled_quant_nvfp4", x.data_ptr(), _ptr(row_scale), _ptr(gamma), q.data_ptr(),
                  s.data_ptr(), r, k, _ptr(g), _stream(x))
    return q, s


def rmsnorm_quantize(x: torch.Tensor, eps: float = 1e-6, gamma: Optional[torch.Tensor] = None,
                     global_scale: Optional[torch.Tensor] = None):
    """Fused RMSNorm -> NVFP4 of a bf16 [R, K] matrix -> (q, s, inv_rms f32 [R])."""
    _check_bf16(x, "rmsnorm_quantize")
    _require(x.dim() == 2, "rmsnorm_quantize expects a 2-D tensor")
    x = x.contiguous()
    r, k = x.shape
    _require(k % 16 == 0, "K must be divisible by 16 for NVFP4 1x16 scaling.")
    q = torch.empty((r, k // 2), device=x.device, dtype=torch.uint8)
    s = torch.empty(scale_shape(r, k), device=x.device, dtype=torch.uint8)
    inv = torch.empty((r,), device=x.device, dtype=torch.float32)
    g = _scalar_f32(global_scale, x.device)
    if gamma is not None:
        _check_bf16(gamma, "gamma")
        gamma = gamma.contiguous()
    _lib.call("nvfp4b200_rmsnorm_quant_nvfp4", x.data_ptr(), _ptr(gamma), q.data_ptr(), s.data_ptr(),
              inv.data_ptr(), r, k, float(eps), _ptr(g), _stream(x))
    return q, s, inv


def rmsnorm_stats(x: torch.Tensor, eps: float = 1e-6, gamma: Optional[torch.Tensor] = None):
    """-> (inv_rms f32 [R], global scale of (x*inv_rms)*gamma as a 1-element f32 tensor)."""
    _check_bf16(x, "rmsnorm_stats")
    x = x.contiguous()
    r, k = x.shape
    inv = torch.empty((r,), device=x.device, dtype=torch.float32)
    g = torch.empty((1,), device=x.device, dtype=torch.float32)
    if gamma is not None:
        gamma = gamma.contiguous()
    _lib.call("nvfp4b200_rmsnorm_stats", x.data_ptr(), _ptr(gamma), inv.data_ptr(), r, k, float(eps),
              workspace(x.device).data_ptr(), g.data_ptr(), _stream(x))
    return inv, g


def quantize_t(x: torch.Tensor, global_scale: Optional[torch.Tensor] = None,
               row_scale: Optional[torch.Tensor] = None, gamma: Optional[torch.Tensor] = None, out=None):
    """Quantize x^T (x bf16 [R, C]) along R -> (q u8 [C, R/2], s swizzled for (C, R));
    ``out=(q, s)`` writes into given tensors of those shapes."""
    _check_bf16(x, "quantize_t")
    x = x.contiguous()
    r, c = x.shape
    _require(r % 16 == 0 and c % 8 == 0, "quantize_t needs rows % 16 == 0 and cols % 8 == 0")
    q, s = _outputs(out, (c, r // 2), scale_shape(c, r), x.device)
    g = _scalar_f32(global_scale, x.device)
    if row_scale is not None:
        row_scale = row_scale.contiguous()
    if gamma is not None:
        gamma = gamma.contiguous()
    _lib.call("nvfp4b200_quant_nvfp4_t", x.data_ptr(), _ptr(row_scale), _ptr(gamma), q.data_ptr(), s.data_ptr(),
              r, c, _ptr(g), _stream(x))
    return q, s


def global_scale(x: torch.Tensor, with_amax: bool = False):
    """g = amax(|x|)/(6*448) of a bf16 tensor, as a 1-element float32 CUDA tensor."""
    _check_bf16(x, "global_scale")
    x = x.contiguous()
    g = torch.empty((1,), device=x.device, dtype=torch.float32)
    amax = torch.empty((1,), device=x.device, dtype=torch.float32) if with_amax else None
    _lib.call("nvfp4b200_global_scale", x.data_ptr(), x.numel(), workspace(x.device).data_ptr(), g.data_ptr(),
              _ptr(amax), _stream(x))
    return (g, amax) if with_amax else g


# ----------------------------------------------------------------------------
# GEMM
# ----------------------------------------------------------------------------


def set_gemm_max_sms(max_sms: int) -> None:
    """Cap the SMs a GEMM launch occupies (0 = all).  Process-wide; a
    data-parallel step lowers it so NCCL kernels run beside the GEMMs."""
    _lib.call("nvfp4b200_set_gemm_max_sms", int(max_sms))


def mx_scale_shape(rows: int, k: int):
    """(padded rows, padded columns) of an MXFP4 scale tensor: one UE8M0 scale per 1x32 block."""
    return ((rows + 127) // 128) * 128, ((k // 32 + 3) // 4) * 4


def mxfp4_mm(qa: torch.Tensor, sa: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor,
             bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MXFP4 GEMM: D[m, n] = bf16(A . B^T + bias), E2M1 operands with UE8M0 scales per 1x32 block.

    qa: [m, k/2] packed bytes, qb: [n, k/2] packed bytes; sa / sb: swizzled
    [round_up(rows,128), round_up(k/32,4)] UE8M0 bytes."""
    _require(qa.is_cuda and qb.is_cuda, "mxfp4_mm requires CUDA tensors")
    m, kh = qa.shape
    n, kh2 = qb.shape
    _require(kh == kh2, f"K mismatch: A has {2 * kh}, B has {2 * kh2}")
    k = 2 * kh
    _require(k % 32 == 0, "K must be divisible by 32 for MXFP4 1x32 scaling.")
    _require(qa.is_contiguous() and qb.is_contiguous() and sa.is_contiguous() and sb.is_contiguous(),
             "gemm operands must be contiguous")
    _require(sa.numel() == math.prod(mx_scale_shape(m, k)) and sb.numel() == math.prod(mx_scale_shape(n, k)),
             "MXFP4 scale tensors must be the padded swizzled [round_up(rows,128), round_up(k/32,4)] layout")
    if bias is not None:
        _check_bf16(bias, "bias")
        _require(bias.numel() == n, "bias is bf16 [n]")
        bias = bias.contiguous()
    out = torch.empty((m, n), device=qa.device, dtype=torch.bfloat16)
    _lib.call("nvfp4b200_mxfp4_mm", qa.data_ptr(), qb.data_ptr(), sa.data_ptr(), sb.data_ptr(), _ptr(bias),
              out.data_ptr(), m, n, k, _stream(qa))
    return out


def gemm(qa: torch.Tensor, sa: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor, *,
         scale_a: Optional[torch.Tensor] = None, scale_b: Optional[torch.Tensor] = None,
         bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
         out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
         accumulate: bool = False, epilogue: int = EPI_NONE) -> torch.Tensor:
    """D[m, n] = epilogue(scale_a*scale_b * A.B^T + bias) + residual on packed NVFP4 operands.

    qa: [m, k/2] packed bytes, qb: [n, k/2] packed bytes (row-major, i.e. B K-major)."""
    _require(qa.is_cuda and qb.is_cuda, "gemm requires CUDA tensors")
    m, kh = qa.shape
    n, kh2 = qb.shape
    _require(kh == kh2, f"K mismatch: A has {2 * kh}, B has {2 * kh2}")
    k = 2 * kh
    _require(qa.is_contiguous() and qb.is_contiguous() and sa.is_contiguous() and sb.is_contiguous(),
             "gemm operands must be contiguous")
    _require(sa.numel() == math.prod(scale_shape(m, k)) and sb.numel() == math.prod(scale_shape(n, k)),
             "scale tensors must be the padded swizzled [round_up(rows,128), round_up(k/16,4)] layout")
    if out is None:
        _require(not accumulate, "accumulate needs an existing output")
        out = torch.empty((m, n), device=qa.device, dtype=out_dtype)
    _require(out.dtype in (torch.bfloat16, torch.float32), "output dtype must be bf16 or fp32")
    _require(out.dim() == 2 and out.shape == (m, n) and out.stride(1) == 1, "output must be [m, n] with unit column stride")
    if bias is not None:
        _check_bf16(bias, "bias")
        _require(bias.numel() == n, "bias is bf16 [n]")
        bias = bias.contiguous()
    if residual is not None:
        _check_bf16(residual, "residual")
        _require(residual.shape == (m, n) and residual.stride() == out.stride(), "residual must match the output layout")
    dt = _DT_BF16 if out.dtype == torch.bfloat16 else _DT_F32
    _lib.call("nvfp4b200_gemm", qa.data_ptr(), qb.data_ptr(), sa.data_ptr(), sb.data_ptr(),
              _ptr(_scalar_f32(scale_a, qa.device)), _ptr(_scalar_f32(scale_b, qa.device)), _ptr(bias),
              _ptr(residual), out.data_ptr(), dt, int(bool(accumulate)), int(epilogue), m, n, k, out.stride(0),
              _stream(qa))
    return out


# ----------------------------------------------------------------------------
# training-step element-wise kernels
# ----------------------------------------------------------------------------


def swiglu_fwd(gu: torch.Tensor, with_scale: bool = False, interleave: int = 0):
    """h = silu(gate)*up for gu bf16 [T, 2F] ([gate | up] per row, or gate/up
    alternating in blocks of ``interleave`` = 128 columns); optionally also g(h)."""
    _check_bf16(gu, "swiglu_fwd")
    t, f2 = gu.shape
    f = f2 // 2
    h = torch.empty((t, f), device=gu.device, dtype=torch.bfloat16)
    g = torch.empty((1,), device=gu.device, dtype=torch.float32) if with_scale else None
    ws = workspace(gu.device) if with_scale else None
    _lib.call("nvfp4b200_swiglu_fwd", gu.data_ptr(), h.data_ptr(), t, f, int(interleave), _ptr(ws), _ptr(g),
              _stream(gu))
    return (h, g) if with_scale else h


def swiglu_bwd(gu: torch.Tensor, dh: torch.Tensor, with_scale: bool = False, interleave: int = 0):
    _check_bf16(gu, "swiglu_bwd")
    t, f2 = gu.shape
    f = f2 // 2
    dh = dh.contiguous()
    dgu = torch.empty_like(gu)
    g = torch.empty((1,), device=gu.device, dtype=torch.float32) if with_scale else None
    ws = workspace(gu.device) if with_scale else None
    _lib.call("nvfp4b200_swiglu_bwd", gu.data_ptr(), dh.data_ptr(), dgu.data_ptr(), t, f, int(interleave), _ptr(ws),
              _ptr(g), _stream(gu))
    return (dgu, g) if with_scale else dgu


def gemm_swiglu(qa: torch.Tensor, sa: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor, *,
                scale_a: Optional[torch.Tensor] = None, scale_b: Optional[torch.Tensor] = None,
                store_gu: bool = True, with_scale: bool = True):
    """Gate/up GEMM with SwiGLU in the epilogue.  qb's rows interleave gate and
    up weights in blocks of 128.  Returns (h [m, n/2], gu [m, n] or None,
    g(h) or None), all bf16 except the fp32 global scale."""
    _require(qa.is_cuda and qb.is_cuda, "gemm_swiglu requires CUDA tensors")
    m, kh = qa.shape
    n, kh2 = qb.shape
    _require(kh == kh2, f"K mismatch: A has {2 * kh}, B has {2 * kh2}")
    _require(n % 256 == 0, "gemm_swiglu needs n (= 2F) % 256 == 0")
    k = 2 * kh
    _require(qa.is_contiguous() and qb.is_contiguous() and sa.is_contiguous() and sb.is_contiguous(),
             "gemm operands must be contiguous")
    _require(sa.numel() == math.prod(scale_shape(m, k)) and sb.numel() == math.prod(scale_shape(n, k)),
             "scale tensors must be the padded swizzled [round_up(rows,128), round_up(k/16,4)] layout")
    h = torch.empty((m, n // 2), device=qa.device, dtype=torch.bfloat16)
    gu = torch.empty((m, n), device=qa.device, dtype=torch.bfloat16) if store_gu else None
    g = torch.empty((1,), device=qa.device, dtype=torch.float32) if with_scale else None
    ws = workspace(qa.device) if with_scale else None
    _lib.call("nvfp4b200_gemm_swiglu", qa.data_ptr(), qb.data_ptr(), sa.data_ptr(), sb.data_ptr(),
              _ptr(_scalar_f32(scale_a, qa.device)), _ptr(_scalar_f32(scale_b, qa.device)), h.data_ptr(), _ptr(gu),
              _ptr(ws), _ptr(g), m, n, k, _stream(qa))
    return h, gu, g


def gemm_dswiglu(qa: torch.Tensor, sa: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor, gu: torch.Tensor, *,
                 scale_a: Optional[torch.Tensor] = None, scale_b: Optional[torch.Tensor] = None,
                 with_scale: bool = True):
    """dh GEMM (A = dy [m, k], B = W_down^T [n, k]) with the SwiGLU backward in
    the epilogue against gu [m, 2n] (gate/up interleaved in blocks of 128).
    Returns (dgu bf16 [m, 2n], g(dgu) or None); dh itself is not stored."""
    _require(qa.is_cuda and qb.is_cuda and gu.is_cuda, "gemm_dswiglu requires CUDA tensors")
    m, kh = qa.shape
    n, kh2 = qb.shape
    _require(kh == kh2, f"K mismatch: A has {2 * kh}, B has {2 * kh2}")
    _require(n % 256 == 0, "gemm_dswiglu needs n (= F) % 256 == 0")
    _check_bf16(gu, "gu")
    _require(tuple(gu.shape) == (m, 2 * n) and gu.is_contiguous(), "gu must be contiguous bf16 [m, 2n]")
    k = 2 * kh
    _require(qa.is_contiguous() and qb.is_contiguous() and sa.is_contiguous() and sb.is_contiguous(),
             "gemm operands must be contiguous")
    _require(sa.numel() == math.prod(scale_shape(m, k)) and sb.numel() == math.prod(scale_shape(n, k)),
             "scale tensors must be the padded swizzled [round_up(rows,128), round_up(k/16,4)] layout")
    dgu = torch.empty((m, 2 * n), device=qa.device, dtype=torch.bfloat16)
    g = torch.empty((1,), device=qa.device, dtype=torch.float32) if with_scale else None
    ws = workspace(qa.device) if with_scale else None
    _lib.call("nvfp4b200_gemm_dswiglu", qa.data_ptr(), qb.data_ptr(), sa.data_ptr(), sb.data_ptr(),
              _ptr(_scalar_f32(scale_a, qa.device)), _ptr(_scalar_f32(scale_b, qa.device)), gu.data_ptr(),
              dgu.data_ptr(), _ptr(ws), _ptr(g), m, n, k, _stream(qa))
    return dgu, g


def rmsnorm_bwd(x: torch.Tensor, gamma: Optional[torch.Tensor], inv_rms: torch.Tensor, dy: torch.Tensor,
                dres: Optional[torch.Tensor] = None, dgamma_acc: Optional[torch.Tensor] = None) -> torch.Tensor:
    r, k = x.shape
    dx = torch.empty_like(x)
    _lib.call("nvfp4b200_rmsnorm_bwd", x.data_ptr(), _ptr(gamma), inv_rms.data_ptr(), dy.contiguous().data_ptr(),
              _ptr(dres), dx.data_ptr(), _ptr(dgamma_acc), r, k, _stream(x))
    return dx


def add_bf16(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty_like(a) if out is None else out
    _lib.call("nvfp4b200_add_bf16", a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream(a))
    return out


def adamw_step(param: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor, *, lr: float,
               beta1: float, beta2: float, eps: float, weight_decay: float, step: int,
               grad_scale: float = 1.0) -> None:
    _require(param.dtype == torch.bfloat16 and m.dtype == torch.float32 and v.dtype == torch.float32,
             "AdamW: bf16 parameter, fp32 moments")
    _require(grad.dtype in (torch.bfloat16, torch.float32), "AdamW: bf16 or fp32 gradient")
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    _lib.call("nvfp4b200_adamw_step", param.data_ptr(), grad.data_ptr(),
              _DT_BF16 if grad.dtype == torch.bfloat16 else _DT_F32, m.data_ptr(), v.data_ptr(), param.numel(),
              lr, beta1, beta2, eps, weight_decay, bc1, bc2, grad_scale, _stream(param))


def adamw_master_step(param: torch.Tensor, master: torch.Tensor, grad: torch.Tensor, m: torch.Tensor,
                      v: torch.Tensor, *, lr: float, beta1: float, beta2: float, eps: float, weight_decay: float,
                      step: int, grad_scale: float = 1.0, amax_bits: Optional[torch.Tensor] = None) -> None:
    """AdamW on an fp32 master copy (torch.optim.AdamW's operation order);
    the bf16 ``param`` receives bf16(master) after the update.  ``amax_bits``
    (a 1-element int32 CUDA tensor, zeroed by the caller) collects the
    largest |bf16 parameter| written, as float bits (atomic max)."""
    _require(param.dtype == torch.bfloat16 and master.dtype == torch.float32 and m.dtype == torch.float32
             and v.dtype == torch.float32, "AdamW: bf16 parameter, fp32 master and moments")
    _require(grad.dtype in (torch.bfloat16, torch.float32), "AdamW: bf16 or fp32 gradient")
    n = param.numel()
    _require(master.numel() == n and m.numel() == n and v.numel() == n and grad.numel() == n,
             "AdamW: parameter, master, gradient and moments must have the same length")
    _lib.call("nvfp4b200_adamw_master_step", param.data_ptr(), master.data_ptr(), grad.data_ptr(),
              _DT_BF16 if grad.dtype == torch.bfloat16 else _DT_F32, m.data_ptr(), v.data_ptr(), n,
              *adamw_master_scalars(lr, beta1, beta2, eps, weight_decay, step), grad_scale, _ptr(amax_bits),
              _stream(param))


def global_scale_from_amax(amax_bits: torch.Tensor) -> torch.Tensor:
    """float32 global scales amax/(6*448) (1 for 0 or non-finite) from an int32
    tensor of amax float bits; same shape."""
    _require(amax_bits.is_cuda and amax_bits.dtype == torch.int32 and amax_bits.is_contiguous(),
             "amax bits are a contiguous int32 CUDA tensor")
    g = torch.empty(amax_bits.shape, device=amax_bits.device, dtype=torch.float32)
    _lib.call("nvfp4b200_global_scale_from_amax", amax_bits.data_ptr(), g.data_ptr(), amax_bits.numel(),
              _stream(amax_bits))
    return g


def adamw_master_scalars(lr: float, beta1: float, beta2: float, eps: float, weight_decay: float, step: int):
    """Host-side scalars of torch.optim.AdamW's step t, in the order
    nvfp4b200_adamw_master_step takes them: 1 - lr*wd, 1 - beta1, beta2,
    1 - beta2, eps, lr / (1 - beta1^t), sqrt(1 - beta2^t) (computed in
    double precision, passed as float32)."""
    return (1.0 - lr * weight_decay, 1.0 - beta1, beta2, 1.0 - beta2, eps, lr / (1.0 - beta1 ** step),
            math.sqrt(1.0 - beta2 ** step))


def device_error() -> int:
    """Read and clear the library's device error word (synchronises)."""
    import ctypes
    out = ctypes.c_int(0)
    _lib.check(_lib.load().nvfp4b200_get_device_error(ctypes.byref(out)), "nvfp4b200_get_device_error")
    return out.value
