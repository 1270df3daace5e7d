"""CPU oracle for the NVFP4 hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (the package's CUDA
library) never calls into this file, and fails loudly when its extension is
missing instead of falling back here.

It restates, in vectorised numpy, the arithmetic of the reference quantizer
kernels in ``float4utils.py`` (xTimeCrystal/NVFP4.5090):

* ``quant_nvfp4_fused_opt``         float4utils.py:79-148
* ``rmsnorm_quant_nvfp4_smem_opt``  float4utils.py:169-295
* E4M3 encode/decode helpers         float4utils.py:64-77
* the 128x4 scale swizzle            float4utils.py:118-123
* the wrapper shapes/padding         float4utils.py:327-401

and the GEMM contract of ``cutlass_sm120a_nvfp4_mm``
(cutlass_mm_fp4.cu:167-272): D = bf16(output_scale * (A . B^T) + bias), with
A and B dequantised exactly (E2M1 value x E4M3 block scale) and the
contraction done in float64.

Parity pin: the quantizer restatement is checked bit-for-bit against golden
vectors produced by the reference's own kernels (compiled from their source
by ``oracle/build_ref.py`` and run by ``tests/golden/make_golden.py``); the
GEMM emulation is checked against the reference's on-Blackwell GEMM route
(``torch.nn.functional.scaled_mm`` with BlockWise1x16 / SWIZZLE_32_4_4,
float4utils.py:427-436) on the same golden inputs.

Extension beyond the reference (per-tensor global scale ``g``): block scale
``e4m3((amax_blk * (1/6)) * (1/g))`` and element multiplier
``1 / (scale_fq * g)``.  With ``g = 1`` both reduce exactly to the reference's
``e4m3(amax_blk * (1/6))`` and ``1 / scale_fq`` (multiplying a float32 by 1.0
is exact), so the reference behaviour is the ``g = 1`` special case.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

F32 = np.float32

# --------------------------------------------------------------------------
# bf16 <-> f32 (bit level)
# --------------------------------------------------------------------------


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32, the shift-by-16 of float4utils.py:101-102."""
    u16 = np.ascontiguousarray(u16, dtype=np.uint16)
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounding_bias = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding_bias) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


# --------------------------------------------------------------------------
# E4M3 (float8_e4m3fn): table-driven RNE with satfinite
# --------------------------------------------------------------------------


def _e4m3_table() -> np.ndarray:
    """Value of every non-negative finite E4M3 code 0..126 (0x7F is NaN)."""
    vals = np.empty(127, dtype=np.float64)
    for c in range(127):
        e, m = c >> 3, c & 7
        vals[c] = m * 2.0 ** -9 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_TABLE = _e4m3_table()
E4M3_MAX = 448.0


def e4m3_encode_satfinite(v: np.ndarray) -> np.ndarray:
    """float32 >= 0 -> E4M3 code, as ``cvt.rn.satfinite.e4m3x2.f32``.

    float4utils.py:64-68.  Round-to-nearest, ties to the even code; values
    above 448 (and +inf) saturate to 448 (0x7E).  Only non-negative inputs
    reach this in the quantizer (the block scale is an absolute max).
    """
    v = np.asarray(v, dtype=np.float64)
    if np.any(v < 0) or np.any(np.isnan(v)):
        raise ValueError("e4m3_encode_satfinite: expects non-negative, non-NaN input")
    v = np.minimum(v, E4M3_MAX)
    hi = np.searchsorted(E4M3_TABLE, v, side="left")  # first code with value >= v
    hi = np.minimum(hi, 126)
    lo = np.maximum(hi - 1, 0)
    d_lo = v - E4M3_TABLE[lo]
    d_hi = E4M3_TABLE[hi] - v
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(E4M3_TABLE[hi] == v, hi, code)
    return code.astype(np.uint8)


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    """E4M3 code -> float32 (float4utils.py:69-77); 0x7F/0xFF decode to NaN."""
    code = np.asarray(code, dtype=np.uint8)
    mag = code & 0x7F
    out = np.where(mag == 0x7F, np.nan, E4M3_TABLE[np.minimum(mag, 126)])
    out = np.where(code & 0x80, -out, out)
    return out.astype(np.float32)


# --------------------------------------------------------------------------
# E2M1 (float4_e2m1fn): the reference's comparison ladder
# --------------------------------------------------------------------------

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
_LADDER = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)


def e2m1_encode(f: np.ndarray, inv_scale: np.ndarray) -> np.ndarray:
    """Encode float32 values to 4-bit E2M1 codes, float4utils.py:127-140.

    ``ax = min(|f * inv_scale|, 6)`` (NaN passes the ``> 6`` test untouched),
    code = number of ladder thresholds t with ``!(ax < t)`` (ties round away
    from zero; NaN gives 7), sign bit = ``f < 0`` on the unscaled value.
    """
    f = np.asarray(f, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        ax = np.abs((f * inv_scale).astype(np.float32))
    ax = np.where(ax > F32(6.0), F32(6.0), ax)
    with np.errstate(invalid="ignore"):
        code = np.zeros(ax.shape, dtype=np.uint8)
        for t in _LADDER:
            code += (~(ax < t)).astype(np.uint8)
    sign = (f < 0).astype(np.uint8)
    return (sign << 3) | code


def e2m1_decode(nib: np.ndarray) -> np.ndarray:
    nib = np.asarray(nib, dtype=np.uint8)
    v = E2M1_VALUES[nib & 7]
    return np.where(nib & 8, -v, v).astype(np.float32)


# --------------------------------------------------------------------------
# swizzled scale layout (float4utils.py:118-123)
# --------------------------------------------------------------------------


def round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m


def scale_shape(rows: int, k: int) -> Tuple[int, int]:
    """(pad_R, pad_cols) of the scale tensor, float4utils.py:343-348."""
    return round_up(rows, 128), round_up(k // 16, 4)


def swizzle_offset(r: np.ndarray, c: np.ndarray, pad_cols: int) -> np.ndarray:
    """Byte offset of block (r, c) in the 128x4-atom swizzled scale tensor.

    float4utils.py:118-122: atom (r//128, c//4) is 512 contiguous bytes laid
    out as 32 lines of 16 bytes: line r%32 holds, for the four 32-row groups
    (r%128)//32, the four block scales c%4.
    """
    r = np.asarray(r, dtype=np.int64)
    c = np.asarray(c, dtype=np.int64)
    tile = (r >> 7) * (pad_cols >> 2) + (c >> 2)
    r_in = r & 127
    return (tile << 9) + ((r_in & 31) << 4) + ((r_in >> 5) << 2) + (c & 3)


def unswizzle_scales(s: np.ndarray, rows: int, k: int) -> np.ndarray:
    """Swizzled scale tensor -> row-major [rows, k//16] codes."""
    pad_r, pad_c = scale_shape(rows, k)
    flat = np.ascontiguousarray(s, dtype=np.uint8).reshape(-1)
    assert flat.size == pad_r * pad_c
    rr, cc = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    return flat[swizzle_offset(rr, cc, pad_c)]


# --------------------------------------------------------------------------
# quantizers
# --------------------------------------------------------------------------


def _check_g(global_scale: Optional[float]) -> F32:
    return F32(1.0) if global_scale is None else F32(global_scale)


def quant_blocks(f: np.ndarray, global_scale: Optional[float] = None):
    """Quantize float32 blocks f[..., 16] -> (nibbles[..., 16], scale codes[...]).

    float4utils.py:95-116 (amax with fmaxf semantics, NaN dropped; scale =
    satfinite-RNE E4M3 of amax*(1/6); inv_scale = 1/scale_fq or 1 when the
    decoded scale is 0) with the global scale g folded in as documented in
    the module header.
    """
    g = _check_g(global_scale)
    inv_g = F32(1.0) / g
    f = np.asarray(f, dtype=np.float32)
    amax = np.fmax.reduce(np.abs(f), axis=-1, initial=F32(0.0)).astype(np.float32)
    pos = amax > 0
    scale_f = ((amax * (F32(1.0) / F32(6.0))).astype(np.float32) * inv_g).astype(np.float32)
    scale_f = np.where(pos, scale_f, F32(0.0))
    code = e4m3_encode_satfinite(scale_f)
    code = np.where(pos, code, np.uint8(0)).astype(np.uint8)
    scale_fq = e4m3_decode(code)
    with np.errstate(divide="ignore", over="ignore"):
        denom = (scale_fq * g).astype(np.float32)
        inv_scale = np.where(scale_fq > 0, (F32(1.0) / denom).astype(np.float32), F32(1.0))
    inv_scale = np.where(pos, inv_scale, F32(1.0)).astype(np.float32)
    nib = e2m1_encode(f, inv_scale[..., None])
    return nib, code


def pack_nibbles(nib: np.ndarray) -> np.ndarray:
    """[..., 2n] nibbles -> [..., n] bytes, low nibble = even element (float4utils.py:141)."""
    nib = np.asarray(nib, dtype=np.uint8)
    return (nib[..., 0::2] & 0xF) | ((nib[..., 1::2] & 0xF) << 4)


def unpack_nibbles(q: np.ndarray) -> np.ndarray:
    q = np.asarray(q, dtype=np.uint8)
    out = np.empty(q.shape[:-1] + (q.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = q & 0xF
    out[..., 1::2] = q >> 4
    return out


def quant_nvfp4_f32(x: np.ndarray, global_scale: Optional[float] = None):
    """Quantize a float32 [R, K] matrix along K: returns (q [R, K/2] u8, s swizzled u8)."""
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    if k % 16:
        raise RuntimeError("K must be divisible by 16 for NVFP4 1x16 scaling.")
    nib, code = quant_blocks(x.reshape(rows, k // 16, 16), global_scale)
    q = pack_nibbles(nib.reshape(rows, k))
    pad_r, pad_c = scale_shape(rows, k)
    s = np.zeros(pad_r * pad_c, dtype=np.uint8)
    rr, cc = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    s[swizzle_offset(rr, cc, pad_c)] = code
    return q, s.reshape(pad_r, pad_c)


def quant_nvfp4(x_bf16_bits: np.ndarray, global_scale: Optional[float] = None):
    """``quant_nvfp4_fused`` (float4utils.py:327-357) on bf16 bit patterns [R, K]."""
    return quant_nvfp4_f32(bf16_bits_to_f32(x_bf16_bits), global_scale)


def rms_inv(x_bf16_bits: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """1/RMS of each row in float64 (float4utils.py:183-223 computes it in fp32
    with ``rsqrtf``; tests compare the kernel's value with a ulp tolerance)."""
    x = bf16_bits_to_f32(x_bf16_bits).astype(np.float64)
    return 1.0 / np.sqrt(np.mean(x * x, axis=-1) + eps)


def rmsnorm_quant_nvfp4(x_bf16_bits: np.ndarray, inv_rms: np.ndarray,
                        gamma_bf16_bits: Optional[np.ndarray] = None,
                        global_scale: Optional[float] = None):
    """``rmsnorm_quant_nvfp4_smem_opt`` phase 2 (float4utils.py:233-294) given inv_rms.

    ``f = x * inv_rms`` in float32 (float4utils.py:247-248); the optional gamma
    (not in the reference) multiplies afterwards: ``f = (x * inv_rms) * gamma``.
    """
    x = bf16_bits_to_f32(x_bf16_bits)
    f = (x * np.asarray(inv_rms, dtype=np.float32)[:, None]).astype(np.float32)
    if gamma_bf16_bits is not None:
        f = (f * bf16_bits_to_f32(gamma_bf16_bits)[None, :]).astype(np.float32)
    return quant_nvfp4_f32(f, global_scale)


def global_scale_of(x_f32: np.ndarray) -> F32:
    """g = amax/(6*448) (NaN-dropping amax); 1.0 when amax is 0 or not finite."""
    amax = F32(np.fmax.reduce(np.abs(np.asarray(x_f32, dtype=np.float32)).reshape(-1), initial=F32(0)))
    if not (amax > 0) or not np.isfinite(amax):
        return F32(1.0)
    return F32(amax / F32(2688.0))


# --------------------------------------------------------------------------
# dequantize and GEMM emulation
# --------------------------------------------------------------------------


def dequant_nvfp4(q: np.ndarray, s: np.ndarray, rows: int, k: int,
                  global_scale: Optional[float] = None) -> np.ndarray:
    """Exact dequantisation: e2m1(nibble) * e4m3(scale) [* g], as float32."""
    vals = e2m1_decode(unpack_nibbles(np.asarray(q).reshape(rows, k // 2)))
    sc = e4m3_decode(unswizzle_scales(s, rows, k)).astype(np.float32)
    out = vals.reshape(rows, k // 16, 16) * sc[:, :, None]
    if global_scale is not None:
        out = out * F32(global_scale)
    return out.reshape(rows, k).astype(np.float32)


def gemm_emulation_f64(qa, sa, qb, sb, m: int, n: int, k: int,
                       output_scale: float = 1.0,
                       bias_bf16_bits: Optional[np.ndarray] = None) -> np.ndarray:
    """float64 value of ``output_scale * dequant(A) @ dequant(B)^T + bias``.

    cutlass_mm_fp4.cu:182-184 (EVT: multiply by the scalar output scale, add
    the row-broadcast bias, cast).  A is [m, k/2] packed, B is [n, k/2] packed
    (the reference passes ``b.mT``, i.e. B column-major = B^T row-major).
    """
    a = dequant_nvfp4(qa, sa, m, k).astype(np.float64)
    b = dequant_nvfp4(qb, sb, n, k).astype(np.float64)
    d = (a @ b.T) * float(np.float32(output_scale))
    if bias_bf16_bits is not None:
        d = d + bf16_bits_to_f32(bias_bf16_bits).astype(np.float64)[None, :]
    return d


def ue8m0_decode(code: np.ndarray) -> np.ndarray:
    """UE8M0 scale byte -> 2^(code - 127) as float64 (0xFF is NaN).  The MXFP4
    scale type of cutlass_mm_fp4.cu:79 (``mx_float4_t<float_e2m1_t>``)."""
    c = np.asarray(code, dtype=np.int64)
    out = np.ldexp(1.0, c - 127)
    return np.where(c == 255, np.nan, out)


def mx_scale_shape(rows: int, k: int) -> Tuple[int, int]:
    """(pad_R, pad_cols) of an MXFP4 scale tensor: one scale per 1x32 block."""
    return round_up(rows, 128), round_up(k // 32, 4)


def dequant_mxfp4(q: np.ndarray, s: np.ndarray, rows: int, k: int) -> np.ndarray:
    """e2m1(nibble) * 2^(e - 127) per 1x32 block, as float64.  Scales sit in
    the same 128x4-atom swizzle as NVFP4's, one column per 32 k."""
    vals = e2m1_decode(unpack_nibbles(np.asarray(q).reshape(rows, k // 2))).astype(np.float64)
    pad_r, pad_c = mx_scale_shape(rows, k)
    flat = np.ascontiguousarray(s, dtype=np.uint8).reshape(-1)
    assert flat.size == pad_r * pad_c
    rr, cc = np.meshgrid(np.arange(rows), np.arange(k // 32), indexing="ij")
    sc = ue8m0_decode(flat[swizzle_offset(rr, cc, pad_c)])
    return (vals.reshape(rows, k // 32, 32) * sc[:, :, None]).reshape(rows, k)


def mxfp4_gemm_emulation_f64(qa, sa, qb, sb, m: int, n: int, k: int,
                             bias_bf16_bits: Optional[np.ndarray] = None) -> np.ndarray:
    """float64 value of ``dequant(A) @ dequant(B)^T + bias`` for the MXFP4 op
    (cutlass_mm_fp4.cu:82-83: bias add then cast, no output scale)."""
    d = dequant_mxfp4(qa, sa, m, k) @ dequant_mxfp4(qb, sb, n, k).T
    if bias_bf16_bits is not None:
        d = d + bf16_bits_to_f32(bias_bf16_bits).astype(np.float64)[None, :]
    return d


def gemm_emulation_bf16(*args, **kw) -> np.ndarray:
    """GEMM emulation rounded to bf16 (returned as float32 values)."""
    d = gemm_emulation_f64(*args, **kw).astype(np.float32)
    return bf16_bits_to_f32(f32_to_bf16_bits(d))


def rel_frobenius(d: np.ndarray, ref: np.ndarray) -> float:
    d = np.asarray(d, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = math.sqrt(float(np.sum(ref * ref)))
    return math.sqrt(float(np.sum((d - ref) ** 2))) / max(den, 1e-300)


def bytes_nvfp4_quant(rows: int, k: int) -> float:
    """Algorithmic bytes of one quantize launch, float4utils.py:534-538."""
    pad_r, pad_c = scale_shape(rows, k)
    return rows * k * 2.0 + rows * k * 0.5 + pad_r * pad_c * 1.0
