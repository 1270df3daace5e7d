"""GPU parity of the MXFP4 GEMM (E2M1 operands, one UE8M0 scale per 1x32
block; the reference's cutlass_sm120a_mxfp4_mm, cutlass_mm_fp4.cu:71-165)
against the oracle's dequantize -> float64 matmul emulation.

Same tolerance as the NVFP4 GEMM: each element within one bf16 rounding
(2^-8 relative) of the emulation plus 2^-20 * sum|terms| for fp32
accumulation, and relative Frobenius error <= 1e-2."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
REL_FROB_TOL = 1e-2


def make_mx(rows, k, rng):
    """Random packed E2M1 [rows, k/2] and swizzled UE8M0 scales (2^-9 .. 2^9),
    padding entries zero."""
    q = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    pad_r, pad_c = orc.mx_scale_shape(rows, k)
    s = np.zeros(pad_r * pad_c, dtype=np.uint8)
    rr, cc = np.meshgrid(np.arange(rows), np.arange(k // 32), indexing="ij")
    s[orc.swizzle_offset(rr, cc, pad_c)] = rng.integers(118, 137, size=(rows, k // 32), dtype=np.uint8)
    return q, s.reshape(pad_r, pad_c)


def check_close_mx(d, qa, sa, qb, sb, m, n, k, bias=None):
    ref = orc.mxfp4_gemm_emulation_f64(qa, sa, qb, sb, m, n, k, bias)
    mag = np.abs(orc.dequant_mxfp4(qa, sa, m, k)) @ np.abs(orc.dequant_mxfp4(qb, sb, n, k)).T
    tol = np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20 + 1e-30
    d = np.asarray(d, dtype=np.float64)
    bad = np.abs(d - ref) > tol
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, worst {np.max(np.abs(d - ref) - tol)}"
    assert orc.rel_frobenius(d, ref) <= REL_FROB_TOL


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (1, 8, 32), (100, 136, 96), (129, 264, 288),
                                   (300, 520, 1024), (64, 256, 4096), (384, 768, 2080)])
def test_mxfp4_gemm_shapes(pkg, m, n, k):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    qa, sa = make_mx(m, k, rng)
    qb, sb = make_mx(n, k, rng)
    d = pkg.ops.mxfp4_mm(dev(qa), dev(sa), dev(qb), dev(sb))
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    check_close_mx(d.float().cpu().numpy(), qa, sa, qb, sb, m, n, k)


def test_mxfp4_gemm_bias_and_op_contract(pkg):
    """bias add, and the gn_kernels-shaped op (B passed as the column-major
    [K/2, N] view) giving the same bits as the direct call."""
    from nvfp4_b200 import gn_kernels
    m, n, k = 257, 384, 640
    rng = np.random.default_rng(5)
    qa, sa = make_mx(m, k, rng)
    qb, sb = make_mx(n, k, rng)
    bias = (torch.randn(n) * 4).to(torch.bfloat16)
    d = pkg.ops.mxfp4_mm(dev(qa), dev(sa), dev(qb), dev(sb), bias=bias.cuda())
    d_op = gn_kernels.cutlass_mxfp4_mm(dev(qa), dev(qb).mT, dev(sa), dev(sb), bias.cuda())
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    assert torch.equal(d.view(torch.int16), d_op.view(torch.int16))
    bias_bits = bias.view(torch.int16).numpy().view(np.uint16)
    check_close_mx(d.float().cpu().numpy(), qa, sa, qb, sb, m, n, k, bias=bias_bits)


def test_mxfp4_gemm_full_size_sampled(pkg):
    """8192^3 MXFP4 GEMM: 256 sampled output elements against float64."""
    m = n = k = 8192
    rng = np.random.default_rng(11)
    qa, sa = make_mx(m, k, rng)
    qb, sb = make_mx(n, k, rng)
    d = pkg.ops.mxfp4_mm(dev(qa), dev(sa), dev(qb), dev(sb)).float().cpu().numpy()
    assert pkg.ops.device_error() == 0
    ri = rng.integers(0, m, 16)
    ci = rng.integers(0, n, 16)
    a = orc.dequant_mxfp4(qa[ri], _rows(sa, ri, k), 16, k)
    b = orc.dequant_mxfp4(qb[ci], _rows(sb, ci, k), 16, k)
    ref = a @ b.T
    mag = np.abs(a) @ np.abs(b).T
    tol = np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20
    assert (np.abs(d[np.ix_(ri, ci)] - ref) <= tol).all()


def _rows(s, idx, k):
    """Scale tensor of the rows ``idx`` only (re-swizzled for a 16-row matrix)."""
    pad_r, pad_c = orc.mx_scale_shape(s.shape[0], k)
    flat = np.ascontiguousarray(s).reshape(-1)
    out_r, out_c = orc.mx_scale_shape(len(idx), k)
    out = np.zeros(out_r * out_c, dtype=np.uint8)
    rr, cc = np.meshgrid(np.arange(len(idx)), np.arange(k // 32), indexing="ij")
    out[orc.swizzle_offset(rr, cc, out_c)] = flat[orc.swizzle_offset(np.asarray(idx)[rr], cc, pad_c)]
    return out
