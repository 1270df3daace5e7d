"""GPU parity of the tcgen05 NVFP4 GEMM against the oracle's dequantize ->
float64 matmul emulation.

Tolerance: the kernel accumulates exact E2M1 x E4M3 products in fp32 and
rounds once to bf16, so every element must lie within one bf16 rounding
(2^-8 relative) of the float64 emulation plus an fp32 accumulation allowance
of 2^-20 * k * max|term|; the relative Frobenius error over the matrix must
also be <= 1e-2 (the stated bar).
"""
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
REL_FROB_TOL = 1e-2


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def check_close(d, ref, qa, sa, qb, sb, m, n, k, scale=1.0):
    d = np.asarray(d, dtype=np.float64)
    a = np.abs(orc.dequant_nvfp4(qa, sa, m, k)).astype(np.float64)
    b = np.abs(orc.dequant_nvfp4(qb, sb, n, k)).astype(np.float64)
    mag = (a @ b.T) * abs(scale)          # sum of |terms|: bounds fp32 accumulation error
    tol = np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20 + 1e-30
    bad = np.abs(d - ref) > tol
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, worst {np.max(np.abs(d - ref) - tol)}"
    assert orc.rel_frobenius(d, ref) <= REL_FROB_TOL


def make(pkg, m, n, k, seed=0, scale_b=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", generator=g) * scale_b).to(torch.bfloat16)
    qa, sa = pkg.ops.quantize(a)
    qb, sb = pkg.ops.quantize(b)
    return qa, sa, qb, sb


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 1024, 512), (1, 8, 32), (100, 136, 96),
                                   (129, 264, 288), (300, 520, 1024), (64, 256, 4096), (384, 768, 2080)])
def test_gemm_shapes(pkg, m, n, k):
    qa, sa, qb, sb = make(pkg, m, n, k, seed=m + n + k)
    d = pkg.ops.gemm(qa, sa, qb, sb)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    ref = orc.gemm_emulation_f64(u8(qa), u8(sa), u8(qb), u8(sb), m, n, k)
    check_close(d.float().cpu().numpy(), ref, u8(qa), u8(sa), u8(qb), u8(sb), m, n, k)


def test_gemm_config0_round_trip(pkg, f4):
    """Round-trip workload: A [256x512] with outliers, W [1024x512] N(0,0.02)."""
    import golden_cases as gc
    a_bits, w_bits = gc.config0_a_w()
    to_dev = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda()
    a, w = to_dev(a_bits), to_dev(w_bits)
    c = f4.nvfp4mm(a, w)
    qa, sa = orc.quant_nvfp4(a_bits)
    qw, sw = orc.quant_nvfp4(w_bits)
    ref = orc.gemm_emulation_f64(qa, sa, qw, sw, 256, 1024, 512)
    check_close(c.float().cpu().numpy(), ref, qa, sa, qw, sw, 256, 1024, 512)
    # with per-tensor global scales (g = amax/(6*448)) the product is still the emulation
    c2 = f4.nvfp4mm(a, w, use_global_scale=True)
    ga = orc.global_scale_of(orc.bf16_bits_to_f32(a_bits))
    gw = orc.global_scale_of(orc.bf16_bits_to_f32(w_bits))
    qa2, sa2 = orc.quant_nvfp4(a_bits, ga)
    qw2, sw2 = orc.quant_nvfp4(w_bits, gw)
    ref2 = orc.gemm_emulation_f64(qa2, sa2, qw2, sw2, 256, 1024, 512, output_scale=np.float32(ga * gw))
    check_close(c2.float().cpu().numpy(), ref2, qa2, sa2, qw2, sw2, 256, 1024, 512, scale=float(ga * gw))
    # and much closer to the unquantized product than the g = 1 path on the small-valued W
    exact = orc.bf16_bits_to_f32(a_bits).astype(np.float64) @ orc.bf16_bits_to_f32(w_bits).astype(np.float64).T
    assert orc.rel_frobenius(c2.float().cpu().numpy(), exact) < orc.rel_frobenius(c.float().cpu().numpy(), exact)


def test_gemm_matches_reference_golden(pkg):
    """Same operands as the reference's scaled_mm route (float4utils.py:427-436)."""
    gold = np.load(os.path.join(GOLDEN, "golden_gemm.npz"))
    for name in ("cfg0", "k4096"):
        m, n, k = (int(v) for v in gold[f"{name}__mnk"])
        t = lambda key: torch.from_numpy(gold[f"{name}__{key}"]).cuda()
        d = pkg.ops.gemm(t("qa"), t("sa"), t("qb"), t("sb"))
        ref = orc.bf16_bits_to_f32(gold[f"{name}__d"]).reshape(m, n)
        assert orc.rel_frobenius(d.float().cpu().numpy(), ref) < REL_FROB_TOL
        emu = orc.gemm_emulation_f64(gold[f"{name}__qa"], gold[f"{name}__sa"], gold[f"{name}__qb"],
                                     gold[f"{name}__sb"], m, n, k)
        check_close(d.float().cpu().numpy(), emu, gold[f"{name}__qa"], gold[f"{name}__sa"], gold[f"{name}__qb"],
                    gold[f"{name}__sb"], m, n, k)


@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_epilogues_bias_scale(pkg, epi):
    m, n, k = 200, 392, 640
    qa, sa, qb, sb = make(pkg, m, n, k, seed=epi)
    bias = torch.randn(n, device="cuda").to(torch.bfloat16)
    sc_a = torch.tensor([0.75], device="cuda")
    sc_b = torch.tensor([0.125], device="cuda")
    d = pkg.ops.gemm(qa, sa, qb, sb, scale_a=sc_a, scale_b=sc_b, bias=bias, epilogue=epi)
    ref = orc.gemm_emulation_f64(u8(qa), u8(sa), u8(qb), u8(sb), m, n, k, output_scale=np.float32(0.75 * 0.125),
                                 bias_bf16_bits=bits(bias))
    if epi >= 1:
        ref = np.maximum(ref, 0.0)
    if epi == 2:
        ref = ref * ref
    got = d.float().cpu().numpy()
    tol = np.abs(ref) * 2.0 ** -7 + 1e-2 * (np.abs(ref).mean() + 1e-6)
    assert np.all(np.abs(got - ref) <= tol)
    assert orc.rel_frobenius(got, ref) <= REL_FROB_TOL


def test_gemm_f32_accumulate_and_residual(pkg):
    m, n, k = 160, 264, 512
    qa, sa, qb, sb = make(pkg, m, n, k, seed=5)
    ref = orc.gemm_emulation_f64(u8(qa), u8(sa), u8(qb), u8(sb), m, n, k)
    out = torch.full((m, n), 2.0, device="cuda", dtype=torch.float32)
    pkg.ops.gemm(qa, sa, qb, sb, out=out, accumulate=True)
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - (ref + 2.0)) <= 1e-4 * (np.abs(ref) + 2.0))
    d32 = pkg.ops.gemm(qa, sa, qb, sb, out_dtype=torch.float32)
    assert np.all(np.abs(d32.cpu().numpy() - ref) <= 1e-4 * np.abs(ref) + 1e-4)
    res = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    dr = pkg.ops.gemm(qa, sa, qb, sb, residual=res)
    want = ref + orc.bf16_bits_to_f32(bits(res)).astype(np.float64)
    assert orc.rel_frobenius(dr.float().cpu().numpy(), want) < 1e-2


def test_gemm_f32_strided_output_store_then_reduce_add(pkg):
    """fp32 results go out through TMA stores (overwrite) and TMA reduce-adds
    (accumulate) into a column window of a wider matrix; the columns around
    the window stay untouched."""
    m, n, k = 300, 520, 256
    qa, sa, qb, sb = make(pkg, m, n, k, seed=9)
    ref = orc.gemm_emulation_f64(u8(qa), u8(sa), u8(qb), u8(sb), m, n, k)
    big = torch.full((m, 1024), -7.0, device="cuda", dtype=torch.float32)
    out = big[:, 8:8 + n]
    pkg.ops.gemm(qa, sa, qb, sb, out=out)
    pkg.ops.gemm(qa, sa, qb, sb, out=out, accumulate=True)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - 2 * ref) <= 2e-4 * np.abs(ref) + 2e-4)
    rest = torch.cat([big[:, :8], big[:, 8 + n:]], dim=1)
    assert torch.all(rest == -7.0)


def test_gemm_8192_cubed_sampled(pkg):
    """Headline GEMM size: check 256 sampled output elements against float64."""
    m = n = k = 8192
    qa, sa, qb, sb = make(pkg, m, n, k, seed=1)
    d = pkg.ops.gemm(qa, sa, qb, sb)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(m, 16, replace=False))
    cols = np.sort(rng.choice(n, 16, replace=False))
    qa_r = u8(qa[torch.from_numpy(rows).cuda()])
    qb_r = u8(qb[torch.from_numpy(cols).cuda()])
    sa_all, sb_all = u8(sa), u8(sb)
    ca = orc.unswizzle_scales(sa_all, m, k)[rows]
    cb = orc.unswizzle_scales(sb_all, n, k)[cols]
    va = orc.e2m1_decode(orc.unpack_nibbles(qa_r)).reshape(16, -1, 16) * orc.e4m3_decode(ca)[..., None]
    vb = orc.e2m1_decode(orc.unpack_nibbles(qb_r)).reshape(16, -1, 16) * orc.e4m3_decode(cb)[..., None]
    ref = va.reshape(16, k).astype(np.float64) @ vb.reshape(16, k).astype(np.float64).T
    got = d[torch.from_numpy(rows).cuda()][:, torch.from_numpy(cols).cuda()].float().cpu().numpy()
    mag = np.abs(va.reshape(16, k)).astype(np.float64) @ np.abs(vb.reshape(16, k)).astype(np.float64).T
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20)


def test_gn_kernels_op_contract(pkg, f4):
    """cutlass_nvfp4_mm(a, b.mT, s_a, s_b, output_scale) as float4utils.py:456 calls it."""
    a = torch.randn(130, 256, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(72, 256, device="cuda", dtype=torch.bfloat16)
    qa, sa = f4.quant_nvfp4_fused(a)
    qb, sb = f4.quant_nvfp4_fused(b)
    assert qa.dtype == f4.FP4_DTYPE and sa.dtype == f4.FP8_SCALE_DTYPE
    one = torch.tensor(1.0, device="cuda")
    for op in (f4.cutlass_nvfp4_mm, f4.cutlass_nvfp4_mm_relu, f4.cutlass_nvfp4_mm_relu_2):
        d = op(qa, qb.mT, sa, sb, one)
        assert d.shape == (130, 72) and d.dtype == torch.bfloat16
    d0 = f4.cutlass_nvfp4_mm(qa, qb.mT, sa, sb, one)
    d1 = f4.cutlass_nvfp4_mm_relu(qa, qb.mT, sa, sb, one)
    d2 = f4.cutlass_nvfp4_mm_relu_2(qa, qb.mT, sa, sb, one)
    assert torch.equal(d1, torch.relu(d0))
    assert torch.allclose(d2.float(), torch.relu(d0.float()) ** 2, rtol=2e-2, atol=1e-2)
