"""GPU parity of the reference's Python API as this package keeps it
(float4utils.py:327-401, 440-515, 619-714 of the reference) and of the
reference's op names ``torch.ops.gn_kernels.cutlass_sm120a_*``
(cutlass_mm_fp4.cu:479-486), against the CPU oracle.

Quantizer outputs are compared bit-exact; GEMM outputs against the
dequantize -> float64 emulation within one bf16 rounding per element plus an
fp32 accumulation allowance, and <= 1e-2 relative Frobenius error.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-2


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def f32(t):
    return t.detach().float().cpu().numpy()


def close(got, qa, sa, qb, sb, m, n, k, scale=1.0, bias=None, epi=0):
    """got vs bf16-free float64 emulation of epi(scale * A.B^T + bias)."""
    pre = orc.gemm_emulation_f64(qa, sa, qb, sb, m, n, k, output_scale=np.float32(scale),
                                 bias_bf16_bits=None if bias is None else bits(bias))
    ref = np.maximum(pre, 0.0) if epi >= 1 else pre
    if epi == 2:
        ref = ref * ref
    a = np.abs(orc.dequant_nvfp4(qa, sa, m, k)).astype(np.float64)
    b = np.abs(orc.dequant_nvfp4(qb, sb, n, k)).astype(np.float64)
    # fp32 accumulation allowance; relu^2 doubles a relative error of its input
    mag = (a @ b.T) * abs(scale) * (2 * np.abs(pre) + 1 if epi == 2 else 1)
    got = np.asarray(got, dtype=np.float64)
    tol = np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20 + 1e-30
    assert np.all(np.abs(got - ref) <= tol), np.max(np.abs(got - ref) - tol)
    assert orc.rel_frobenius(got, ref) <= TOL


def test_rmsnorm_quant_nvfp4_fused_batched(f4):
    """rmsnorm_quant_nvfp4_fused on a [2, 3, 40, 512] input: shapes and dtypes of
    the reference wrapper (float4utils.py:359-401), 1/RMS per row, nibbles and
    scales bit-exact given 1/RMS."""
    gen = torch.Generator(device="cuda").manual_seed(31)
    x = (3 * torch.randn(2, 3, 40, 512, device="cuda", generator=gen)).to(torch.bfloat16)
    q, s, inv = f4.rmsnorm_quant_nvfp4_fused(x, epsilon=1e-5)
    assert q.dtype == f4.FP4_DTYPE and s.dtype == f4.FP8_SCALE_DTYPE and inv.dtype == torch.float32
    assert q.shape == (2, 3, 40, 256) and inv.shape == (2, 3, 40)
    assert s.shape == (256, 32)                                 # round_up(240, 128), round_up(512/16, 4)
    xb = bits(x.reshape(-1, 512))
    inv_np = inv.reshape(-1).cpu().numpy()
    inv64 = orc.rms_inv(xb, 1e-5)
    assert np.all(np.abs(inv_np - inv64) <= 2e-6 * inv64)
    oq, os_ = orc.rmsnorm_quant_nvfp4(xb, inv_np)
    assert np.array_equal(u8(q).reshape(240, 256), oq) and np.array_equal(u8(s), os_)
    with pytest.raises(RuntimeError):
        f4.rmsnorm_quant_nvfp4_fused(x.float())


@pytest.mark.parametrize("fn,epi", [("nvfp4mm", 0), ("nvfp4mm_relu", 1), ("nvfp4mm_relu_2", 2)])
@pytest.mark.parametrize("rms", [False, True])
def test_nvfp4mm_family(f4, fn, epi, rms):
    """nvfp4mm / nvfp4mm_relu / nvfp4mm_relu_2 (float4utils.py:440-515), with and
    without the fused RMSNorm of the left operand."""
    m, n, k = 192, 264, 640
    gen = torch.Generator(device="cuda").manual_seed(epi * 2 + rms)
    a = (2 * torch.randn(m, k, device="cuda", generator=gen)).to(torch.bfloat16)
    b = (0.1 * torch.randn(n, k, device="cuda", generator=gen)).to(torch.bfloat16)
    out = getattr(f4, fn)(a, b, apply_rmsnorm_lhs=rms, rms_eps=1e-6)
    if rms:
        c, inv = out
        assert inv.shape == (m,)
        inv_np = inv.cpu().numpy()
        qa, sa = orc.rmsnorm_quant_nvfp4(bits(a), inv_np)
    else:
        c = out
        qa, sa = orc.quant_nvfp4(bits(a))
    qb, sb = orc.quant_nvfp4(bits(b))
    assert c.shape == (m, n) and c.dtype == torch.bfloat16
    close(f32(c), qa, sa, qb, sb, m, n, k, epi=epi)


def test_nvfp4mm_global_scale_option(f4):
    m, n, k = 130, 200, 256
    gen = torch.Generator(device="cuda").manual_seed(41)
    a = (1e-3 * torch.randn(m, k, device="cuda", generator=gen)).to(torch.bfloat16)
    b = (50 * torch.randn(n, k, device="cuda", generator=gen)).to(torch.bfloat16)
    c = f4.nvfp4mm(a, b, use_global_scale=True)
    ga = orc.global_scale_of(orc.bf16_bits_to_f32(bits(a)))
    gb = orc.global_scale_of(orc.bf16_bits_to_f32(bits(b)))
    qa, sa = orc.quant_nvfp4(bits(a), ga)
    qb, sb = orc.quant_nvfp4(bits(b), gb)
    close(f32(c), qa, sa, qb, sb, m, n, k, scale=float(np.float32(ga) * np.float32(gb)))


@pytest.mark.parametrize("nvfp4_backward", [False, True])
def test_nvfp4_linear_forward_backward(f4, nvfp4_backward):
    """NVFP4Linear with bias on a 3-D input (float4utils.py:619-714): forward is
    the NVFP4 GEMM plus bias; the backward is the reference's bf16 one by
    default, NVFP4 dgrad/wgrad with per-tensor global scales otherwise."""
    torch.manual_seed(5)
    lin = f4.NVFP4Linear(256, 192, bias=True, device="cuda", nvfp4_backward=nvfp4_backward)
    x = torch.randn(2, 64, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = lin(x)
    assert y.shape == (2, 64, 192) and y.dtype == torch.bfloat16
    dy = (0.1 * torch.randn(2, 64, 192, device="cuda")).to(torch.bfloat16)
    y.backward(dy)
    torch.cuda.synchronize()
    x2, w, b = bits(x.detach().reshape(128, 256)), bits(lin.weight), lin.bias.detach()
    if nvfp4_backward:
        gx = orc.global_scale_of(orc.bf16_bits_to_f32(x2))
        gw = orc.global_scale_of(orc.bf16_bits_to_f32(w))
    else:
        gx = gw = None
    qa, sa = orc.quant_nvfp4(x2, gx)
    qb, sb = orc.quant_nvfp4(w, gw)
    scale = 1.0 if gx is None else float(np.float32(gx) * np.float32(gw))
    # forward: bf16(out) then `out += bias` in bf16 (float4utils.py:640-648)
    ref = orc.gemm_emulation_bf16(qa, sa, qb, sb, 128, 192, 256, output_scale=np.float32(scale))
    ref = orc.bf16_bits_to_f32(orc.f32_to_bf16_bits((ref + f32(b)[None, :]).astype(np.float32)))
    assert orc.rel_frobenius(f32(y.reshape(128, 192)), ref) < TOL
    dyb = bits(dy.reshape(128, 192))
    dyf = orc.bf16_bits_to_f32(dyb).astype(np.float64)
    assert np.allclose(f32(lin.bias.grad), dyf.sum(0), rtol=2e-2, atol=2e-2)
    if not nvfp4_backward:
        # torch bf16 matmuls, as the reference does
        gi = dyf @ orc.bf16_bits_to_f32(w).astype(np.float64)
        gw_ = dyf.T @ orc.bf16_bits_to_f32(x2).astype(np.float64)
        assert orc.rel_frobenius(f32(x.grad.reshape(128, 256)), gi) < TOL
        assert orc.rel_frobenius(f32(lin.weight.grad), gw_) < TOL
        return
    g_dy = orc.global_scale_of(orc.bf16_bits_to_f32(dyb))
    # dgrad: Q(dy) . Q_t(W)^T, wgrad: Q_t(dy) . Q_t(x)^T, each along its contraction dim
    qd, sd = orc.quant_nvfp4(dyb, g_dy)
    qwt, swt = orc.quant_nvfp4(np.ascontiguousarray(w.T), gw)
    close(f32(x.grad.reshape(128, 256)), qd, sd, qwt, swt, 128, 256, 192, scale=float(np.float32(g_dy) * np.float32(gw)))
    qdt, sdt = orc.quant_nvfp4(np.ascontiguousarray(dyb.T), g_dy)
    qxt, sxt = orc.quant_nvfp4(np.ascontiguousarray(x2.T), gx)
    close(f32(lin.weight.grad), qdt, sdt, qxt, sxt, 192, 256, 128, scale=float(np.float32(g_dy) * np.float32(gx)))


def test_gn_kernels_reference_op_names(pkg, f4):
    """torch.ops.gn_kernels.cutlass_sm120a_* resolve to this library (the names
    cutlass_mm_fp4.cu:479-486 registers) and equal the package's GEMM bit for bit."""
    import importlib
    gk = importlib.import_module("nvfp4_b200.gn_kernels")
    gk.register_reference_namespace()
    gen = torch.Generator(device="cuda").manual_seed(51)
    a = torch.randn(200, 512, device="cuda", generator=gen).to(torch.bfloat16)
    b = torch.randn(136, 512, device="cuda", generator=gen).to(torch.bfloat16)
    bias = torch.randn(136, device="cuda", generator=gen).to(torch.bfloat16)
    qa, sa = f4.quant_nvfp4_fused(a)
    qb, sb = f4.quant_nvfp4_fused(b)
    osc = torch.tensor(0.5, device="cuda")
    u = lambda t: t.view(torch.uint8)
    for name, epi in (("cutlass_sm120a_nvfp4_mm", 0), ("cutlass_sm120a_nvfp4_mm_relu", 1),
                      ("cutlass_sm120a_nvfp4_mm_relu_2", 2)):
        op = getattr(torch.ops.gn_kernels, name)
        for bb in (None, bias):
            d = op(qa, qb.mT, sa, sb, osc, bb)
            ref = pkg.ops.gemm(u(qa), u(sa), u(qb), u(sb), scale_a=osc.reshape(1), bias=bb, epilogue=epi)
            assert torch.equal(d.view(torch.int16), ref.view(torch.int16)), name
    # MXFP4 (cutlass_mm_fp4.cu:71-165): UE8M0 scales, no output scale
    mqa = torch.randint(0, 256, (200, 256), dtype=torch.uint8, device="cuda", generator=gen)
    mqb = torch.randint(0, 256, (136, 256), dtype=torch.uint8, device="cuda", generator=gen)
    msa = torch.randint(120, 135, pkg.ops.mx_scale_shape(200, 512), dtype=torch.uint8, device="cuda", generator=gen)
    msb = torch.randint(120, 135, pkg.ops.mx_scale_shape(136, 512), dtype=torch.uint8, device="cuda", generator=gen)
    d = torch.ops.gn_kernels.cutlass_sm120a_mxfp4_mm(mqa, mqb.mT, msa, msb, bias)
    ref = pkg.ops.mxfp4_mm(mqa, msa, mqb, msb, bias)
    assert torch.equal(d.view(torch.int16), ref.view(torch.int16))
    emu = orc.mxfp4_gemm_emulation_f64(u8(mqa), u8(msa), u8(mqb), u8(msb), 200, 136, 512, bias_bf16_bits=bits(bias))
    assert orc.rel_frobenius(f32(d), emu) < TOL
