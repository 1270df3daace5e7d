"""GPU parity of the NVFP4 SwiGLU MLP block (forward, dgrad, wgrad) against the
oracle's dequantize -> float64 matmul emulation.  Tolerance: relative
Frobenius error <= 1e-2 on every bf16 output (intermediate bf16 rounding may
flip single nibbles downstream; the stated bar absorbs that)."""
import pytest
import torch

from oracle import mlp_oracle, nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
TOL = 1e-2


def f32(t):
    return t.detach().float().cpu().numpy()


def test_block_forward_backward_matches_emulation(pkg):
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 256, 256, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(t, d, device="cuda", generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(d, device="cuda", generator=g)).to(torch.bfloat16)
    w_gu = (0.02 * torch.randn(2 * f, d, device="cuda", generator=g)).to(torch.bfloat16)
    w_down = (0.02 * torch.randn(d, f, device="cuda", generator=g)).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=g)).to(torch.bfloat16)
    qw = mlp.quantize_weights(w_gu, w_down)
    y, sv = mlp.block_forward(x, gamma, qw)
    gg = torch.zeros(d, device="cuda")
    dgu = torch.empty(2 * f, d, device="cuda", dtype=torch.bfloat16)
    dd = torch.empty(d, f, device="cuda", dtype=torch.bfloat16)
    dx = mlp.block_backward(dy, gamma, qw, sv, gg, dgu, dd, accumulate=False)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0

    inv = sv.inv_rms.cpu().numpy()
    ey, esv = mlp_oracle.block_forward(f32(x), f32(gamma), f32(w_gu), f32(w_down), inv)
    assert orc.rel_frobenius(f32(y), ey) < TOL
    assert orc.rel_frobenius(f32(sv.gu), esv["gu"]) < TOL
    edx, edg, edgu, edd = mlp_oracle.block_backward(f32(dy), f32(x), f32(gamma), f32(w_gu), f32(w_down), inv, esv)
    assert orc.rel_frobenius(f32(dx), edx) < TOL
    assert orc.rel_frobenius(f32(dd), edd) < 2 * TOL
    assert orc.rel_frobenius(f32(dgu), edgu) < 2 * TOL
    assert orc.rel_frobenius(gg.cpu().numpy(), edg) < 2 * TOL


def test_autograd_module_close_to_bf16_reference(pkg):
    """NVFP4 module vs an unquantized torch fp32 computation of the same block:
    NVFP4 error is ~5-15% relative; gradients must point the same way."""
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    torch.manual_seed(0)
    m = mlp.NVFP4SwiGLUMLP(256, 512, device="cuda")
    x = torch.randn(128, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = m(x)
    dy = torch.randn_like(y) * 1e-2
    y.backward(dy)
    xr = x.detach().float().requires_grad_(True)
    gam = m.gamma.detach().float().requires_grad_(True)
    wgu = m.w_gu.detach().float().requires_grad_(True)
    wd = m.w_down.detach().float().requires_grad_(True)
    xn = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * gam
    gu = xn @ wgu.T
    gate, up = gu.chunk(2, dim=-1)
    yr = xr + (torch.nn.functional.silu(gate) * up) @ wd.T
    yr.backward(dy.float())
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    assert rel(y.detach(), yr.detach()) < 0.05
    assert rel(x.grad, xr.grad) < 0.3
    assert rel(m.w_down.grad, wd.grad) < 0.3
    assert rel(m.w_gu.grad, wgu.grad) < 0.3
    cos = torch.nn.functional.cosine_similarity(m.w_gu.grad.float().flatten(), wgu.grad.flatten(), dim=0)
    assert cos.item() > 0.95


def test_stack_trainer_microbatch_accumulation_is_exact_sum(pkg):
    """Two micro-batches accumulate fp32 wgrads: the accumulators must equal the
    sum of the two micro-batch gradients computed separately (same weights, same
    per-micro-batch scales), up to fp32 summation order."""
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 512, 256, 512
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(t, d, device="cuda", generator=g).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=g)).to(torch.bfloat16)
    tr = mlp.NVFP4MLPStackTrainer(1, d, f, seed=7, micro_tokens=256, max_local_tokens=t)
    blk = tr.blocks[0]
    p0 = blk.param.clone()
    qw = mlp.quantize_weights(blk.w_gu, blk.w_down)
    acc_gu = torch.zeros(2 * f, d, device="cuda")
    acc_dn = torch.zeros(d, f, device="cuda")
    acc_gam = torch.zeros(d, device="cuda")
    for lo in (0, 256):
        y, sv = mlp.block_forward(x[lo:lo + 256], blk.gamma, qw, interleave=tr.interleave)
        ggu = torch.empty(2 * f, d, device="cuda")
        gdn = torch.empty(d, f, device="cuda")
        mlp.block_backward(dy[lo:lo + 256], blk.gamma, qw, sv, acc_gam, ggu, gdn, accumulate=False,
                           interleave=tr.interleave)
        acc_gu += ggu
        acc_dn += gdn
    r = tr.step(x, dy)
    torch.cuda.synchronize()
    assert torch.isfinite(r).all()
    rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()
    # one rank: the fp32 accumulators are the gradient AdamW reads (no bf16 bucket copy)
    assert rel(blk.acc_gu, acc_gu) < 1e-5
    assert rel(blk.acc_down, acc_dn) < 1e-5
    assert rel(blk.grad_gamma32, acc_gam) < 1e-2
    # AdamW moved the parameters by at most ~lr per element
    delta = (blk.param.float() - p0.float()).abs()
    assert 0 < delta.max().item() < 1e-2
    assert pkg.ops.device_error() == 0


def test_stack_trainer_full_batch_vs_microbatch_consistent(pkg):
    """Full-batch and micro-batched steps estimate the same gradient: NVFP4
    noise differs (per-micro-batch global scales), direction must agree."""
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 512, 256, 512
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(t, d, device="cuda", generator=g).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=g)).to(torch.bfloat16)
    a = mlp.NVFP4MLPStackTrainer(2, d, f, seed=7, micro_tokens=512, max_local_tokens=t)
    b = mlp.NVFP4MLPStackTrainer(2, d, f, seed=7, micro_tokens=256, max_local_tokens=t)
    assert torch.equal(a.blocks[0].param, b.blocks[0].param)
    a.step(x, dy)
    b.step(x, dy)
    for ba, bb in zip(a.blocks, b.blocks):
        ga = ba.grad[:ba.numel].float()                       # one micro-batch: the bf16 bucket
        gb = torch.cat([bb.grad_gamma32, bb.acc_gu.flatten(), bb.acc_down.flatten()])   # fp32 accumulators
        assert ((ga - gb).norm() / ga.norm()).item() < 0.3
        assert torch.nn.functional.cosine_similarity(ga, gb, dim=0).item() > 0.95


def _interleave_rows(w_gu: torch.Tensor) -> torch.Tensor:
    """[W_gate; W_up] (2F rows) -> gate/up rows alternating in blocks of 128."""
    f = w_gu.shape[0] // 2
    idx = []
    for t in range(f // 128):
        idx += list(range(128 * t, 128 * t + 128)) + list(range(f + 128 * t, f + 128 * t + 128))
    return w_gu[torch.tensor(idx, device=w_gu.device)]


def _interleave_cols(gu: torch.Tensor) -> torch.Tensor:
    return _interleave_rows(gu.t().contiguous()).t().contiguous()


def test_gemm_swiglu_equals_gemm_then_swiglu(pkg):
    """The SwiGLU epilogue gives bit-identical gate/up, h and global scale of h
    to the plain GEMM followed by the element-wise SwiGLU kernel."""
    m, f, k = 300, 512, 384
    gen = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
    w = (0.05 * torch.randn(2 * f, k, device="cuda", generator=gen)).to(torch.bfloat16)
    ga, gw = pkg.ops.global_scale(a), pkg.ops.global_scale(w)
    qa, sa = pkg.ops.quantize(a, global_scale=ga)
    qw, sw = pkg.ops.quantize(w, global_scale=gw)
    h, gu, gh = pkg.ops.gemm_swiglu(qa, sa, qw, sw, scale_a=ga, scale_b=gw)
    gu_ref = pkg.ops.gemm(qa, sa, qw, sw, scale_a=ga, scale_b=gw)
    h_ref, gh_ref = pkg.ops.swiglu_fwd(gu_ref, with_scale=True, interleave=128)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    assert torch.equal(gu.view(torch.int16), gu_ref.view(torch.int16))
    assert torch.equal(h.view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(gh, gh_ref)
    h2, gu2, g2 = pkg.ops.gemm_swiglu(qa, sa, qw, sw, scale_a=ga, scale_b=gw, store_gu=False, with_scale=False)
    assert gu2 is None and g2 is None and torch.equal(h2.view(torch.int16), h_ref.view(torch.int16))


@pytest.mark.parametrize("m,n,k,max_sms", [(300, 512, 384, 0), (2048, 2560, 512, 0), (700, 1024, 256, 8)])
def test_gemm_dswiglu_equals_gemm_then_swiglu_bwd(pkg, m, n, k, max_sms):
    """The SwiGLU-backward epilogue gives bit-identical dgu and global scale to
    the plain dh GEMM followed by the element-wise SwiGLU backward (ragged M,
    a partial last K tile, and clusters that walk many tiles when the GEMM is
    capped to 8 SMs)."""
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    dy = (1e-3 * torch.randn(m, k, device="cuda", generator=gen)).to(torch.bfloat16)
    wdt = (0.05 * torch.randn(n, k, device="cuda", generator=gen)).to(torch.bfloat16)
    gu = (2 * torch.randn(m, 2 * n, device="cuda", generator=gen)).to(torch.bfloat16)
    ga, gw = pkg.ops.global_scale(dy), pkg.ops.global_scale(wdt)
    qa, sa = pkg.ops.quantize(dy, global_scale=ga)
    qw, sw = pkg.ops.quantize(wdt, global_scale=gw)
    try:
        pkg.ops.set_gemm_max_sms(max_sms)
        dgu, g = pkg.ops.gemm_dswiglu(qa, sa, qw, sw, gu, scale_a=ga, scale_b=gw)
        dh = pkg.ops.gemm(qa, sa, qw, sw, scale_a=ga, scale_b=gw)
    finally:
        pkg.ops.set_gemm_max_sms(0)
    dgu_ref, g_ref = pkg.ops.swiglu_bwd(gu, dh, with_scale=True, interleave=128)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    assert torch.equal(dgu.view(torch.int16), dgu_ref.view(torch.int16))
    assert torch.equal(g, g_ref)
    dgu2, g2 = pkg.ops.gemm_dswiglu(qa, sa, qw, sw, gu, scale_a=ga, scale_b=gw, with_scale=False)
    assert g2 is None and torch.equal(dgu2.view(torch.int16), dgu_ref.view(torch.int16))


def test_swiglu_interleaved_layout_equals_halves(pkg):
    t, f = 96, 256
    gen = torch.Generator(device="cuda").manual_seed(12)
    gu = torch.randn(t, 2 * f, device="cuda", generator=gen).to(torch.bfloat16)
    dh = (0.1 * torch.randn(t, f, device="cuda", generator=gen)).to(torch.bfloat16)
    h0, g0 = pkg.ops.swiglu_fwd(gu, with_scale=True)
    h1, g1 = pkg.ops.swiglu_fwd(_interleave_cols(gu), with_scale=True, interleave=128)
    assert torch.equal(h0.view(torch.int16), h1.view(torch.int16)) and torch.equal(g0, g1)
    d0, gd0 = pkg.ops.swiglu_bwd(gu, dh, with_scale=True)
    d1, gd1 = pkg.ops.swiglu_bwd(_interleave_cols(gu), dh, with_scale=True, interleave=128)
    assert torch.equal(_interleave_cols(d0).view(torch.int16), d1.view(torch.int16)) and torch.equal(gd0, gd1)


def test_block_fused_swiglu_equals_unfused(pkg):
    """A block with interleaved W_gu (SwiGLU in the GEMM epilogue) against the
    same block with [W_gate; W_up]: forward bit-identical; backward identical up
    to the row permutation except dx/dgamma, whose dgrad GEMM contracts over
    the permuted 2F dimension (fp32 summation order)."""
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 256, 256, 512
    gen = torch.Generator(device="cuda").manual_seed(13)
    x = torch.randn(t, d, device="cuda", generator=gen).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(d, device="cuda", generator=gen)).to(torch.bfloat16)
    w_gu = (0.02 * torch.randn(2 * f, d, device="cuda", generator=gen)).to(torch.bfloat16)
    w_down = (0.02 * torch.randn(d, f, device="cuda", generator=gen)).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=gen)).to(torch.bfloat16)
    w_il = _interleave_rows(w_gu)
    outs = []
    for wg, il in ((w_gu, 0), (w_il, 128)):
        qw = mlp.quantize_weights(wg, w_down)
        y, sv = mlp.block_forward(x, gamma, qw, interleave=il)
        gg = torch.zeros(d, device="cuda")
        dgu = torch.empty(2 * f, d, device="cuda", dtype=torch.bfloat16)
        dd = torch.empty(d, f, device="cuda", dtype=torch.bfloat16)
        dx = mlp.block_backward(dy, gamma, qw, sv, gg, dgu, dd, accumulate=False, interleave=il)
        outs.append((y, sv.h, dx, gg, dgu, dd))
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    (y0, h0, dx0, gg0, dgu0, dd0), (y1, h1, dx1, gg1, dgu1, dd1) = outs
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
    assert torch.equal(h0.view(torch.int16), h1.view(torch.int16))
    assert torch.equal(dd0.view(torch.int16), dd1.view(torch.int16))
    assert torch.equal(_interleave_rows(dgu0).view(torch.int16), dgu1.view(torch.int16))
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert rel(dx1, dx0) < 1e-2 and rel(gg1, gg0) < 1e-2
