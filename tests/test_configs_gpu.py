"""GPU parity at the benchmark workloads' own sizes, against the CPU oracle.

The full-size outputs are too large to emulate whole on the CPU, so each test
checks what the domain makes independent, exactly:

* GEMM (N = K = 8192, M in {128, 1024, 8192, 16384}, per-tensor global
  scales as the benchmark uses them): 16 x 16 sampled output elements
  against float64, every one within 2^-8 |ref| + 2^-20 sum|terms|.
* RMSNorm -> NVFP4 on x [32768 x 4096] with gamma: 1/RMS of every row from
  both kernels (2e-6 relative to float64), nibbles and scale codes of 48 sampled rows
  bit-exact, the global scale of the normalised tensor exact, and the
  global-scale and transposed quantizers on sampled rows / columns bit-exact.
* One MLP block training step at 16384 tokens, d 4096, ff 14336 (the
  single-block benchmark shape, gate/up interleaved as the trainer keeps
  them): every global scale exact; forward and dgrad outputs of 8 sampled
  token rows (rows are independent given the global scales) against the
  dequantize -> float64 emulation with relative Frobenius error <= 1e-2;
  8 x 8 sampled entries of both weight gradients (each a dot product over
  all 16384 tokens) within the per-element GEMM bound; dgamma against
  float64 of the kernel's own dxn.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
F32 = np.float32
TOL = 1e-2


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def f32(t):
    return t.detach().float().cpu().numpy()


def bf16_global_scale(u16: np.ndarray) -> F32:
    """Exact g = amax/(6*448) of a bf16 tensor from its bit patterns (NaN dropped)."""
    a = (u16.reshape(-1) & np.uint16(0x7FFF)).astype(np.uint16)
    a = np.where(a > 0x7F80, np.uint16(0), a)
    amax = orc.bf16_bits_to_f32(np.array([a.max()], dtype=np.uint16))
    return orc.global_scale_of(amax)


def deq_f64(q, s, rows, k, g=None):
    """Exact dequantisation of a quantized [rows, k] operand given as numpy arrays, float64."""
    out = orc.dequant_nvfp4(q, s, rows, k).astype(np.float64)
    return out if g is None else out * float(g)


def qdq_rows(x_f32: np.ndarray, g) -> np.ndarray:
    """Oracle-quantize float32 rows along their last dimension with global scale g, dequantize (float64)."""
    x_f32 = np.ascontiguousarray(x_f32, dtype=np.float32)
    q, s = orc.quant_nvfp4_f32(x_f32, g)
    return deq_f64(q, s, *x_f32.shape) * float(g)


class DeqWeight:
    """A quantized [n, k] operand held on the CPU: row-major codes, dequantized in chunks."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor, g: torch.Tensor):
        self.n, kh = q.shape
        self.k = 2 * kh
        self.q = u8(q)
        self.codes = orc.unswizzle_scales(u8(s), self.n, self.k)
        self.g = float(g.item())

    def rows(self, lo, hi):
        vals = orc.e2m1_decode(orc.unpack_nibbles(self.q[lo:hi])).reshape(hi - lo, self.k // 16, 16)
        return (vals * orc.e4m3_decode(self.codes[lo:hi])[..., None]).reshape(hi - lo, self.k).astype(np.float64)

    def matmul_t(self, a_deq: np.ndarray) -> np.ndarray:
        """a_deq [r, k] (float64, dequantized with its global scale) @ (g * W)^T -> [r, n]."""
        out = [a_deq @ self.rows(lo, min(lo + 4096, self.n)).T for lo in range(0, self.n, 4096)]
        return np.concatenate(out, axis=1) * self.g


def bf16r(x):
    return orc.bf16_bits_to_f32(orc.f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def gemm_bound_ok(got, ref, mag):
    return np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + mag * 2.0 ** -20 + 1e-30)


# ---------------------------------------------------------------------------
# GEMM sweep with global scales
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def b_operand(pkg):
    n = k = 8192
    gen = torch.Generator(device="cuda").manual_seed(1)
    b = torch.randn(n, k, device="cuda", generator=gen).to(torch.bfloat16)
    gb = pkg.ops.global_scale(b)
    qb, sb = pkg.ops.quantize(b, global_scale=gb)
    torch.cuda.synchronize()
    assert gb.item() == float(bf16_global_scale(bits(b)))
    rows = np.array([0, 5, 4097, 8191])
    oq, _ = orc.quant_nvfp4(bits(b[torch.from_numpy(rows).cuda()]), gb.item())
    assert np.array_equal(u8(qb)[rows], oq)
    return qb, sb, gb


@pytest.mark.parametrize("m", [128, 1024, 8192, 16384])
def test_gemm_sweep_global_scales_sampled(pkg, b_operand, m):
    qb, sb, gb = b_operand
    n, k = qb.shape[0], 2 * qb.shape[1]
    gen = torch.Generator(device="cuda").manual_seed(100 + m)
    a = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
    ga = pkg.ops.global_scale(a)
    qa, sa = pkg.ops.quantize(a, global_scale=ga)
    d = pkg.ops.gemm(qa, sa, qb, sb, scale_a=ga, scale_b=gb)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    assert ga.item() == float(bf16_global_scale(bits(a)))
    rng = np.random.default_rng(m)
    rows = np.sort(rng.choice(m, 16, replace=False))
    cols = np.sort(rng.choice(n, 16, replace=False))
    ri, ci = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    oq, _ = orc.quant_nvfp4(bits(a[ri]), ga.item())        # the sampled A rows are the oracle's
    assert np.array_equal(u8(qa)[rows], oq)
    codes = orc.unswizzle_scales(u8(sa), m, k)[rows]
    va = (orc.e2m1_decode(orc.unpack_nibbles(u8(qa[ri]))).reshape(16, -1, 16)
          * orc.e4m3_decode(codes)[..., None]).reshape(16, k).astype(np.float64)
    cb = orc.unswizzle_scales(u8(sb), n, k)[cols]
    vb = (orc.e2m1_decode(orc.unpack_nibbles(u8(qb[ci]))).reshape(16, -1, 16)
          * orc.e4m3_decode(cb)[..., None]).reshape(16, k).astype(np.float64)
    alpha = float(F32(ga.item()) * F32(gb.item()))
    ref = (va @ vb.T) * alpha
    mag = (np.abs(va) @ np.abs(vb).T) * alpha
    got = d[ri][:, ci].float().cpu().numpy().astype(np.float64)
    assert gemm_bound_ok(got, ref, mag)
    assert orc.rel_frobenius(got, ref) <= TOL


# ---------------------------------------------------------------------------
# RMSNorm -> NVFP4, 32768 x 4096 with gamma
# ---------------------------------------------------------------------------

def test_rmsnorm_quant_full_size_paths(pkg):
    r, k = 32768, 4096
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(r, k, device="cuda", generator=g)
    rs = torch.exp(torch.empty(r, 1, device="cuda").uniform_(np.log(0.1), np.log(10.0), generator=g))
    x = (x * rs).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).to(torch.bfloat16)
    q, s, inv = pkg.ops.rmsnorm_quantize(x, 1e-6, gamma=gamma)          # single pass, g = 1
    inv2, gs = pkg.ops.rmsnorm_stats(x, 1e-6, gamma=gamma)             # global-scale path
    q2, s2 = pkg.ops.quantize(x, global_scale=gs, row_scale=inv2, gamma=gamma)
    qt, st = pkg.ops.quantize_t(x, global_scale=gs, row_scale=inv2, gamma=gamma)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0
    xb, gb = bits(x), bits(gamma)
    inv_np = inv.cpu().numpy()
    inv64 = orc.rms_inv(xb, 1e-6)
    assert np.all(np.abs(inv_np - inv64) <= 2e-6 * inv64)
    # the global-scale path's 1/RMS is reduced in its own order: within 2e-6 of float64 too
    inv2_np = inv2.cpu().numpy()
    assert np.all(np.abs(inv2_np - inv64) <= 2e-6 * inv64)
    y = (orc.bf16_bits_to_f32(xb) * inv2_np[:, None]).astype(np.float32) * orc.bf16_bits_to_f32(gb)[None, :]
    g_ref = orc.global_scale_of(y.astype(np.float32))
    del y
    assert gs.item() == float(g_ref)
    idx = np.sort(np.random.default_rng(2).choice(r, 48, replace=False))
    for qq, ss, gg, iv in ((q, s, None, inv_np), (q2, s2, float(g_ref), inv2_np)):
        oq, _ = orc.rmsnorm_quant_nvfp4(xb[idx], iv[idx], gb, global_scale=gg)
        assert np.array_equal(u8(qq)[idx], oq)
        xf = (orc.bf16_bits_to_f32(xb[idx]) * iv[idx, None]).astype(np.float32)
        xf = (xf * orc.bf16_bits_to_f32(gb)[None, :]).astype(np.float32)
        _, codes = orc.quant_blocks(xf.reshape(48, -1, 16), gg)
        assert np.array_equal(orc.unswizzle_scales(u8(ss), r, k)[idx], codes)
    cols = np.array([0, 3, 1000, 2049, 4095])
    xc = (orc.bf16_bits_to_f32(xb[:, cols]) * inv2_np[:, None]).astype(np.float32)
    xc = (xc * orc.bf16_bits_to_f32(gb)[cols][None, :]).astype(np.float32)
    oqt, _ = orc.quant_nvfp4_f32(np.ascontiguousarray(xc.T), float(g_ref))
    assert np.array_equal(u8(qt)[cols], oqt)
    _, ct = orc.quant_blocks(np.ascontiguousarray(xc.T).reshape(len(cols), -1, 16), float(g_ref))
    assert np.array_equal(orc.unswizzle_scales(u8(st), k, r)[cols], ct)


# ---------------------------------------------------------------------------
# MLP block training step, 16384 tokens, d 4096, ff 14336
# ---------------------------------------------------------------------------

def _gate_cols(f):
    """Interleaved gate/up layout: gate j of block t at column 256 t + j, up at +128."""
    j = np.arange(f)
    return (j // 128) * 256 + (j % 128)


def _sigmoid(x):
    return (F32(1.0) / (F32(1.0) + np.exp(-x.astype(np.float32)))).astype(np.float32)


def test_mlp_block_full_size_sampled(pkg):
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 16384, 4096, 14336
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(t, d, device="cuda", generator=gen).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(d, device="cuda", generator=gen)).to(torch.bfloat16)
    w_gu = (0.02 * torch.randn(2 * f, d, device="cuda", generator=gen)).to(torch.bfloat16)   # interleaved rows
    w_down = (0.02 * torch.randn(d, f, device="cuda", generator=gen)).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=gen)).to(torch.bfloat16)
    qw = mlp.quantize_weights(w_gu, w_down)
    y, sv = mlp.block_forward(x, gamma, qw, interleave=128)
    keep = {}
    ggam = torch.zeros(d, device="cuda")
    dwgu = torch.empty(2 * f, d, device="cuda", dtype=torch.bfloat16)
    dwd = torch.empty(d, f, device="cuda", dtype=torch.bfloat16)
    dx = mlp.block_backward(dy, gamma, qw, sv, ggam, dwgu, dwd, accumulate=False, interleave=128, keep=keep)
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == 0

    xb, gamb, dyb = bits(x), bits(gamma), bits(dy)
    xf, gamf, dyf = orc.bf16_bits_to_f32(xb), orc.bf16_bits_to_f32(gamb), orc.bf16_bits_to_f32(dyb)
    inv = sv.inv_rms.cpu().numpy()
    inv64 = orc.rms_inv(xb, 1e-6)
    assert np.all(np.abs(inv - inv64) <= 2e-6 * inv64)
    xn = ((xf * inv[:, None]).astype(np.float32) * gamf[None, :]).astype(np.float32)
    # global scales: exactly the oracle's over the whole tensors
    assert sv.g_xn.item() == float(orc.global_scale_of(xn))
    assert qw.g_gu.item() == float(bf16_global_scale(bits(w_gu)))
    assert qw.g_down.item() == float(bf16_global_scale(bits(w_down)))
    h_gpu = bits(sv.h)
    assert sv.g_h.item() == float(bf16_global_scale(h_gpu))
    assert keep["g_dy"].item() == float(bf16_global_scale(dyb))
    dgu_gpu = bits(keep["dgu"])
    assert keep["g_dgu"].item() == float(bf16_global_scale(dgu_gpu))
    g_xn, g_h, g_dy, g_dgu = (F32(v.item()) for v in (sv.g_xn, sv.g_h, keep["g_dy"], keep["g_dgu"]))

    # weight quantization, sampled rows of each orientation, bit-exact
    wr = np.array([0, 129, 20000, 2 * f - 1])
    assert np.array_equal(u8(qw.q_gu)[wr], orc.quant_nvfp4(bits(w_gu)[wr], qw.g_gu.item())[0])
    wdr = np.array([0, 77, d - 1])
    assert np.array_equal(u8(qw.q_down)[wdr], orc.quant_nvfp4(bits(w_down)[wdr], qw.g_down.item())[0])
    assert np.array_equal(u8(qw.q_gu_t)[wdr],
                          orc.quant_nvfp4(np.ascontiguousarray(bits(w_gu)[:, wdr].T), qw.g_gu.item())[0])
    assert np.array_equal(u8(qw.q_down_t)[wr[:2]],
                          orc.quant_nvfp4(np.ascontiguousarray(bits(w_down)[:, wr[:2]].T), qw.g_down.item())[0])

    W_gu = DeqWeight(qw.q_gu, qw.s_gu, qw.g_gu)            # [2F, D] along D
    W_down = DeqWeight(qw.q_down, qw.s_down, qw.g_down)    # [D, F] along F
    W_gu_t = DeqWeight(qw.q_gu_t, qw.s_gu_t, qw.g_gu)      # [D, 2F] along 2F
    W_down_t = DeqWeight(qw.q_down_t, qw.s_down_t, qw.g_down)  # [F, D] along D

    rows = np.sort(np.random.default_rng(3).choice(t, 8, replace=False))
    ri = torch.from_numpy(rows).cuda()
    gc = _gate_cols(f)
    # forward
    gu_r = bf16r(W_gu.matmul_t(qdq_rows(xn[rows], g_xn)))
    gate, up = gu_r[:, gc], gu_r[:, gc + 128]
    h_r = bf16r(gate * _sigmoid(gate) * up)
    y_r = bf16r(W_down.matmul_t(qdq_rows(h_r, g_h)) + xf[rows].astype(np.float64))
    assert orc.rel_frobenius(f32(sv.gu[ri]), gu_r) < TOL
    assert orc.rel_frobenius(orc.bf16_bits_to_f32(h_gpu[rows]), h_r) < TOL
    assert orc.rel_frobenius(f32(y[ri]), y_r) < TOL
    # dgrad
    dh_r = bf16r(W_down_t.matmul_t(qdq_rows(dyf[rows], g_dy)))
    s_ = _sigmoid(gate)
    dgu_r = np.empty_like(gu_r)
    dgu_r[:, gc + 128] = bf16r(dh_r * (gate * s_))
    dgu_r[:, gc] = bf16r(dh_r * up * (s_ * (F32(1.0) + gate * (F32(1.0) - s_))))
    assert orc.rel_frobenius(orc.bf16_bits_to_f32(dgu_gpu[rows]), dgu_r) < TOL
    dxn_r = bf16r(W_gu_t.matmul_t(qdq_rows(dgu_r, g_dgu)))
    assert orc.rel_frobenius(f32(keep["dxn"][ri]), dxn_r) < TOL
    xnr = (xf[rows] * inv[rows, None]).astype(np.float64)
    dyg = dxn_r.astype(np.float64) * gamf[None, :]
    mean = np.sum(dyg * xnr, axis=1, keepdims=True) / d
    dx_r = bf16r(inv[rows, None] * (dyg - xnr * mean) + dyf[rows])
    assert orc.rel_frobenius(f32(dx[ri]), dx_r) < TOL
    # wgrads: sampled entries, each a contraction over all tokens (operands quantized along tokens)
    rng = np.random.default_rng(4)
    ii, jj = np.sort(rng.choice(d, 8, replace=False)), np.sort(rng.choice(f, 8, replace=False))
    a_t = qdq_rows(np.ascontiguousarray(dyf[:, ii].T), g_dy)
    b_t = qdq_rows(np.ascontiguousarray(orc.bf16_bits_to_f32(h_gpu[:, jj]).T), g_h)
    ref = a_t @ b_t.T
    mag = np.abs(a_t) @ np.abs(b_t).T
    got = f32(dwd[torch.from_numpy(ii).cuda()][:, torch.from_numpy(jj).cuda()]).astype(np.float64)
    assert gemm_bound_ok(got, ref, mag) and orc.rel_frobenius(got, ref) < TOL
    i2, j2 = np.sort(rng.choice(2 * f, 8, replace=False)), np.sort(rng.choice(d, 8, replace=False))
    a_t = qdq_rows(np.ascontiguousarray(orc.bf16_bits_to_f32(dgu_gpu[:, i2]).T), g_dgu)
    b_t = qdq_rows(np.ascontiguousarray(xn[:, j2].T), g_xn)
    ref = a_t @ b_t.T
    mag = np.abs(a_t) @ np.abs(b_t).T
    got = f32(dwgu[torch.from_numpy(i2).cuda()][:, torch.from_numpy(j2).cuda()]).astype(np.float64)
    assert gemm_bound_ok(got, ref, mag) and orc.rel_frobenius(got, ref) < TOL
    # dgamma: sum over tokens of dxn * xn (fp32 atomics across CTAs; float64 reference)
    xn_plain = (xf * inv[:, None]).astype(np.float32).astype(np.float64)
    dgam_ref = np.sum(f32(keep["dxn"]).astype(np.float64) * xn_plain, axis=0)
    assert orc.rel_frobenius(ggam.cpu().numpy(), dgam_ref) < 1e-3
