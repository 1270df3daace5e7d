"""CPU tests of the oracle: self-consistency, and the pin against golden
vectors produced by the reference's own kernels (tests/golden/)."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.fail(f"golden fixture {name} missing (generate with tests/golden/make_golden.py on a GPU)")
    return np.load(path, allow_pickle=False)


# --------------------------------------------------------------------------
# E4M3 / E2M1 / swizzle primitives
# --------------------------------------------------------------------------

def test_e4m3_table_matches_torch():
    codes = np.arange(127, dtype=np.uint8)
    via_torch = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(orc.E4M3_TABLE.astype(np.float32), via_torch)


def test_e4m3_encode_rne_satfinite():
    t = orc.E4M3_TABLE
    mids = (t[:-1] + t[1:]) / 2
    vals = np.concatenate([t, mids, np.nextafter(mids.astype(np.float32), np.float32(0)).astype(np.float64),
                           np.nextafter(mids.astype(np.float32), np.float32(1e9)).astype(np.float64),
                           [448.0, 460.0, 464.0, 480.0, 1e6, np.inf, 1e-12, 2.0 ** -10, 3 * 2.0 ** -11]])
    vals = vals.astype(np.float32)
    got = orc.e4m3_encode_satfinite(vals)
    # torch's float8_e4m3fn conversion is RNE but maps >= 464 to NaN: clamp first (satfinite)
    ref = torch.from_numpy(np.minimum(vals, 448.0).astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(got, ref)
    # ties to even code at every midpoint
    tie_codes = orc.e4m3_encode_satfinite(mids.astype(np.float32))
    exact = orc.E4M3_TABLE.astype(np.float32)
    is_exact_mid = mids.astype(np.float32).astype(np.float64) == mids
    assert np.all(tie_codes[is_exact_mid] % 2 == 0)
    assert exact[orc.e4m3_encode_satfinite(np.array([np.inf], np.float32))[0]] == 448.0


def test_e2m1_ladder_ties_away_from_zero():
    thr = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    got = orc.e2m1_encode(thr, np.float32(1.0))
    assert list(got) == [1, 2, 3, 4, 5, 6, 7]
    assert list(orc.e2m1_encode(-thr, np.float32(1.0))) == [9, 10, 11, 12, 13, 14, 15]
    below = np.nextafter(thr, np.float32(0))
    assert list(orc.e2m1_encode(below, np.float32(1.0))) == [0, 1, 2, 3, 4, 5, 6]
    special = np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 7.0, -1e-30], np.float32)
    assert list(orc.e2m1_encode(special, np.float32(1.0))) == [0, 0, 7, 7, 15, 7, 8]


_E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _e2m1_rne_satfinite(x: np.ndarray) -> np.ndarray:
    """numpy model of cvt.rn.satfinite.e2m1x2.f32 on one value: nearest grid
    point, ties to the even code, saturation to +-6, sign kept, NaN -> +6
    (the behaviour the kernel's encoder relies on; a GPU sweep checks it)."""
    x = x.astype(np.float64)
    ax = np.abs(x)
    d = np.abs(ax[:, None] - _E2M1_GRID[None, :])
    best = d.min(axis=1, keepdims=True)
    cand = d == best
    two = cand.sum(axis=1) > 1
    code = np.where(two, np.argmax(cand & (np.arange(8) % 2 == 0)[None, :], axis=1), np.argmax(cand, axis=1))
    code = np.where(ax >= 6.0, 7, code)
    code = np.where(np.signbit(x), code | 8, code)
    return np.where(np.isnan(x), 7, code).astype(np.uint8)


def _kernel_e2m1_input(p: np.ndarray) -> np.ndarray:
    """numpy restatement of common.cuh e2m1_input after the fma: min(bits, 0xFF7FFFFF) | 1."""
    b = p.astype(np.float32).view(np.uint32)
    return (np.minimum(b, np.uint32(0xFF7FFFFF)) | np.uint32(1)).view(np.float32)


def test_hardware_e2m1_encoder_identity_equals_ladder():
    """Round-to-nearest-even E2M1 of (bits | 1), with -inf clamped, equals the
    reference's ties-away ladder for every f32 except -0.0, which the kernel's
    fma(f, inv_scale, +0) turns into +0 first."""
    hi16 = np.arange(0, 0x10000, dtype=np.uint32) << 16
    lows = np.array([0, 1, 2, 0x7FFF, 0x8000, 0xFFFF], dtype=np.uint32)
    bits = (hi16[:, None] | lows[None, :]).reshape(-1)
    thr = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], np.float32).view(np.uint32)
    near = (thr[:, None].astype(np.int64) + np.arange(-3, 4)[None, :]).reshape(-1).astype(np.uint32)
    rng = np.random.default_rng(0)
    bits = np.concatenate([bits, near, near | 0x80000000, rng.integers(0, 0xFFFFFFFF, 1 << 18, dtype=np.uint32)])
    bits = bits[bits != 0x80000000]
    p = bits.view(np.float32)
    # the fma's NaN results are the positive canonical NaN 0x7FFFFFFF
    p_fma = np.where(np.isnan(p), np.uint32(0x7FFFFFFF).view(np.float32), p)
    with np.errstate(invalid="ignore", over="ignore"):
        got = _e2m1_rne_satfinite(_kernel_e2m1_input(p_fma))
    ref = orc.e2m1_encode(p, np.float32(1.0))
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, [(hex(int(bits[i])), int(got[i]), int(ref[i])) for i in bad[:8]]
    # the fma with +0 maps -0.0 to +0 but keeps the sign of a negative underflow
    assert np.signbit(np.float32(-0.0) * np.float32(3.0))          # plain product keeps -0 ...
    assert not np.signbit(np.float32(-0.0) * np.float32(3.0) + np.float32(0.0))  # ... + 0 clears it



def test_swizzle_matches_reference_formula_and_is_bijective():
    for rows, k in [(1, 16), (129, 80), (256, 512), (300, 1024)]:
        pad_r, pad_c = orc.scale_shape(rows, k)
        rr, cc = np.meshgrid(np.arange(pad_r), np.arange(pad_c), indexing="ij")
        off = orc.swizzle_offset(rr, cc, pad_c).reshape(-1)
        assert np.array_equal(np.sort(off), np.arange(pad_r * pad_c))
        # float4utils.py:118-122, written out with Python ints
        for r, c in [(0, 0), (rows - 1, k // 16 - 1), (pad_r - 1, pad_c - 1), (37 % pad_r, 3 % pad_c)]:
            r_blk, c_blk, r_in, c_in = r >> 7, c >> 2, r & 127, c & 3
            tile_idx = r_blk * (pad_c >> 2) + c_blk
            new_row, new_col = r_in & 31, ((r_in >> 5) << 2) + c_in
            assert orc.swizzle_offset(r, c, pad_c) == (tile_idx << 9) + (new_row << 4) + new_col


def test_dequant_roundtrip_error_bound():
    import golden_cases as gc
    a, w = gc.config0_a_w()
    for x in (a, w):
        q, s = orc.quant_nvfp4(x)
        xf = orc.bf16_bits_to_f32(x)
        d = orc.dequant_nvfp4(q, s, *x.shape)
        # each block: |err| <= half the E2M1 step at the top (1.0 * scale) plus the
        # E4M3 scale rounding (< 2^-4 relative) on the block amax
        blk = np.abs(xf).reshape(x.shape[0], -1, 16).max(-1, keepdims=True)
        err = np.abs(d - xf).reshape(x.shape[0], -1, 16)
        normal = (orc.unswizzle_scales(s, *x.shape) >= 8)[..., None]   # E4M3 exponent field > 0
        assert np.all(np.where(normal, err <= blk * (1.0 / 6.0) * 1.07 + 1e-30, True))
        assert orc.rel_frobenius(d, xf) < 0.2


def test_global_scale_identity_at_one():
    import golden_cases as gc
    a, _ = gc.config0_a_w()
    q1, s1 = orc.quant_nvfp4(a)
    q2, s2 = orc.quant_nvfp4(a, global_scale=1.0)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)


def test_global_scale_rescues_small_gradients():
    # with g = 1 an N(0, 1e-3) tensor underflows every block scale; with
    # g = amax/(6*448) the blocks keep their information
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((128, 256)) * 1e-3).astype(np.float32)
    xb = orc.f32_to_bf16_bits(x)
    xf = orc.bf16_bits_to_f32(xb)
    g = orc.global_scale_of(xf)
    q, s = orc.quant_nvfp4(xb, global_scale=g)
    d = orc.dequant_nvfp4(q, s, 128, 256, global_scale=g)
    assert orc.rel_frobenius(d, xf) < 0.12


# --------------------------------------------------------------------------
# pin: oracle == reference kernels on the golden vectors
# --------------------------------------------------------------------------

def test_oracle_matches_reference_quantizer_golden():
    import golden_cases as gc
    gold = _load("golden_quant.npz")
    cases = gc.quant_cases()
    assert len(cases) >= 10
    for name, x in cases.items():
        assert str(gold[f"{name}__sha"]) == gc.sha(x), f"input drift for {name}"
        q, s = orc.quant_nvfp4(x)
        assert np.array_equal(q, gold[f"{name}__q"]), f"nibbles differ from the reference kernel: {name}"
        assert np.array_equal(s, gold[f"{name}__s"]), f"scales differ from the reference kernel: {name}"


def test_oracle_matches_reference_rmsnorm_golden():
    import golden_cases as gc
    gold = _load("golden_rmsnorm.npz")
    eps = float(gold["eps"])
    for name, x in gc.rms_cases().items():
        assert str(gold[f"{name}__sha"]) == gc.sha(x), f"input drift for {name}"
        inv_ref = gold[f"{name}__inv_rms"]
        inv64 = orc.rms_inv(x, eps)
        # rsqrtf + fp32 tree sum: a few ulp of float64
        assert np.all(np.abs(inv_ref.astype(np.float64) - inv64) <= 2e-6 * inv64 + 1e-30), name
        # given the kernel's own inv_rms, nibbles and scales are bit-exact
        q, s = orc.rmsnorm_quant_nvfp4(x, inv_ref)
        assert np.array_equal(q, gold[f"{name}__q"]), name
        assert np.array_equal(s, gold[f"{name}__s"]), name


def test_gemm_emulation_matches_reference_gemm_golden():
    gold = _load("golden_gemm.npz")
    for name in ("cfg0", "k4096"):
        m, n, k = (int(v) for v in gold[f"{name}__mnk"])
        ref = orc.bf16_bits_to_f32(gold[f"{name}__d"]).reshape(m, n)
        emu = orc.gemm_emulation_f64(gold[f"{name}__qa"], gold[f"{name}__sa"], gold[f"{name}__qb"],
                                     gold[f"{name}__sb"], m, n, k)
        err = orc.rel_frobenius(ref, emu)
        assert err < 1e-2, (name, err)
        # bf16 output rounding bounds the element error (plus accumulation slack)
        assert np.all(np.abs(ref - emu) <= np.abs(emu) * 2.0 ** -8 + 1e-3 * math.sqrt(k)), name


def test_mxfp4_dequant_known_answer():
    """UE8M0 scales are powers of two (2^(e-127), 0xFF NaN) applied per 1x32
    block through the 128x4-atom swizzle; nibbles decode as E2M1."""
    assert orc.ue8m0_decode(np.array([127, 128, 120, 0]))[:3].tolist() == [1.0, 2.0, 2.0 ** -7]
    assert np.isnan(orc.ue8m0_decode(np.array([255])))[0]
    rows, k = 3, 64
    q = np.zeros((rows, k // 2), dtype=np.uint8)
    q[1, 0] = 0x2F       # row 1: element 0 = -6 (0xF), element 1 = +1 (0x2)
    q[2, 16] = 0x07      # row 2: element 32 = +6 (second block)
    pad_r, pad_c = orc.mx_scale_shape(rows, k)
    s = np.zeros(pad_r * pad_c, dtype=np.uint8)
    s[orc.swizzle_offset(np.array(1), np.array(0), pad_c)] = 129   # x4
    s[orc.swizzle_offset(np.array(2), np.array(1), pad_c)] = 126   # x1/2
    d = orc.dequant_mxfp4(q, s, rows, k)
    assert d[1, 0] == -24.0 and d[1, 1] == 4.0 and d[2, 32] == 3.0
    assert np.count_nonzero(d) == 3


def test_mxfp4_gemm_emulation_matches_scalar_loops():
    """The MXFP4 emulation (dequantize, float64 matmul) against plain scalar
    loops that decode every nibble and scale on their own: E2M1 magnitudes
    {0, .5, 1, 1.5, 2, 3, 4, 6} with the sign in bit 3, element 2j in the low
    nibble, scale of (row r, block c) at the 128x4-atom position, 2^(e-127)."""
    rng = np.random.default_rng(3)
    m, n, k = 5, 3, 96                     # three 32-element blocks: a partial 4-block group
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]

    def operand(rows):
        q = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
        pad_r, pad_c = orc.round_up(rows, 128), orc.round_up(k // 32, 4)
        s = np.zeros(pad_r * pad_c, dtype=np.uint8)
        codes = rng.integers(120, 135, size=(rows, k // 32))
        for r in range(rows):
            for c in range(k // 32):
                pos = ((r // 128) * (pad_c // 4) + c // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4
                s[pos] = codes[r, c]
        return q, s, codes

    def value(q, codes, r, j):
        byte = int(q[r, j // 2])
        nib = byte & 0xF if j % 2 == 0 else byte >> 4
        v = mags[nib & 7] * (-1.0 if nib & 8 else 1.0)
        return v * 2.0 ** (int(codes[r, j // 32]) - 127)

    qa, sa, ca = operand(m)
    qb, sb, cb = operand(n)
    ref = np.array([[sum(value(qa, ca, i, j) * value(qb, cb, t, j) for j in range(k)) for t in range(n)]
                    for i in range(m)])
    got = orc.mxfp4_gemm_emulation_f64(qa, sa, qb, sb, m, n, k)
    assert np.array_equal(got, ref) or np.allclose(got, ref, rtol=1e-12, atol=0)
