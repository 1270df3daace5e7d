"""GPU parity of the quantizers against the oracle (bit-exact) and against
the reference kernels' golden vectors."""
import os

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def dev(b):
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).cuda()


def u8(t):
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def test_quant_matches_reference_golden(pkg):
    import golden_cases as gc
    gold = np.load(os.path.join(GOLDEN, "golden_quant.npz"))
    for name, x in gc.quant_cases().items():
        q, s = pkg.ops.quantize(dev(x))
        assert np.array_equal(u8(q), gold[f"{name}__q"]), name
        assert np.array_equal(u8(s), gold[f"{name}__s"]), name


@pytest.mark.parametrize("rows,k", [(1, 16), (3, 32), (127, 48), (128, 256), (129, 80), (255, 272),
                                    (300, 512), (64, 1040), (8, 4096)])
def test_quant_random_shapes(pkg, rows, k):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + k)
    x = (torch.randn(rows, k, device="cuda", generator=g) * 5).to(torch.bfloat16)
    q, s = pkg.ops.quantize(x)
    oq, os_ = orc.quant_nvfp4(bits(x))
    assert np.array_equal(u8(q), oq) and np.array_equal(u8(s), os_)


@pytest.mark.parametrize("gs", [0.5, 1e-3 / 2688, 7.25])
def test_quant_global_scale(pkg, gs):
    x = (torch.randn(200, 320, device="cuda") * 1e-3).to(torch.bfloat16)
    gt = torch.tensor([gs], device="cuda", dtype=torch.float32)
    q, s = pkg.ops.quantize(x, global_scale=gt)
    oq, os_ = orc.quant_nvfp4(bits(x), global_scale=np.float32(gs))
    assert np.array_equal(u8(q), oq) and np.array_equal(u8(s), os_)


def test_global_scale_kernel(pkg):
    x = torch.randn(1000, 77, device="cuda").to(torch.bfloat16)   # 77000 elements: vector + tail
    x[3, 5] = float("nan")
    x[10, 7] = -123.5
    g, amax = pkg.ops.global_scale(x, with_amax=True)
    ref = orc.global_scale_of(orc.bf16_bits_to_f32(bits(x)))
    assert amax.item() == 123.5
    assert g.item() == float(ref)
    # workspace reset: a second call gives the same answer
    g2 = pkg.ops.global_scale(x * 0.5)
    assert g2.item() == float(np.float32(61.75) / np.float32(2688.0))
    z = torch.zeros(64, device="cuda", dtype=torch.bfloat16)
    assert pkg.ops.global_scale(z).item() == 1.0


@pytest.mark.parametrize("rows,k,use_gamma", [(256, 512, False), (129, 4096, True), (5, 16, False),
                                              (64, 8192, True), (3, 12288, False), (300, 1040, True)])
def test_rmsnorm_quant(pkg, rows, k, use_gamma):
    g = torch.Generator(device="cuda").manual_seed(rows + k)
    x = (torch.randn(rows, k, device="cuda", generator=g) * 3).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).to(torch.bfloat16) if use_gamma else None
    q, s, inv = pkg.ops.rmsnorm_quantize(x, 1e-6, gamma=gamma)
    inv_np = inv.cpu().numpy()
    inv64 = orc.rms_inv(bits(x), 1e-6)
    assert np.all(np.abs(inv_np - inv64) <= 2e-6 * inv64)
    oq, os_ = orc.rmsnorm_quant_nvfp4(bits(x), inv_np, None if gamma is None else bits(gamma))
    assert np.array_equal(u8(q), oq) and np.array_equal(u8(s), os_)


def test_rmsnorm_matches_reference_golden(pkg):
    import golden_cases as gc
    gold = np.load(os.path.join(GOLDEN, "golden_rmsnorm.npz"))
    for name, x in gc.rms_cases().items():
        q, s, inv = pkg.ops.rmsnorm_quantize(dev(x), float(gold["eps"]))
        ref_inv = gold[f"{name}__inv_rms"]
        # the kernel reproduces the reference's fp32 reduction order: 1/RMS is bit-identical
        assert np.array_equal(inv.cpu().numpy().view(np.uint32), ref_inv.view(np.uint32)), name
        assert np.array_equal(u8(q), gold[f"{name}__q"]) and np.array_equal(u8(s), gold[f"{name}__s"]), name


@pytest.mark.parametrize("rows,k,with_gamma", [(96, 1024, True), (1203, 4096, True), (700, 4000, False),
                                                (301, 8192, True), (64, 12288, False), (37, 16384, True)])
def test_rmsnorm_stats_and_global_scale_path(pkg, rows, k, with_gamma):
    """rmsnorm_stats for one, two and four 16-element slices per thread (k up
    to 16384, ragged k and row counts that leave CTAs with different row
    counts): 1/RMS within 2e-6 of float64, the global scale exactly that of
    (x * inv_rms) * gamma, and the quantizer bit-exact given both."""
    gen = torch.Generator(device="cuda").manual_seed(rows + k)
    x = (torch.randn(rows, k, device="cuda", generator=gen) * 4).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(k, device="cuda", generator=gen)).to(torch.bfloat16) if with_gamma else None
    inv, g = pkg.ops.rmsnorm_stats(x, 1e-6, gamma=gamma)
    inv_np = inv.cpu().numpy()
    inv64 = orc.rms_inv(bits(x), 1e-6)
    assert np.all(np.abs(inv_np - inv64) <= 2e-6 * inv64)
    y = (orc.bf16_bits_to_f32(bits(x)) * inv_np[:, None]).astype(np.float32)
    if with_gamma:
        y = y * orc.bf16_bits_to_f32(bits(gamma))[None, :]
    assert g.item() == float(orc.global_scale_of(y.astype(np.float32)))
    q, s = pkg.ops.quantize(x, global_scale=g, row_scale=inv, gamma=gamma)
    oq, os_ = orc.rmsnorm_quant_nvfp4(bits(x), inv_np, None if gamma is None else bits(gamma), global_scale=g.item())
    assert np.array_equal(u8(q), oq) and np.array_equal(u8(s), os_)


@pytest.mark.parametrize("rows,cols,opts", [(256, 128, ""), (16, 8, ""), (272, 200, "row"), (512, 136, "gamma"),
                                            (48, 384, "row,gamma"), (1040, 64, "g")])
def test_quant_transposed(pkg, rows, cols, opts):
    gen = torch.Generator(device="cuda").manual_seed(rows * 3 + cols)
    x = (torch.randn(rows, cols, device="cuda", generator=gen) * 2).to(torch.bfloat16)
    rs = torch.rand(rows, device="cuda", generator=gen) + 0.5 if "row" in opts else None
    gamma = (1 + 0.1 * torch.randn(cols, device="cuda", generator=gen)).to(torch.bfloat16) if "gamma" in opts else None
    gs = torch.tensor([0.01], device="cuda") if "g" in opts else None
    q, s = pkg.ops.quantize_t(x, global_scale=gs, row_scale=rs, gamma=gamma)
    xf = orc.bf16_bits_to_f32(bits(x))
    if rs is not None:
        xf = (xf * rs.cpu().numpy()[:, None]).astype(np.float32)
    if gamma is not None:
        xf = (xf * orc.bf16_bits_to_f32(bits(gamma))[None, :]).astype(np.float32)
    oq, os_ = orc.quant_nvfp4_f32(np.ascontiguousarray(xf.T), None if gs is None else 0.01)
    assert np.array_equal(u8(q), oq) and np.array_equal(u8(s), os_)


def test_full_size_rows_sampled(pkg):
    """RMSNorm->quantize workload size (32768 x 4096): rows are independent, so
    every quantized row must equal the oracle on that row; check a sample."""
    r, k = 32768, 4096
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(r, k, device="cuda", generator=g)
    rs = torch.exp(torch.empty(r, 1, device="cuda").uniform_(np.log(0.1), np.log(10.0), generator=g))
    x = (x * rs).to(torch.bfloat16)
    q, s = pkg.ops.quantize(x)
    qt, st = pkg.ops.quantize_t(x)
    idx = torch.randperm(r, generator=torch.Generator().manual_seed(0))[:48].sort().values
    xs = bits(x[idx.cuda()])
    oq, _ = orc.quant_nvfp4(xs)
    assert np.array_equal(u8(q)[idx.numpy()], oq)
    scodes = orc.unswizzle_scales(u8(s), r, k)[idx.numpy()]
    _, oc = orc.quant_blocks(orc.bf16_bits_to_f32(xs).reshape(48, -1, 16))
    assert np.array_equal(scodes, oc)
    cidx = np.array([0, 1, 77, 2048, 4095])
    colsx = np.ascontiguousarray(bits(x[:, torch.from_numpy(cidx).cuda()]).T)
    oqt, _ = orc.quant_nvfp4(colsx)
    assert np.array_equal(u8(qt)[cidx], oqt)
