"""CPU checks of the rank-major bucket layout used for sharded weight
quantization (ShardQuantLayout) and of the assembly of every rank's quantized
rows into the full NVFP4 weights (GatheredWeights.qweights), against the
oracle quantizer of the whole matrices."""
import importlib

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as orc


@pytest.fixture(scope="module")
def mlp(pkg):
    return importlib.import_module("nvfp4_b200.mlp")


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("d,f,world", [(256, 256, 2), (512, 512, 4), (1024, 512, 8), (384, 192, 3)])
def test_layout_round_trip_and_segments(mlp, d, f, world):
    lay = mlp.ShardQuantLayout(d, f, world)
    n = d + 3 * d * f
    assert lay.shard * world == n and lay.shard % 16 == 0
    gen = torch.Generator().manual_seed(d + f + world)
    gamma = torch.randn(d, generator=gen)
    w_gu = torch.randn(2 * f, d, generator=gen)
    w_down = torch.randn(d, f, generator=gen)
    buf = torch.full((n,), float("nan"))
    lay.store(buf, gamma, w_gu, w_down)
    assert not torch.isnan(buf).any()                      # the pieces tile the bucket exactly
    g2, gu2, dn2 = lay.load(buf)
    assert torch.equal(g2, gamma) and torch.equal(gu2, w_gu) and torch.equal(dn2, w_down)
    for r in range(world):                                  # rank r's shard holds its rows, in order
        sh = buf[r * lay.shard:(r + 1) * lay.shard]
        (a, b, _), (c, e, _), (h, k, _) = lay.segments()
        assert torch.equal(sh[a:b], gamma[r * lay.gn:(r + 1) * lay.gn])
        assert torch.equal(sh[c:e].view(lay.r1, d), w_gu[r * lay.r1:(r + 1) * lay.r1])
        assert torch.equal(sh[h:k].view(lay.r2, f), w_down[r * lay.r2:(r + 1) * lay.r2])


def test_layout_fits():
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    assert mlp.ShardQuantLayout.fits(8192, 28672, 8) and mlp.ShardQuantLayout.fits(8192, 28672, 2)
    assert not mlp.ShardQuantLayout.fits(256, 512, 4)       # D/N = 64 rows: not whole 128-row groups
    assert not mlp.ShardQuantLayout.fits(256, 512, 1)
    with pytest.raises(ValueError):
        mlp.ShardQuantLayout(256, 512, 4)


@pytest.mark.parametrize("d,f,world", [(256, 256, 2), (384, 192, 3), (512, 256, 4)])
def test_gathered_pieces_assemble_the_full_weights(mlp, d, f, world):
    """Each rank's rows quantized by the oracle in both orientations, placed
    where the gathers put them, give exactly the oracle's quantization of the
    full W_gu and W_down (codes and swizzled scales, both orientations)."""
    lay = mlp.ShardQuantLayout(d, f, world)
    gen = torch.Generator().manual_seed(3 * d + f)
    w_gu = (0.05 * torch.randn(2 * f, d, generator=gen)).to(torch.bfloat16)
    w_down = (0.05 * torch.randn(d, f, generator=gen)).to(torch.bfloat16)
    g_gu = orc.global_scale_of(orc.bf16_bits_to_f32(bits(w_gu)))
    g_dn = orc.global_scale_of(orc.bf16_bits_to_f32(bits(w_down)))
    gw = mlp.GatheredWeights(lay, "cpu")
    for r in range(world):
        gu_r = bits(w_gu[r * lay.r1:(r + 1) * lay.r1])
        dn_r = bits(w_down[r * lay.r2:(r + 1) * lay.r2])
        for full_q, full_s, rows, x, g in ((gw.q_gu, gw.s_gu, lay.r1, gu_r, g_gu), (gw.q_down, gw.s_down, lay.r2, dn_r, g_dn)):
            q, s = orc.quant_nvfp4(x, g)
            full_q[r * rows:(r + 1) * rows] = torch.from_numpy(q)
            full_s[r * rows:(r + 1) * rows] = torch.from_numpy(s.reshape(rows, -1))
        for pq, ps, x, g in ((gw.pq_gu_t, gw.ps_gu_t, gu_r, g_gu), (gw.pq_down_t, gw.ps_down_t, dn_r, g_dn)):
            q, s = orc.quant_nvfp4(np.ascontiguousarray(x.T), g)
            pq[r] = torch.from_numpy(q)
            ps[r] = torch.from_numpy(s.reshape(ps.shape[1:]))
    gw.permuted = False
    qw = gw.qweights(torch.tensor([g_gu]), torch.tensor([g_dn]))
    gw.ensure_transposed()
    for q, s, x, g in ((qw.q_gu, qw.s_gu, bits(w_gu), g_gu), (qw.q_down, qw.s_down, bits(w_down), g_dn),
                       (qw.q_gu_t, qw.s_gu_t, np.ascontiguousarray(bits(w_gu).T), g_gu),
                       (qw.q_down_t, qw.s_down_t, np.ascontiguousarray(bits(w_down).T), g_dn)):
        oq, os_ = orc.quant_nvfp4(x, g)
        assert np.array_equal(q.numpy(), oq) and np.array_equal(s.numpy().reshape(-1), os_.reshape(-1))


def test_quantizer_out_buffers_checked(pkg):
    """ops.quantize / quantize_t accept caller buffers (slots of a gather
    buffer) only with the exact shape, dtype, device and contiguity."""
    import importlib
    ops = importlib.import_module("nvfp4_b200.ops")
    q_shape, s_shape = (256, 64), ops.scale_shape(256, 128)
    q = torch.empty(q_shape, dtype=torch.uint8)
    s = torch.empty(s_shape, dtype=torch.uint8)
    assert ops._outputs((q, s), q_shape, s_shape, q.device)[0] is q
    big = torch.empty((512, 64), dtype=torch.uint8)
    assert ops._outputs((big[128:384], s), q_shape, s_shape, q.device)[0].data_ptr() == big[128].data_ptr()
    for bad in ((q.float(), s), (q[:, :32], s), (q, s[:128]), (big[:, ::2][:256, :32], s)):
        with pytest.raises(RuntimeError):
            ops._outputs(bad, q_shape, s_shape, q.device)
    q2, s2 = ops._outputs(None, q_shape, s_shape, q.device)
    assert q2.shape == q_shape and s2.shape == s_shape and q2.dtype == torch.uint8
