"""NVFP4 SwiGLU MLP: forward, dgrad and wgrad with NVFP4 operands.

The reference ships only an NVFP4-forward / bf16-backward linear layer
(float4utils.py:621-714) and mentions an unshipped "NVFP4 MLP" (README.md:1).
This module builds that MLP block on the library's kernels:

    y  = x + W_down . h,    h = silu(g) * u,    [g | u] = W_gu . n(x),
    n(x) = (x * inv_rms(x)) * gamma

with W_gu = [W_gate; W_up] ([2F, D]) and W_down ([D, F]).  Every GEMM takes
NVFP4 operands blocked 1x16 along its contraction dimension with a
per-tensor global scale g = amax/(6*448) folded into the GEMM's output scale:

    forward   gu  = Q(n(x))     . Q(W_gu)^T          K = D
              y   = Q(h)        . Q(W_down)^T + x    K = F  (residual fused)
    dgrad     dh  = Q(dy)       . Q_t(W_down)^T      K = D
              dxn = Q(dgu)      . Q_t(W_gu)^T        K = 2F
    wgrad     dWd = Q_t(dy)     . Q_t(h)^T           K = tokens
              dWgu= Q_t(dgu)    . Q_t(n(x))^T        K = tokens

Q quantizes along rows' last dimension, Q_t along the first (transposed
quantizer).  Quantization is treated as identity in the backward
(straight-through).  Weights are quantized once per optimizer step and
reused across micro-batches.

W_gu's 2F rows may be stored [W_gate; W_up] (``interleave=0``) or with gate
and up rows alternating in blocks of 128 (``interleave=128``).  The latter
lets the gate/up GEMM apply SwiGLU in its epilogue (each 256-column output
tile holds 128 gate columns and their up columns), so h and its global
scale come out of that GEMM, and the dh GEMM to apply the SwiGLU backward
in its epilogue (each 256-column dh tile meets two whole gate/up blocks;
F % 256 == 0), so dgu and its global scale come out of that GEMM and dh is
never stored.  Every other GEMM only sees a relabelled 2F dimension.
NVFP4MLPStackTrainer keeps W_gu interleaved.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn

from . import ops
from .dp import BucketAllReducer, ShardedBucketOptimizer


@dataclass
class QWeights:
    """Per-step NVFP4 copies of one block's weights (forward and dgrad layouts)."""
    g_gu: torch.Tensor
    g_down: torch.Tensor
    q_gu: torch.Tensor
    s_gu: torch.Tensor
    q_down: torch.Tensor
    s_down: torch.Tensor
    q_gu_t: torch.Tensor
    s_gu_t: torch.Tensor
    q_down_t: torch.Tensor
    s_down_t: torch.Tensor


def quantize_weights(w_gu: torch.Tensor, w_down: torch.Tensor, need_t: bool = True,
                     g_gu: Optional[torch.Tensor] = None, g_down: Optional[torch.Tensor] = None) -> QWeights:
    """Both NVFP4 orientations of a block's weights.  The global scales are
    computed here unless given (the trainer takes them from the previous
    AdamW update, which already saw every weight it wrote)."""
    g_gu = ops.global_scale(w_gu) if g_gu is None else g_gu
    g_down = ops.global_scale(w_down) if g_down is None else g_down
    q_gu, s_gu = ops.quantize(w_gu, global_scale=g_gu)
    q_down, s_down = ops.quantize(w_down, global_scale=g_down)
    if need_t:
        q_gu_t, s_gu_t = ops.quantize_t(w_gu, global_scale=g_gu)        # [D, 2F] along 2F
        q_down_t, s_down_t = ops.quantize_t(w_down, global_scale=g_down)  # [F, D] along D
    else:
        q_gu_t = s_gu_t = q_down_t = s_down_t = None
    return QWeights(g_gu, g_down, q_gu, s_gu, q_down, s_down, q_gu_t, s_gu_t, q_down_t, s_down_t)


@dataclass
class Saved:
    x: torch.Tensor
    inv_rms: torch.Tensor
    g_xn: torch.Tensor
    gu: torch.Tensor
    h: torch.Tensor
    g_h: torch.Tensor


def block_forward(x: torch.Tensor, gamma: torch.Tensor, qw: QWeights, eps: float = 1e-6, save: bool = True,
                  interleave: int = 0):
    """One RMSNorm+SwiGLU block on bf16 x [T, D] -> (y [T, D], saved activations).

    ``interleave=128``: W_gu rows alternate gate/up in blocks of 128 and the
    gate/up GEMM computes h in its epilogue."""
    inv_rms, g_xn = ops.rmsnorm_stats(x, eps, gamma=gamma)
    q_xn, s_xn = ops.quantize(x, global_scale=g_xn, row_scale=inv_rms, gamma=gamma)
    if interleave:
        h, gu, g_h = ops.gemm_swiglu(q_xn, s_xn, qw.q_gu, qw.s_gu, scale_a=g_xn, scale_b=qw.g_gu, store_gu=save)
        del q_xn, s_xn
    else:
        gu = ops.gemm(q_xn, s_xn, qw.q_gu, qw.s_gu, scale_a=g_xn, scale_b=qw.g_gu)
        del q_xn, s_xn
        h, g_h = ops.swiglu_fwd(gu, with_scale=True)
    q_h, s_h = ops.quantize(h, global_scale=g_h)
    y = ops.gemm(q_h, s_h, qw.q_down, qw.s_down, scale_a=g_h, scale_b=qw.g_down, residual=x)
    saved = Saved(x, inv_rms, g_xn, gu, h, g_h) if save else None
    return y, saved


def _wgrad(qa, sa, qb, sb, ga, gb, out: torch.Tensor, accumulate: bool) -> None:
    """Weight-gradient GEMM into ``out``: a [rows, cols] tensor, or a
    [pieces, rows / pieces, cols] tensor of row blocks (a rank-major bucket),
    one GEMM per block; a block is whole 128-row groups of A, so its rows of
    qa and sa are contiguous slices."""
    if out.dim() == 2:
        ops.gemm(qa, sa, qb, sb, scale_a=ga, scale_b=gb, out=out, accumulate=accumulate)
        return
    rows = out.shape[1]
    for i in range(out.shape[0]):
        lo, hi = i * rows, (i + 1) * rows
        ops.gemm(qa[lo:hi], sa[lo:hi], qb, sb, scale_a=ga, scale_b=gb, out=out[i], accumulate=accumulate)


def block_backward(dy: torch.Tensor, gamma: torch.Tensor, qw: QWeights, sv: Saved,
                   grad_gamma: torch.Tensor, grad_gu: torch.Tensor, grad_down: torch.Tensor,
                   accumulate: bool, interleave: int = 0, keep: Optional[dict] = None) -> torch.Tensor:
    """Backward of block_forward given dy [T, D].

    grad_gamma (fp32 [D]) is accumulated; grad_gu ([2F, D]) and grad_down
    ([D, F]) are written (bf16) or accumulated (fp32, accumulate=True).
    grad_gu / grad_down may also be [pieces, rows / pieces, cols] row-block
    views (see _wgrad).  Returns dx [T, D] (including the residual path).  ``keep`` (a dict)
    receives the intermediates dgu, dxn and the global scales g_dy, g_dgu,
    for inspection; normally they are freed as soon as they are consumed."""
    g_dy = ops.global_scale(dy)
    q_dy, s_dy = ops.quantize(dy, global_scale=g_dy)
    # interleaved gate/up with whole 256-column dh tiles: the SwiGLU backward
    # runs in the dh GEMM's epilogue and dh is never stored
    fused = interleave == 128 and (sv.gu.shape[1] // 2) % 256 == 0
    if fused:
        dgu, g_dgu = ops.gemm_dswiglu(q_dy, s_dy, qw.q_down_t, qw.s_down_t, sv.gu, scale_a=g_dy, scale_b=qw.g_down)
    else:
        dh = ops.gemm(q_dy, s_dy, qw.q_down_t, qw.s_down_t, scale_a=g_dy, scale_b=qw.g_down)
    del q_dy, s_dy
    # wgrad of W_down: dy^T . h  (contraction over tokens)
    q_dyt, s_dyt = ops.quantize_t(dy, global_scale=g_dy)
    q_ht, s_ht = ops.quantize_t(sv.h, global_scale=sv.g_h)
    _wgrad(q_dyt, s_dyt, q_ht, s_ht, g_dy, sv.g_h, grad_down, accumulate)
    del q_dyt, s_dyt, q_ht, s_ht
    if not fused:
        dgu, g_dgu = ops.swiglu_bwd(sv.gu, dh, with_scale=True, interleave=interleave)
        del dh
    q_dgu, s_dgu = ops.quantize(dgu, global_scale=g_dgu)
    dxn = ops.gemm(q_dgu, s_dgu, qw.q_gu_t, qw.s_gu_t, scale_a=g_dgu, scale_b=qw.g_gu)
    del q_dgu, s_dgu
    if keep is not None:
        keep.update(dgu=dgu, dxn=dxn, g_dy=g_dy, g_dgu=g_dgu)
    # wgrad of W_gu: dgu^T . n(x)
    q_dgut, s_dgut = ops.quantize_t(dgu, global_scale=g_dgu)
    del dgu
    q_xnt, s_xnt = ops.quantize_t(sv.x, global_scale=sv.g_xn, row_scale=sv.inv_rms, gamma=gamma)
    _wgrad(q_dgut, s_dgut, q_xnt, s_xnt, g_dgu, sv.g_xn, grad_gu, accumulate)
    del q_dgut, s_dgut, q_xnt, s_xnt
    dx = ops.rmsnorm_bwd(sv.x, gamma, sv.inv_rms, dxn, dres=dy, dgamma_acc=grad_gamma)
    return dx


# ----------------------------------------------------------------------------
# autograd front end
# ----------------------------------------------------------------------------

class NVFP4SwiGLUFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, w_gu, w_down, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        qw = quantize_weights(w_gu, w_down, need_t=True)
        y, sv = block_forward(x2, gamma, qw, eps)
        ctx.qw, ctx.sv = qw, sv
        ctx.save_for_backward(gamma)
        ctx.shape = shape
        return y.reshape(shape)

    @staticmethod
    def backward(ctx, dy):
        (gamma,) = ctx.saved_tensors
        dy2 = dy.reshape(-1, ctx.shape[-1]).contiguous().to(torch.bfloat16)
        d = gamma.numel()
        grad_gamma = torch.zeros(d, device=dy.device, dtype=torch.float32)
        grad_gu = torch.empty((ctx.sv.gu.shape[1], d), device=dy.device, dtype=torch.bfloat16)
        grad_down = torch.empty((d, ctx.sv.h.shape[1]), device=dy.device, dtype=torch.bfloat16)
        dx = block_backward(dy2, gamma, ctx.qw, ctx.sv, grad_gamma, grad_gu, grad_down, accumulate=False)
        ctx.qw = ctx.sv = None
        return dx.reshape(ctx.shape), grad_gamma.to(gamma.dtype), grad_gu, grad_down, None


class NVFP4SwiGLUMLP(nn.Module):
    """Pre-norm residual SwiGLU MLP block with NVFP4 GEMMs in forward and backward."""

    def __init__(self, d_model: int, d_ff: int, eps: float = 1e-6, device=None, dtype=torch.bfloat16,
                 init_std: float = 0.02):
        super().__init__()
        self.d_model, self.d_ff, self.eps = d_model, d_ff, eps
        self.gamma = nn.Parameter(torch.ones(d_model, device=device, dtype=dtype))
        self.w_gu = nn.Parameter(torch.empty(2 * d_ff, d_model, device=device, dtype=dtype))
        self.w_down = nn.Parameter(torch.empty(d_model, d_ff, device=device, dtype=dtype))
        with torch.no_grad():
            self.w_gu.normal_(0.0, init_std)
            self.w_down.normal_(0.0, init_std)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return NVFP4SwiGLUFunction.apply(x, self.gamma, self.w_gu, self.w_down, self.eps)


# ----------------------------------------------------------------------------
# explicit training step for a stack of blocks (no autograd), with DP
# ----------------------------------------------------------------------------

@dataclass
class AdamConfig:
    """AdamW hyper-parameters.  ``master_weights`` (default) keeps an fp32
    master copy of every bf16 parameter (of this rank's shard under ZeRO-1):
    AdamW updates the master and the bf16 parameter is its round-to-nearest
    copy, so steps smaller than half a bf16 ulp of a weight (lr = 1e-4 against
    |w| > ~0.05) still move it over time.  Without it the update is applied
    to the bf16 parameter directly and such steps are lost."""
    lr: float = 1e-4
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    weight_decay: float = 0.0
    master_weights: bool = True


class ShardQuantLayout:
    """Rank-major layout of one block's flat bucket for sharded weight
    quantization under ZeRO-1 (N = world > 1 ranks).

    Rank r's shard of S = n / N elements is [gamma_r | W_gu rows r | W_down
    rows r]: gamma elements [r D/N, (r+1) D/N), W_gu rows [r R1, (r+1) R1)
    with R1 = 2F/N and W_down rows [r R2, (r+1) R2) with R2 = D/N.  Both row
    ranges are whole 128-row groups, so the rank can quantize its own rows in
    both NVFP4 orientations after its AdamW update: the row-wise codes and
    swizzled scales of its rows are contiguous slices of the full tensors
    (gathered in place), the transposed ones are column slices of the full
    transposed tensors (gathered rank-major, then permuted into place).  The
    ranks then exchange 1.125 bytes per parameter of NVFP4 weights instead of
    2 bytes of bf16 parameters, and each quantizes 1/N of the weights."""

    def __init__(self, d: int, f: int, world: int):
        if not ShardQuantLayout.fits(d, f, world):
            raise ValueError(f"d={d}, f={f} do not split into 128-row groups over {world} ranks")
        self.d, self.f, self.world = d, f, world
        self.gn = d // world
        self.r1 = 2 * f // world
        self.r2 = d // world
        self.off_gu = self.gn
        self.off_down = self.gn + self.r1 * d
        self.shard = self.off_down + self.r2 * f

    @staticmethod
    def fits(d: int, f: int, world: int) -> bool:
        return (world > 1 and d % world == 0 and (2 * f) % world == 0 and (d // world) % 128 == 0
                and (2 * f // world) % 128 == 0)

    def _pieces(self, buf: torch.Tensor, off: int, shape, strides) -> torch.Tensor:
        return torch.as_strided(buf, shape, strides, buf.storage_offset() + off)

    def gamma_pieces(self, buf: torch.Tensor) -> torch.Tensor:      # [N, D/N]
        return self._pieces(buf, 0, (self.world, self.gn), (self.shard, 1))

    def gu_pieces(self, buf: torch.Tensor) -> torch.Tensor:         # [N, R1, D]
        return self._pieces(buf, self.off_gu, (self.world, self.r1, self.d), (self.shard, self.d, 1))

    def down_pieces(self, buf: torch.Tensor) -> torch.Tensor:       # [N, R2, F]
        return self._pieces(buf, self.off_down, (self.world, self.r2, self.f), (self.shard, self.f, 1))

    def store(self, buf: torch.Tensor, gamma: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> None:
        """Write standard-layout gamma [D], W_gu [2F, D], W_down [D, F] into a rank-major bucket."""
        self.gamma_pieces(buf).copy_(gamma.reshape(self.world, self.gn))
        self.gu_pieces(buf).copy_(w_gu.reshape(self.world, self.r1, self.d))
        self.down_pieces(buf).copy_(w_down.reshape(self.world, self.r2, self.f))

    def load(self, buf: torch.Tensor):
        """Standard-layout copies (gamma, W_gu, W_down) of a rank-major bucket."""
        return (self.gamma_pieces(buf).reshape(self.d), self.gu_pieces(buf).reshape(2 * self.f, self.d),
                self.down_pieces(buf).reshape(self.d, self.f))

    def segments(self):
        """(lo, hi, which) of the shard: gamma, W_gu rows, W_down rows (which = None, 0, 1)."""
        return ((0, self.gn, None), (self.gn, self.off_down, 0), (self.off_down, self.shard, 1))


class GatheredWeights:
    """One block's NVFP4 weights assembled from every rank's quantized rows
    (ShardQuantLayout): persistent full tensors in QWeights' layouts, plus
    rank-major landing buffers for the transposed orientation."""

    def __init__(self, lay: ShardQuantLayout, device):
        n, d, f, r1, r2 = lay.world, lay.d, lay.f, lay.r1, lay.r2
        u8 = dict(device=device, dtype=torch.uint8)
        self.lay = lay
        self.gamma = torch.empty(d, device=device, dtype=torch.bfloat16)
        self.q_gu = torch.empty((2 * f, d // 2), **u8)
        self.s_gu = torch.empty(ops.scale_shape(2 * f, d), **u8)
        self.q_down = torch.empty((d, f // 2), **u8)
        self.s_down = torch.empty(ops.scale_shape(d, f), **u8)
        self.q_gu_t = torch.empty((d, f), **u8)                         # [D, 2F/2]
        self.s_gu_t = torch.empty(ops.scale_shape(d, 2 * f), **u8)
        self.q_down_t = torch.empty((f, d // 2), **u8)
        self.s_down_t = torch.empty(ops.scale_shape(f, d), **u8)
        self.pq_gu_t = torch.empty((n, d, r1 // 2), **u8)
        self.ps_gu_t = torch.empty((n,) + ops.scale_shape(d, r1), **u8)
        self.pq_down_t = torch.empty((n, f, r2 // 2), **u8)
        self.ps_down_t = torch.empty((n,) + ops.scale_shape(f, r2), **u8)
        self.works: List[object] = []      # gathers of gamma and the row-wise weights (forward)
        self.works_t: List[object] = []    # gathers of the transposed pieces (backward)
        self.permuted = True

    def quantize(self, rank: int, param: torch.Tensor, g_gu: torch.Tensor, g_down: torch.Tensor) -> None:
        """Quantize this rank's rows of the block (rank-major param bucket) in
        both orientations with the weights' global scales, into the slots the
        gathers send from."""
        lay, r = self.lay, rank
        gu_r, down_r = lay.gu_pieces(param)[r], lay.down_pieces(param)[r]
        a1, b1 = r * lay.r1, (r + 1) * lay.r1
        a2, b2 = r * lay.r2, (r + 1) * lay.r2
        ops.quantize(gu_r, global_scale=g_gu, out=(self.q_gu[a1:b1], self.s_gu[a1:b1]))
        ops.quantize(down_r, global_scale=g_down, out=(self.q_down[a2:b2], self.s_down[a2:b2]))
        ops.quantize_t(gu_r, global_scale=g_gu, out=(self.pq_gu_t[r], self.ps_gu_t[r]))
        ops.quantize_t(down_r, global_scale=g_down, out=(self.pq_down_t[r], self.ps_down_t[r]))
        self.permuted = False

    def gather_forward(self, rank: int, param: torch.Tensor, pg) -> None:
        """Start the all-gathers of gamma and the row-wise NVFP4 weights (what the forward uses)."""
        import torch.distributed as dist
        lay, r = self.lay, rank
        a1, b1 = r * lay.r1, (r + 1) * lay.r1
        a2, b2 = r * lay.r2, (r + 1) * lay.r2
        works = [dist.all_gather_into_tensor(self.gamma, lay.gamma_pieces(param)[r], group=pg, async_op=True)]
        for full, lo, hi in ((self.q_gu, a1, b1), (self.s_gu, a1, b1), (self.q_down, a2, b2), (self.s_down, a2, b2)):
            works.append(dist.all_gather_into_tensor(full.view(-1), full[lo:hi].view(-1), group=pg, async_op=True))
        self.works = works

    def gather_transposed(self, rank: int, pg) -> None:
        """Start the all-gathers of the transposed pieces (in place, rank-major; first used by the backward)."""
        import torch.distributed as dist
        self.works_t = [dist.all_gather_into_tensor(buf.view(-1), buf[rank].view(-1), group=pg, async_op=True)
                        for buf in (self.pq_gu_t, self.ps_gu_t, self.pq_down_t, self.ps_down_t)]

    def wait(self) -> None:
        """Make the current stream wait for every gather of the block still in flight."""
        for w in self.works + self.works_t:
            w.wait()
        self.works, self.works_t = [], []

    def qweights(self, g_gu: torch.Tensor, g_down: torch.Tensor) -> QWeights:
        """Wait (on the current stream) for the forward's gathers and return the
        block's QWeights; the transposed fields are valid after ensure_transposed()."""
        for w in self.works:
            w.wait()
        self.works = []
        return QWeights(g_gu, g_down, self.q_gu, self.s_gu, self.q_down, self.s_down, self.q_gu_t, self.s_gu_t,
                        self.q_down_t, self.s_down_t)

    def ensure_transposed(self) -> None:
        """Wait for the transposed pieces and put them in place (once per gather)."""
        for w in self.works_t:
            w.wait()
        self.works_t = []
        if not self.permuted:
            lay, n = self.lay, self.lay.world
            d, f, r1, r2 = lay.d, lay.f, lay.r1, lay.r2
            i64 = torch.int64   # moved as 8-byte words: rows of r/2 bytes, atoms of 512 bytes
            self.q_gu_t.view(i64).view(d, n, r1 // 16).copy_(self.pq_gu_t.view(i64).permute(1, 0, 2))
            self.q_down_t.view(i64).view(f, n, r2 // 16).copy_(self.pq_down_t.view(i64).permute(1, 0, 2))
            # swizzled scales are [128-row group][4-block atom][512 bytes]: the
            # ranks' atoms of one row group are consecutive column ranges
            for full, pieces, rows, kr in ((self.s_gu_t, self.ps_gu_t, d, r1), (self.s_down_t, self.ps_down_t, f, r2)):
                groups = ops.scale_shape(rows, kr)[0] // 128
                full.view(i64).view(groups, n, kr // 64, 64).copy_(
                    pieces.view(i64).view(n, groups, kr // 64, 64).permute(1, 0, 2, 3))
            self.permuted = True


class BlockState:
    """Flat bf16 parameter / gradient buckets and fp32 Adam moments of one block.

    ``pad_to`` (>= the real size) pads both buckets with zeros so that a
    reduce-scatter divides them evenly; ``with_moments=False`` leaves the Adam
    moments to a sharded optimizer.  With ``layout`` (ShardQuantLayout) both
    buckets are rank-major and the standard-layout views (gamma, w_gu, w_down,
    grad_gu, grad_down) are None; the initial weights are the same as in the
    standard layout."""

    def __init__(self, d: int, f: int, device, gen: Optional[torch.Generator], init_std: float,
                 grad_f32: bool, pad_to: int = 0, with_moments: bool = True, master: bool = False,
                 layout: Optional[ShardQuantLayout] = None):
        self.d, self.f = d, f
        n = d + 2 * f * d + d * f
        self.numel = n
        self.layout = layout
        length = max(n, pad_to)
        self.param = torch.zeros(length, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            w = torch.empty(2 * f * d + d * f, device=device, dtype=torch.float32)
            w.normal_(0.0, init_std, generator=gen)
            if layout is None:
                self.gamma = self.param[:d]
                self.w_gu = self.param[d:d + 2 * f * d].view(2 * f, d)
                self.w_down = self.param[d + 2 * f * d:].view(d, f)
                self.gamma.fill_(1.0)
                self.param[d:n].copy_(w)
            else:
                self.gamma = self.w_gu = self.w_down = None
                wb = w.to(torch.bfloat16)
                layout.store(self.param, torch.ones(d, device=device, dtype=torch.bfloat16),
                             wb[:2 * f * d].view(2 * f, d), wb[2 * f * d:].view(d, f))
                del wb
            del w
        # bf16 gradient bucket (the all-reduce / reduce-scatter payload): gamma | W_gu | W_down | padding,
        # or rank-major with a layout
        self.grad = torch.zeros(length, device=device, dtype=torch.bfloat16)
        self.grad_gamma32 = torch.zeros(d, device=device, dtype=torch.float32)
        if layout is None:
            self.grad_gu = self.grad[d:d + 2 * f * d].view(2 * f, d)
            self.grad_down = self.grad[d + 2 * f * d:].view(d, f)
        else:
            self.grad_gu = self.grad_down = None
        if grad_f32:   # micro-batch accumulation buffers
            self.acc_gu = torch.zeros(2 * f, d, device=device, dtype=torch.float32)
            self.acc_down = torch.zeros(d, f, device=device, dtype=torch.float32)
        else:
            self.acc_gu = self.acc_down = None
        self.m = torch.zeros(length, device=device, dtype=torch.float32) if with_moments else None
        self.v = torch.zeros(length, device=device, dtype=torch.float32) if with_moments else None
        # fp32 master weights beside the moments (AdamConfig.master_weights)
        self.master = self.param.float() if (with_moments and master) else None


class NVFP4MLPStackTrainer:
    """Training step of a stack of NVFP4 RMSNorm+SwiGLU blocks.

    One step: forward over all blocks (micro-batched), backward from a given
    upstream gradient, then the fp32 AdamW update.  With a process group of
    more than one rank the per-block bf16 gradient bucket is exchanged as soon
    as the block's wgrads are done, overlapping the backward of the blocks
    below:

    * ``zero=True`` (default): reduce-scatter, AdamW of this rank's shard, and
      an all-gather that the next step waits for just before it uses that
      block's weights.  With ``shard_quant`` (default: whenever
      ShardQuantLayout fits the shapes) the buckets are rank-major, each rank
      quantizes its own rows of the updated weights in both orientations and
      the ranks gather NVFP4 weights (GatheredWeights); otherwise they gather
      the bf16 parameters and every rank quantizes all of them;
    * ``zero=False``: all-reduce and AdamW of the whole block on every rank.

    ``finish()`` waits for gathers still in flight."""

    def __init__(self, n_blocks: int, d_model: int, d_ff: int, *, device="cuda", seed: int = 0,
                 micro_tokens: int = 16384, eps: float = 1e-6, adam: Optional[AdamConfig] = None,
                 init_std: float = 0.02, process_group=None, max_local_tokens: Optional[int] = None,
                 comm_sms: int = 0, zero: bool = True, shard_quant: Optional[bool] = None):
        self.device = torch.device(device)
        self.n_blocks, self.d, self.f = n_blocks, d_model, d_ff
        self.micro_tokens = micro_tokens
        self.eps = eps
        self.adam = adam or AdamConfig()
        self.pg = process_group
        gen = torch.Generator(device=self.device).manual_seed(seed)
        grad_f32 = max_local_tokens is None or max_local_tokens > micro_tokens
        world = 1
        if process_group is not None:
            import torch.distributed as dist
            world = dist.get_world_size(process_group)
        self.world = world
        n = d_model + 3 * d_ff * d_model
        self.opt = None
        self.reducer = None
        self.layout: Optional[ShardQuantLayout] = None
        self.gathered: Optional[List[GatheredWeights]] = None
        if world > 1 and zero:
            if shard_quant is None:
                shard_quant = ShardQuantLayout.fits(d_model, d_ff, world)
            if shard_quant:
                self.layout = ShardQuantLayout(d_model, d_ff, world)
            self.opt = ShardedBucketOptimizer(process_group, {i: n for i in range(n_blocks)}, self.device,
                                              master_weights=self.adam.master_weights)
            if self.layout is not None and self.opt.padded_len(0) != n:
                raise RuntimeError("rank-major buckets must split into equal shards without padding")
            self.blocks = [BlockState(d_model, d_ff, self.device, gen, init_std, grad_f32,
                                      pad_to=self.opt.padded_len(i), with_moments=False, layout=self.layout)
                           for i in range(n_blocks)]
            if self.layout is not None:
                self.gathered = [GatheredWeights(self.layout, self.device) for _ in range(n_blocks)]
        else:
            self.blocks = [BlockState(d_model, d_ff, self.device, gen, init_std, grad_f32,
                                      master=self.adam.master_weights) for _ in range(n_blocks)]
            if world > 1:
                self.reducer = BucketAllReducer(process_group)
        self.step_count = 0
        # the weights' global scales for the next step, from the amaxes the AdamW
        # update records while writing the weights ([block, (W_gu, W_down)]); None
        # until the first update (then they are computed from the weights)
        self.w_amax = torch.zeros(n_blocks, 2, device=self.device, dtype=torch.int32)
        self.w_g: Optional[torch.Tensor] = None
        # W_gu rows interleave gate/up in blocks of 128 (fused SwiGLU epilogue) when F allows
        self.interleave = 128 if d_ff % 128 == 0 else 0
        # SMs left to the gradient collectives while the step's GEMMs run (DP only)
        self.comm_sms = comm_sms if world > 1 else 0
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count

    # -- one optimizer step -------------------------------------------------
    def step(self, x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
        """x, dy: bf16 [T_local, D] on this rank's device.  Returns a 1-element
        fp32 tensor (sum of the output, a cheap device-side step result)."""
        if self.comm_sms > 0:
            ops.set_gemm_max_sms(max(2, self.sm_count - self.comm_sms))
        try:
            return self._step(x, dy)
        finally:
            if self.comm_sms > 0:
                ops.set_gemm_max_sms(0)

    def _step(self, x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
        t = x.shape[0]
        n_micro = max(1, math.ceil(t / self.micro_tokens))
        qws: List[Optional[QWeights]] = [None] * self.n_blocks

        lay = self.layout
        if lay is not None and self.w_g is None:
            self._prime_gathered()

        def qw(bi: int) -> QWeights:   # a block's NVFP4 weights on first use (after its gather landed)
            if qws[bi] is None:
                g = self.w_g
                if lay is not None:
                    qws[bi] = self.gathered[bi].qweights(g[bi, 0:1], g[bi, 1:2])
                    return qws[bi]
                if self.opt is not None:
                    self.opt.wait_params(bi)
                b = self.blocks[bi]
                qws[bi] = quantize_weights(b.w_gu, b.w_down, need_t=True, g_gu=None if g is None else g[bi, 0:1],
                                           g_down=None if g is None else g[bi, 1:2])
            return qws[bi]

        def gamma(bi: int) -> torch.Tensor:
            return self.gathered[bi].gamma if lay is not None else self.blocks[bi].gamma

        for b in self.blocks:
            b.grad_gamma32.zero_()
        out_sum = torch.zeros(1, device=self.device, dtype=torch.float32)
        for mi in range(n_micro):
            lo, hi = mi * self.micro_tokens, min(t, (mi + 1) * self.micro_tokens)
            h = x[lo:hi]
            saved: List[Saved] = []
            for bi in range(self.n_blocks):
                q = qw(bi)
                h, sv = block_forward(h, gamma(bi), q, self.eps, interleave=self.interleave)
                saved.append(sv)
            out_sum += h.sum(dtype=torch.float32)
            g = dy[lo:hi]
            last = mi == n_micro - 1
            for bi in reversed(range(self.n_blocks)):
                b = self.blocks[bi]
                if lay is not None:
                    self.gathered[bi].ensure_transposed()
                if n_micro == 1:
                    # rank-major buckets: one wgrad GEMM per rank's row block
                    tgt_gu = lay.gu_pieces(b.grad) if lay is not None else b.grad_gu
                    tgt_down = lay.down_pieces(b.grad) if lay is not None else b.grad_down
                    g = block_backward(g, gamma(bi), qws[bi], saved[bi], b.grad_gamma32, tgt_gu, tgt_down,
                                       accumulate=False, interleave=self.interleave)
                else:
                    # the first micro-batch writes the fp32 accumulators, later ones add to them
                    g = block_backward(g, gamma(bi), qws[bi], saved[bi], b.grad_gamma32, b.acc_gu, b.acc_down,
                                       accumulate=mi > 0, interleave=self.interleave)
                    if last and self.world > 1:   # the bf16 bucket is only needed for the exchange
                        if lay is not None:   # one contiguous copy per rank's rows (vectorised)
                            gp, dp_ = lay.gu_pieces(b.grad), lay.down_pieces(b.grad)
                            for r in range(lay.world):
                                gp[r].copy_(b.acc_gu[r * lay.r1:(r + 1) * lay.r1])
                                dp_[r].copy_(b.acc_down[r * lay.r2:(r + 1) * lay.r2])
                        else:
                            b.grad_gu.copy_(b.acc_gu)
                            b.grad_down.copy_(b.acc_down)
                saved[bi] = None
                if last and (self.world > 1 or n_micro == 1):
                    if lay is not None:
                        lay.gamma_pieces(b.grad).copy_(b.grad_gamma32.view(lay.world, lay.gn))
                    else:
                        b.grad[:self.d].copy_(b.grad_gamma32)
                if last:
                    if self.opt is not None:
                        self.opt.reduce_scatter(bi, b.grad)
                    elif self.reducer is not None:
                        self.reducer.launch(bi, b.grad)
        self.step_count += 1
        a = self.adam

        def adamw(p, g, m, v, w=None, amax=None):
            kw = dict(lr=a.lr, beta1=a.beta1, beta2=a.beta2, eps=a.eps, weight_decay=a.weight_decay,
                      step=self.step_count, grad_scale=1.0 / self.world)
            if w is not None:
                ops.adamw_master_step(p, w, g, m, v, amax_bits=amax, **kw)
            else:
                ops.adamw_step(p, g, m, v, **kw)

        d, ngu = self.d, 2 * self.f * self.d
        n_real = d + ngu + self.d * self.f
        # segments of a block's flat bucket and where each one's amax goes (gamma is not quantized)
        seg_of = lambda bi: ((0, d, None), (d, d + ngu, self.w_amax[bi, 0:1]),
                             (d + ngu, n_real, self.w_amax[bi, 1:2]))
        track = a.master_weights
        if track:
            self.w_amax.zero_()

        def shard_update(bi):
            """update_fn of the ZeRO-1 optimizer for block bi: AdamW on the shard,
            split at the segment boundaries it crosses (the padding past the
            real parameters is updated as one more segment, without an amax)."""
            sl = self.opt.shard_slice(bi)

            def fn(p, g, m, v, w=None):
                if lay is not None:   # the shard is [gamma_r | W_gu rows | W_down rows]
                    for lo, hi, which in lay.segments():
                        am = None if which is None else self.w_amax[bi, which:which + 1]
                        r = slice(lo, hi)
                        adamw(p[r], g[r], m[r], v[r], None if w is None else w[r], am if track else None)
                    return
                lo0 = sl.start
                cuts = [(lo, hi, am) for lo, hi, am in seg_of(bi)] + [(n_real, sl.stop, None)]
                for lo, hi, am in cuts:
                    lo, hi = max(lo, sl.start), min(hi, sl.stop)
                    if lo < hi:
                        r = slice(lo - lo0, hi - lo0)
                        adamw(p[r], g[r], m[r], v[r], None if w is None else w[r], am if track else None)
            return fn

        # buckets were launched from the last block down: update in that order
        for bi in reversed(range(self.n_blocks)):
            b = self.blocks[bi]
            if self.opt is not None:
                self.opt.update(bi, b.param, shard_update(bi), gather=False)
            else:
                if self.reducer is not None:
                    self.reducer.wait(bi)
                if self.world == 1 and n_micro > 1:
                    # one rank, micro-batched: AdamW reads the fp32 accumulators directly
                    # (no bf16 copy of the gradient)
                    grads = (b.grad_gamma32, b.acc_gu.view(-1), b.acc_down.view(-1))
                else:
                    grads = tuple(b.grad[lo:hi] for lo, hi, _ in seg_of(bi))
                for (lo, hi, am), g in zip(seg_of(bi), grads):
                    adamw(b.param[lo:hi], g, b.m[lo:hi], b.v[lo:hi], None if b.master is None else b.master[lo:hi],
                          am if track else None)
        if lay is not None and not track:   # the update recorded no amax: take it from the shard's rows
            self._shard_amax()
        if track or lay is not None:
            if self.opt is not None:
                # each rank saw its shard of every weight: the global amax is the max over ranks
                import torch.distributed as dist
                dist.all_reduce(self.w_amax, op=dist.ReduceOp.MAX, group=self.pg)
            self.w_g = ops.global_scale_from_amax(self.w_amax)
        if self.opt is not None:
            # gathers in the order the next forward uses the blocks: block 0 lands first
            for bi, b in enumerate(self.blocks):
                if lay is not None:
                    gw = self.gathered[bi]
                    gw.quantize(self.opt.rank, b.param, self.w_g[bi, 0:1], self.w_g[bi, 1:2])
                    gw.gather_forward(self.opt.rank, b.param, self.pg)
                else:
                    self.opt.gather(bi, b.param)
            if lay is not None:   # the backward needs the last block's transposed weights first
                for bi in reversed(range(self.n_blocks)):
                    self.gathered[bi].gather_transposed(self.opt.rank, self.pg)
        return out_sum

    def _shard_amax(self) -> None:
        """w_amax from this rank's rows of every weight (rank-major buckets)."""
        lay, r = self.layout, self.opt.rank
        for bi, b in enumerate(self.blocks):
            for which, pieces in ((0, lay.gu_pieces(b.param)), (1, lay.down_pieces(b.param))):
                _, amax = ops.global_scale(pieces[r], with_amax=True)
                self.w_amax[bi, which:which + 1].copy_(amax.view(torch.int32))

    def _prime_gathered(self) -> None:
        """First step with rank-major buckets: global scales of the initial
        weights (max over ranks of the shard amaxes), then every rank quantizes
        its rows and the NVFP4 weights are gathered."""
        import torch.distributed as dist
        self._shard_amax()
        dist.all_reduce(self.w_amax, op=dist.ReduceOp.MAX, group=self.pg)
        self.w_g = ops.global_scale_from_amax(self.w_amax)
        for bi, b in enumerate(self.blocks):
            gw = self.gathered[bi]
            gw.quantize(self.opt.rank, b.param, self.w_g[bi, 0:1], self.w_g[bi, 1:2])
            gw.gather_forward(self.opt.rank, b.param, self.pg)
        for bi in reversed(range(self.n_blocks)):
            self.gathered[bi].gather_transposed(self.opt.rank, self.pg)

    def gather_masters(self) -> List[tuple]:
        """Standard-layout fp32 (gamma, W_gu, W_down) of every block: the master
        weights (the bf16 parameters widened when there are none).  Collective
        under ZeRO-1 (every rank must call it)."""
        out = []
        for bi, b in enumerate(self.blocks):
            if self.opt is None:
                full = b.master if b.master is not None else b.param.float()
            else:
                import torch.distributed as dist
                sh = self.opt.w.get(bi) if self.adam.master_weights else None
                if sh is None:
                    sh = b.param[self.opt.shard_slice(bi)].float()
                full = torch.empty(sh.numel() * self.world, device=self.device, dtype=torch.float32)
                dist.all_gather_into_tensor(full, sh.contiguous(), group=self.pg)
            if self.layout is not None:
                out.append(self.layout.load(full))
            else:
                d, f = self.d, self.f
                out.append((full[:d].clone(), full[d:d + 2 * f * d].view(2 * f, d).clone(),
                            full[d + 2 * f * d:d + 3 * f * d].view(d, f).clone()))
        return out

    def finish(self) -> None:
        """Make the current stream wait for every gather still in flight."""
        if self.opt is not None:
            self.opt.wait_all()
        for gw in self.gathered or ():
            gw.wait()

    def flops_per_step(self, tokens: int) -> float:
        return 3 * 3 * 2.0 * tokens * self.d * self.f * self.n_blocks
