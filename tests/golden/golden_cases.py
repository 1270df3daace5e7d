"""Seeded inputs for the golden fixtures (shared by make_golden.py and the tests).

Every generator is deterministic (CPU ``torch.Generator``), and the fixture
files store a sha256 of each input so a drift in the generator is caught
instead of silently comparing different data.  Inputs are returned as bf16
bit patterns (numpy uint16).
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config0_a_w():
    """Round-trip workload, seed 0: A [256x512] N(0,1) with 0.1% of entries x20
    (positions from randperm), W [1024x512] N(0, 0.02)."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(256, 512, generator=g, dtype=torch.float32)
    n_out = int(round(0.001 * a.numel()))
    idx = torch.randperm(a.numel(), generator=g)[:n_out]
    a.view(-1)[idx] *= 20.0
    w = torch.randn(1024, 512, generator=g, dtype=torch.float32) * 0.02
    return bits(a.to(torch.bfloat16)), bits(w.to(torch.bfloat16))


def ties_case():
    """Blocks whose scale decodes exactly to 2^e, with elements exactly on
    every E2M1 rounding threshold (and their bf16 neighbours), both signs."""
    thr = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    rows = []
    for e in range(-6, 7):
        s = 2.0 ** e
        for variant in range(4):
            blk = [6.0 * s]  # amax = 6 * 2^e  -> scale 2^e exactly
            for t in thr:
                v = t * s
                if variant == 1:
                    v = -v
                blk.append(v)
            blk += [0.0, -0.0, 6.0 * s * (-1 if variant & 1 else 1), 0.5 * s,
                    -1.0 * s, 3.0 * s, 4.0 * s, -2.0 * s]
            blk = blk[:16]
            x = torch.tensor(blk, dtype=torch.float32)
            if variant == 2:   # nudge to the bf16 neighbour above each threshold
                xb = x.to(torch.bfloat16)
                x = torch.nextafter(xb.float(), torch.full_like(x, math.inf)).to(torch.bfloat16).float()
                x[0] = 6.0 * s
            if variant == 3:   # and below
                x = torch.nextafter(x.to(torch.bfloat16).float(), torch.zeros_like(x)).to(torch.bfloat16).float()
                x[0] = 6.0 * s
            rows.append(x)
    x = torch.stack(rows)                     # [52, 16]
    x = x.reshape(-1, 64)                     # 4 blocks per row
    return bits(x.to(torch.bfloat16))


def special_case():
    """Zero blocks, signed zeros, NaN, +-Inf, subnormal/underflowing and
    saturating block scales."""
    g = torch.Generator().manual_seed(11)
    x = torch.randn(64, 64, generator=g)
    x[0, :16] = 0.0
    x[0, 16:32] = -0.0
    x[1, 3] = float("nan")
    x[1, 20] = float("inf")
    x[1, 40] = float("-inf")
    x[2, :] = float("nan")
    x[3, :16] *= 1e-3      # E4M3 subnormal block scale
    x[3, 16:32] *= 1e-5    # block scale underflows to zero
    x[3, 32:48] *= 1e-40   # bf16 subnormal inputs
    x[4, :16] *= 1e4       # saturating block scale (448)
    x[4, 16:32] = 3e38
    x[5, :] = -x[5, :].abs()
    return bits(x.to(torch.bfloat16))


def scale_sweep_case():
    """Block amax log-uniform over [1e-8, 1e5]: exercises every E4M3 code
    including subnormal, underflow-to-zero and saturation."""
    g = torch.Generator().manual_seed(12)
    x = torch.randn(256, 64, generator=g)
    amax = torch.exp(torch.empty(256, 4).uniform_(math.log(1e-8), math.log(1e5), generator=g))
    x = x.reshape(256, 4, 16)
    x = x / x.abs().amax(-1, keepdim=True) * amax[..., None]
    return bits(x.reshape(256, 64).to(torch.bfloat16))


SHAPES = [(1, 16), (127, 48), (129, 80), (300, 512), (37, 1024), (6, 64), (128, 16), (2, 4096)]


def shape_case(r: int, k: int, seed: int):
    g = torch.Generator().manual_seed(1000 + seed)
    return bits((torch.randn(r, k, generator=g) * 3.0).to(torch.bfloat16))


def rms_rowscale_case(r: int = 129, k: int = 4096):
    """x ~ N(0,1) times a per-row scale log-uniform in [0.1, 10] (seed 2)."""
    g = torch.Generator().manual_seed(2)
    x = torch.randn(r, k, generator=g)
    rs = torch.exp(torch.empty(r, 1).uniform_(math.log(0.1), math.log(10.0), generator=g))
    return bits((x * rs).to(torch.bfloat16))


def gemm_k4096_case():
    g = torch.Generator().manual_seed(1)
    a = torch.randn(128, 4096, generator=g).to(torch.bfloat16)
    b = torch.randn(256, 4096, generator=g).to(torch.bfloat16)
    return bits(a), bits(b)


def quant_cases():
    """name -> bf16 bits [R, K] for the plain quantizer fixtures."""
    a, w = config0_a_w()
    cases = {"cfg0_A": a, "cfg0_W": w, "ties": ties_case(), "special": special_case(),
             "scale_sweep": scale_sweep_case()}
    for i, (r, k) in enumerate(SHAPES):
        cases[f"shape_{r}x{k}"] = shape_case(r, k, i)
    return cases


def rms_cases():
    a, _ = config0_a_w()
    z = shape_case(3, 64, 99)
    z[1, :] = 0
    return {"rms_cfg0": a, "rms_rowscale": rms_rowscale_case(),
            "rms_k16": shape_case(5, 16, 98), "rms_zero_row": z}
