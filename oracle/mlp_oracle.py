"""CPU emulation of the NVFP4 SwiGLU MLP block.  TEST INFRASTRUCTURE ONLY.

Dequantize-then-matmul emulation of ``nvfp4.5090_b200/mlp.py`` (the
reference has no MLP; its NVFP4 GEMM contract is cutlass_mm_fp4.cu:182-184
and its quantizer float4utils.py:79-148, both restated in nvfp4_oracle.py).
Every GEMM operand is quantized with the oracle quantizer and its global
scale g = amax/(6*448), dequantized exactly, multiplied in float64 and
rounded to bf16 at the same points where the CUDA path stores bf16.
"""
from __future__ import annotations

import numpy as np

from . import nvfp4_oracle as orc

F32 = np.float32


def _bf16(x):
    return orc.bf16_bits_to_f32(orc.f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


def _qdq(x_f32: np.ndarray) -> np.ndarray:
    """quantize along the last dim with its own global scale, dequantize (float64)."""
    x_f32 = np.ascontiguousarray(x_f32, dtype=np.float32)
    g = orc.global_scale_of(x_f32)
    q, s = orc.quant_nvfp4_f32(x_f32, g)
    return orc.dequant_nvfp4(q, s, *x_f32.shape).astype(np.float64) * float(g)


def _qdq_g(x_f32: np.ndarray, g) -> np.ndarray:
    x_f32 = np.ascontiguousarray(x_f32, dtype=np.float32)
    q, s = orc.quant_nvfp4_f32(x_f32, g)
    return orc.dequant_nvfp4(q, s, *x_f32.shape).astype(np.float64) * float(g)


def _sigmoid(x):
    return (F32(1.0) / (F32(1.0) + np.exp(-x.astype(np.float32)))).astype(np.float32)


def block_forward(x, gamma, w_gu, w_down, inv_rms):
    """x [T,D], gamma [D], w_gu [2F,D], w_down [D,F]: float32 arrays holding bf16 values;
    inv_rms [T] float32 (the kernel's own 1/RMS)."""
    xn = ((x * inv_rms[:, None]).astype(np.float32) * gamma[None, :]).astype(np.float32)
    g_xn = orc.global_scale_of(xn)
    a = _qdq_g(xn, g_xn)
    g_gu = orc.global_scale_of(w_gu)
    gu = _bf16(a @ _qdq_g(w_gu, g_gu).T)
    f = gu.shape[1] // 2
    gate, up = gu[:, :f], gu[:, f:]
    h = _bf16(gate * _sigmoid(gate) * up)
    g_h = orc.global_scale_of(h)
    g_d = orc.global_scale_of(w_down)
    y = _bf16((_qdq_g(h, g_h) @ _qdq_g(w_down, g_d).T) + x.astype(np.float64))
    return y, dict(xn=xn, g_xn=g_xn, g_gu=g_gu, gu=gu, h=h, g_h=g_h, g_d=g_d)


def block_backward(dy, x, gamma, w_gu, w_down, inv_rms, sv):
    g_dy = orc.global_scale_of(dy)
    dh = _bf16(_qdq_g(dy, g_dy) @ _qdq_g(np.ascontiguousarray(w_down.T), sv["g_d"]).T)
    d_down = _bf16(_qdq_g(np.ascontiguousarray(dy.T), g_dy) @ _qdq_g(np.ascontiguousarray(sv["h"].T), sv["g_h"]).T)
    gu = sv["gu"]
    f = gu.shape[1] // 2
    gate, up = gu[:, :f], gu[:, f:]
    s = _sigmoid(gate)
    d_up = _bf16(dh * (gate * s))
    d_gate = _bf16(dh * up * (s * (F32(1.0) + gate * (F32(1.0) - s))))
    dgu = np.concatenate([d_gate, d_up], axis=1)
    g_dgu = orc.global_scale_of(dgu)
    dxn = _bf16(_qdq_g(dgu, g_dgu) @ _qdq_g(np.ascontiguousarray(w_gu.T), sv["g_gu"]).T)
    d_gu = _bf16(_qdq_g(np.ascontiguousarray(dgu.T), g_dgu) @ _qdq_g(np.ascontiguousarray(sv["xn"].T), sv["g_xn"]).T)
    xnr = (x * inv_rms[:, None]).astype(np.float32)
    dyg = (dxn * gamma[None, :]).astype(np.float64)
    mean = np.sum(dyg * xnr, axis=1, keepdims=True) / x.shape[1]
    dx = _bf16(inv_rms[:, None] * (dyg - xnr * mean) + dy)
    dgamma = np.sum(dxn.astype(np.float64) * xnr, axis=0)
    return dx, dgamma, d_gu, d_down
