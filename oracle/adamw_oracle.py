"""float32 restatement of the training step's AdamW updates.  TEST INFRASTRUCTURE ONLY.

The reference trains with torch's optimizers on bf16 parameters (it ships no
optimizer code); the MLP step here updates parameters with its own CUDA
kernels, so the oracle for them is the published AdamW algorithm
(Loshchilov & Hutter, "Decoupled Weight Decay Regularization"), written
twice in numpy float32, one IEEE-rounded operation at a time, in the order
each kernel evaluates it:

* ``adamw_bf16``: the bf16-parameter update without a master copy
  (``nvfp4b200_adamw_step``);
* ``adamw_master``: the fp32-master update in torch.optim.AdamW's order of
  operations (``nvfp4b200_adamw_master_step``).

numpy float32 +, -, *, / and sqrt are correctly rounded, so the kernels
(explicit ``__f*_rn`` intrinsics, no FMA contraction) must agree bit for bit.
"""
from __future__ import annotations

import math

import numpy as np

from . import nvfp4_oracle as orc

F32 = np.float32


def _grad_f32(grad) -> np.ndarray:
    g = np.asarray(grad)
    if g.dtype == np.uint16:          # bf16 bit patterns
        return orc.bf16_bits_to_f32(g)
    return g.astype(np.float32)


def adamw_bf16(p_bits, grad, m, v, *, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0):
    """One step on bf16 parameter bits ``p_bits`` (uint16), fp32 ``m``/``v``.

    g = grad*gs; m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*(g*g);
    p = p - lr*((m/bc1)/(sqrt(v/bc2)+eps) + wd*p), rounded to bf16.
    Returns (new p bits, m, v)."""
    b1, b2 = F32(beta1), F32(beta2)
    bc1, bc2 = F32(1.0 - beta1 ** step), F32(1.0 - beta2 ** step)
    g = _grad_f32(grad) * F32(grad_scale)
    m = b1 * m.astype(np.float32) + (F32(1.0) - b1) * g
    v = b2 * v.astype(np.float32) + (F32(1.0) - b2) * (g * g)
    mh, vh = m / bc1, v / bc2
    p = orc.bf16_bits_to_f32(p_bits)
    upd = mh / (np.sqrt(vh) + F32(eps)) + F32(weight_decay) * p
    p = p - F32(lr) * upd
    return orc.f32_to_bf16_bits(p.astype(np.float32)), m.astype(np.float32), v.astype(np.float32)


def master_scalars(lr, beta1, beta2, eps, weight_decay, step):
    """The float32 scalars of step t as the host passes them to the kernel
    (computed in double precision, then rounded to float32)."""
    return dict(one_minus_lr_wd=F32(1.0 - lr * weight_decay), one_minus_b1=F32(1.0 - beta1), b2=F32(beta2),
                one_minus_b2=F32(1.0 - beta2), eps=F32(eps), step_size=F32(lr / (1.0 - beta1 ** step)),
                bc2_sqrt=F32(math.sqrt(1.0 - beta2 ** step)))


def adamw_master(w, grad, m, v, *, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0):
    """One step on an fp32 master ``w`` in torch.optim.AdamW's order:
    w = w*(1-lr*wd); m = m + (1-b1)*(g-m); v = b2*v + (1-b2)*(g*g);
    w = w - (lr/bc1) * (m / (sqrt(v)/sqrt(bc2) + eps)).
    Returns (w, m, v, bf16 bits of w)."""
    s = master_scalars(lr, beta1, beta2, eps, weight_decay, step)
    g = _grad_f32(grad) * F32(grad_scale)
    w = w.astype(np.float32) * s["one_minus_lr_wd"]
    m = m.astype(np.float32) + s["one_minus_b1"] * (g - m.astype(np.float32))
    v = v.astype(np.float32) * s["b2"] + s["one_minus_b2"] * (g * g)
    denom = np.sqrt(v) / s["bc2_sqrt"] + s["eps"]
    w = w - s["step_size"] * (m / denom)
    w = w.astype(np.float32)
    return w, m.astype(np.float32), v.astype(np.float32), orc.f32_to_bf16_bits(w)
