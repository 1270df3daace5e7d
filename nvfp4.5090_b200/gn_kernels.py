"""Drop-in for the ``gn_kernels`` NVFP4 GEMM ops used by the reference.

The reference calls ``gn_kernels.cutlass_nvfp4_mm(a, b.mT, s_a, s_b,
output_scale)`` (float4utils.py:456, 462) and the relu / relu^2 variants
(:482, :508), backed by the CUDA impls registered in cutlass_mm_fp4.cu:479-486
with the C++ signature

    Tensor (Tensor A, Tensor B, Tensor scales_A, Tensor scales_B,
            Tensor output_scale, Tensor? bias)                (cutlass_mm_fp4.cu:167-173)

Here the same schema is registered as torch custom ops in the ``nvfp4_b200``
namespace (with fake/meta implementations, so they trace under
``torch.compile``), backed by the tcgen05 GEMM of this library; importing
this module also registers the reference's own op names
``torch.ops.gn_kernels.cutlass_sm120a_*`` (``register_reference_namespace``).  A is packed
E2M1 [M, K/2]; B is the reference's column-major operand ([K/2, N], i.e. the
``.mT`` of a row-major [N, K/2] weight); the result is bf16 [M, N]
(cutlass_mm_fp4.cu:175-178).  To use them where the reference imports
``gn_kernels``, alias the module: ``sys.modules["gn_kernels"] = this module``.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .ops import _stream, scale_shape

FP4_DTYPE = torch.float4_e2m1fn_x2

_EPI = {"cutlass_nvfp4_mm": "nvfp4b200_nvfp4_mm", "cutlass_nvfp4_mm_relu": "nvfp4b200_nvfp4_mm_relu",
        "cutlass_nvfp4_mm_relu_2": "nvfp4b200_nvfp4_mm_relu_2"}


def _b_rows(B: torch.Tensor) -> torch.Tensor:
    """Row-major [N, K/2] storage of the column-major B operand."""
    bt = B.mT
    if not bt.is_contiguous():
        raise RuntimeError("B must be the column-major [K/2, N] view of a contiguous [N, K/2] operand (b.mT)")
    return bt


def _run(entry: str, A, B, scales_A, scales_B, output_scale, bias):
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("NVFP4 GEMM expects 2-D operands")
    m = A.size(0)
    k = A.size(1) * 2          # cutlass_mm_fp4.cu:176
    n = B.size(1)              # cutlass_mm_fp4.cu:177
    if B.size(0) * 2 != k:
        raise RuntimeError(f"K mismatch: A has K={k}, B has K={B.size(0) * 2}")
    A = A.contiguous()
    bt = _b_rows(B)
    sa, sb = scales_A.contiguous(), scales_B.contiguous()
    if sa.numel() != scale_shape(m, k)[0] * scale_shape(m, k)[1] or \
            sb.numel() != scale_shape(n, k)[0] * scale_shape(n, k)[1]:
        raise RuntimeError("scale tensors must use the padded 128x4 swizzled layout")
    if output_scale.dtype != torch.float32 or output_scale.numel() != 1 or not output_scale.is_cuda:
        raise RuntimeError("output_scale must be a 1-element float32 CUDA tensor")
    out = torch.empty((m, n), device=A.device, dtype=torch.bfloat16)
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != n:
            raise RuntimeError("bias must be bf16 [N]")
        bias = bias.contiguous()
    _lib.call(entry, A.data_ptr(), bt.data_ptr(), sa.data_ptr(), sb.data_ptr(), output_scale.data_ptr(),
              None if bias is None else bias.data_ptr(), out.data_ptr(), m, n, k, _stream(A))
    return out


def _define(name: str):
    entry = _EPI[name]

    @torch.library.custom_op(f"nvfp4_b200::{name}", mutates_args=(), device_types="cuda")
    def op(A: torch.Tensor, B: torch.Tensor, scales_A: torch.Tensor, scales_B: torch.Tensor,
           output_scale: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        return _run(entry, A, B, scales_A, scales_B, output_scale, bias)

    @op.register_fake
    def _(A, B, scales_A, scales_B, output_scale, bias=None):
        return A.new_empty((A.size(0), B.size(1)), dtype=torch.bfloat16)

    return op


@torch.library.custom_op("nvfp4_b200::cutlass_mxfp4_mm", mutates_args=(), device_types="cuda")
def cutlass_mxfp4_mm(A: torch.Tensor, B: torch.Tensor, scales_A: torch.Tensor, scales_B: torch.Tensor,
                     bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """MXFP4 op of cutlass_mm_fp4.cu:71-165: bf16(A . B^T + bias) with UE8M0
    scales per 1x32 block (no output scale).  A [M, K/2] packed, B the
    column-major [K/2, N] operand, scales in the 128x4-atom swizzled layout
    with one column per 32 k."""
    from .ops import mxfp4_mm
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("MXFP4 GEMM expects 2-D operands")
    if B.size(0) * 2 != A.size(1) * 2:
        raise RuntimeError(f"K mismatch: A has K={A.size(1) * 2}, B has K={B.size(0) * 2}")
    return mxfp4_mm(A.contiguous(), scales_A.contiguous(), _b_rows(B), scales_B.contiguous(), bias)


@cutlass_mxfp4_mm.register_fake
def _(A, B, scales_A, scales_B, bias=None):
    return A.new_empty((A.size(0), B.size(1)), dtype=torch.bfloat16)


cutlass_nvfp4_mm = _define("cutlass_nvfp4_mm")
cutlass_nvfp4_mm_relu = _define("cutlass_nvfp4_mm_relu")
cutlass_nvfp4_mm_relu_2 = _define("cutlass_nvfp4_mm_relu_2")


# ----------------------------------------------------------------------------
# The reference's own op names: gn_kernels::cutlass_sm120a_* (cutlass_mm_fp4.cu:479-486)
# ----------------------------------------------------------------------------

# Schema strings restate the C++ signatures cutlass_mm_fp4.cu:71-76 (MXFP4) and
# :167-173 (NVFP4; the relu variants :275-281 and :378-384 are identical).
_NVFP4_SCHEMA = ("(Tensor A, Tensor B, Tensor scales_A, Tensor scales_B, Tensor output_scale, "
                 "Tensor? bias=None) -> Tensor")
_MXFP4_SCHEMA = "(Tensor A, Tensor B, Tensor scales_A, Tensor scales_B, Tensor? bias=None) -> Tensor"
REFERENCE_OPS = {
    "cutlass_sm120a_nvfp4_mm": (_NVFP4_SCHEMA, "nvfp4b200_nvfp4_mm"),
    "cutlass_sm120a_nvfp4_mm_relu": (_NVFP4_SCHEMA, "nvfp4b200_nvfp4_mm_relu"),
    "cutlass_sm120a_nvfp4_mm_relu_2": (_NVFP4_SCHEMA, "nvfp4b200_nvfp4_mm_relu_2"),
    "cutlass_sm120a_mxfp4_mm": (_MXFP4_SCHEMA, None),
}
_ref_lib = None
_ref_defined = []


def _ref_nvfp4_impl(entry):
    def impl(A, B, scales_A, scales_B, output_scale, bias=None):
        return _run(entry, A, B, scales_A, scales_B, output_scale, bias)
    return impl


def _ref_mxfp4_impl(A, B, scales_A, scales_B, bias=None):
    from .ops import mxfp4_mm
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("MXFP4 GEMM expects 2-D operands")
    if B.size(0) != A.size(1):
        raise RuntimeError(f"K mismatch: A has K={A.size(1) * 2}, B has K={B.size(0) * 2}")
    return mxfp4_mm(A.contiguous(), scales_A.contiguous(), _b_rows(B), scales_B.contiguous(), bias)


def _op_exists(name: str) -> bool:
    try:
        getattr(torch.ops.gn_kernels, name)
        return True
    except (AttributeError, RuntimeError):
        return False


def register_reference_namespace() -> list:
    """Make ``torch.ops.gn_kernels.cutlass_sm120a_{nvfp4_mm, nvfp4_mm_relu,
    nvfp4_mm_relu_2, mxfp4_mm}`` run this library's kernels on CUDA tensors,
    as cutlass_mm_fp4.cu:479-486 registers the reference's CUTLASS kernels.

    When the gn-kernels package already defined an op's schema, only the CUDA
    implementation is registered (it replaces the package's SM120 kernel);
    otherwise the schema is defined here too, with a fake (meta)
    implementation so the op traces under torch.compile.  Idempotent; returns
    the names whose schema this module defined."""
    global _ref_lib
    if _ref_lib is not None:
        return list(_ref_defined)
    lib = torch.library.Library("gn_kernels", "FRAGMENT")
    for name, (schema, entry) in REFERENCE_OPS.items():
        if not _op_exists(name):
            lib.define(name + schema)
            _ref_defined.append(name)

            def fake(A, B, *rest, **kw):
                return A.new_empty((A.size(0), B.size(1)), dtype=torch.bfloat16)

            torch.library.register_fake(f"gn_kernels::{name}", fake, lib=lib)
        lib.impl(name, _ref_nvfp4_impl(entry) if entry else _ref_mxfp4_impl, "CUDA")
    _ref_lib = lib
    return list(_ref_defined)


register_reference_namespace()

__all__ = ["FP4_DTYPE", "cutlass_nvfp4_mm", "cutlass_nvfp4_mm_relu", "cutlass_nvfp4_mm_relu_2", "cutlass_mxfp4_mm",
           "register_reference_namespace", "REFERENCE_OPS"]
