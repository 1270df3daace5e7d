"""Generate the golden fixtures from the REFERENCE's own kernels (needs a GPU).

* Quantizer fixtures: the reference's ``quant_nvfp4_fused_opt`` and
  ``rmsnorm_quant_nvfp4_smem_opt`` kernels (float4utils.py:79-148, :169-295),
  compiled from their source by ``oracle/build_ref.py`` into
  ``oracle/_ref/libnvfp4_ref.so``, launched with the reference wrappers'
  geometry and buffer conventions (``q`` uninitialised, ``s`` zero-filled,
  float4utils.py:347-348, :378-382).
* GEMM fixtures: the reference's Blackwell GEMM route ``nvfp4mm_torch``
  (float4utils.py:427-436): ``torch.nn.functional.scaled_mm`` with
  BlockWise1x16 scales in the SWIZZLE_32_4_4 layout, on operands quantized by
  the reference kernel.

Usage (on a machine with a B200):
    python oracle/build_ref.py            # in a tree that has the reference
    python tests/golden/make_golden.py --out /tmp/golden
and copy the resulting ``golden_*.npz`` next to this file.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
import golden_cases as gc  # noqa: E402

REF_SO = os.path.join(ROOT, "oracle", "_ref", "libnvfp4_ref.so")


def round_up(x, m):
    return (x + m - 1) // m * m


def to_dev_bf16(bits_u16: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(bits_u16.astype(np.uint16).view(np.int16).copy())
    return t.view(torch.bfloat16).cuda()


class Ref:
    def __init__(self, path=REF_SO):
        self.lib = ctypes.CDLL(path)
        self.lib.ref_quant_nvfp4.restype = ctypes.c_int
        self.lib.ref_quant_nvfp4.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        self.lib.ref_rmsnorm_quant_nvfp4.restype = ctypes.c_int
        self.lib.ref_rmsnorm_quant_nvfp4.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + \
            [ctypes.c_float, ctypes.c_void_p]

    def quant(self, x_bits: np.ndarray):
        r, k = x_bits.shape
        x = to_dev_bf16(x_bits)
        cols = k // 16
        pad_r, pad_c = round_up(r, 128), round_up(cols, 4)
        q = torch.empty((r, k // 2), device="cuda", dtype=torch.uint8)
        s = torch.zeros((pad_r, pad_c), device="cuda", dtype=torch.uint8)
        st = torch.cuda.current_stream().cuda_stream
        rc = self.lib.ref_quant_nvfp4(x.data_ptr(), q.data_ptr(), s.data_ptr(), r * cols, cols, pad_c, st)
        assert rc == 0, rc
        torch.cuda.synchronize()
        return q.cpu().numpy(), s.cpu().numpy()

    def rmsnorm_quant(self, x_bits: np.ndarray, eps: float):
        r, k = x_bits.shape
        x = to_dev_bf16(x_bits)
        cols = k // 16
        pad_r, pad_c = round_up(r, 128), round_up(cols, 4)
        q = torch.empty((r, k // 2), device="cuda", dtype=torch.uint8)
        s = torch.zeros((pad_r, pad_c), device="cuda", dtype=torch.uint8)
        inv = torch.empty((r,), device="cuda", dtype=torch.float32)
        st = torch.cuda.current_stream().cuda_stream
        rc = self.lib.ref_rmsnorm_quant_nvfp4(x.data_ptr(), q.data_ptr(), s.data_ptr(), inv.data_ptr(),
                                              r, k, pad_c, eps, st)
        assert rc == 0, rc
        torch.cuda.synchronize()
        return q.cpu().numpy(), s.cpu().numpy(), inv.cpu().numpy()


def scaled_mm_ref(qa, sa, qb, sb, m, n, k):
    """float4utils.py:427-436 on pre-quantized operands; returns (bf16 bits, note)."""
    import torch.nn.functional as F
    from torch.nn.functional import ScalingType, SwizzleType
    a = torch.from_numpy(qa).cuda().view(torch.float4_e2m1fn_x2)
    b = torch.from_numpy(qb).cuda().view(torch.float4_e2m1fn_x2)
    s_a = torch.from_numpy(sa).cuda().view(torch.float8_e4m3fn)
    s_b = torch.from_numpy(sb).cuda().view(torch.float8_e4m3fn)
    try:
        c = F.scaled_mm(a, b.mT, s_a, ScalingType.BlockWise1x16, s_b, ScalingType.BlockWise1x16,
                        swizzle_a=SwizzleType.SWIZZLE_32_4_4, swizzle_b=SwizzleType.SWIZZLE_32_4_4,
                        output_dtype=torch.bfloat16, contraction_dim=(1, 0))
        note = "scaled_mm(BlockWise1x16, SWIZZLE_32_4_4) as float4utils.py:427-436"
    except Exception as e:  # record the reason, retry with an explicit unit tensor-wise scale
        one = torch.ones((), device="cuda", dtype=torch.float32)
        c = F.scaled_mm(a, b.mT, [s_a, one], [ScalingType.BlockWise1x16, ScalingType.TensorWise],
                        [s_b, one], [ScalingType.BlockWise1x16, ScalingType.TensorWise],
                        swizzle_a=[SwizzleType.SWIZZLE_32_4_4, SwizzleType.NO_SWIZZLE],
                        swizzle_b=[SwizzleType.SWIZZLE_32_4_4, SwizzleType.NO_SWIZZLE],
                        output_dtype=torch.bfloat16)
        note = f"plain call raised {type(e).__name__}: {str(e)[:200]}; used [BlockWise1x16, TensorWise(1.0)]"
    torch.cuda.synchronize()
    assert c.shape == (m, n), c.shape
    return gc.bits(c.cpu()), note


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args(argv)
    os.makedirs(args.out, exist_ok=True)
    ref = Ref()

    quant = {}
    for name, x in gc.quant_cases().items():
        q, s = ref.quant(x)
        quant[f"{name}__q"] = q
        quant[f"{name}__s"] = s
        quant[f"{name}__sha"] = np.array(gc.sha(x))
        quant[f"{name}__shape"] = np.array(x.shape)
    np.savez_compressed(os.path.join(args.out, "golden_quant.npz"), **quant)

    rms = {}
    eps = 1e-6
    for name, x in gc.rms_cases().items():
        q, s, inv = ref.rmsnorm_quant(x, eps)
        rms[f"{name}__q"] = q
        rms[f"{name}__s"] = s
        rms[f"{name}__inv_rms"] = inv
        rms[f"{name}__sha"] = np.array(gc.sha(x))
        rms[f"{name}__shape"] = np.array(x.shape)
    rms["eps"] = np.array(eps, dtype=np.float32)
    np.savez_compressed(os.path.join(args.out, "golden_rmsnorm.npz"), **rms)

    gemm = {}
    notes = {}
    a, w = gc.config0_a_w()
    ka, kb = gc.gemm_k4096_case()
    for name, (xa, xb) in {"cfg0": (a, w), "k4096": (ka, kb)}.items():
        qa, sa = ref.quant(xa)
        qb, sb = ref.quant(xb)
        m, k = xa.shape
        n = xb.shape[0]
        d, note = scaled_mm_ref(qa, sa, qb, sb, m, n, k)
        gemm[f"{name}__qa"], gemm[f"{name}__sa"] = qa, sa
        gemm[f"{name}__qb"], gemm[f"{name}__sb"] = qb, sb
        gemm[f"{name}__d"] = d
        gemm[f"{name}__mnk"] = np.array([m, n, k])
        notes[name] = note
    gemm["notes"] = np.array(json.dumps(notes))
    np.savez_compressed(os.path.join(args.out, "golden_gemm.npz"), **gemm)
    print(json.dumps({"quant_cases": len(gc.quant_cases()), "rms_cases": len(gc.rms_cases()),
                      "gemm_notes": notes, "device": torch.cuda.get_device_name()}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
