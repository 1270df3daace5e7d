"""ctypes binding of the C ABI declared in ``include/nvfp4_b200.h``.

This is the same binding a user of the reference would add to call the
library from Python (the reference's ops are reached through the torch
dispatcher instead, cutlass_mm_fp4.cu:479-486).  There is no fallback: if the
shared library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import _build

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_float = ctypes.c_float

# name -> argument types (all return int status)
SIGNATURES = {
    "nvfp4b200_api_version": [],
    "nvfp4b200_device_check": [],
    "nvfp4b200_get_device_error": [ctypes.POINTER(c_int)],
    "nvfp4b200_set_gemm_max_sms": [c_int],
    "nvfp4b200_wait_selftest": [c_i64, c_void_p],
    "nvfp4b200_quant_nvfp4": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_void_p, c_void_p],
    "nvfp4b200_scaled_quant_nvfp4": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_void_p,
                                     c_void_p],
    "nvfp4b200_rmsnorm_quant_nvfp4": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                                      c_void_p, c_void_p],
    "nvfp4b200_rmsnorm_stats": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_void_p, c_void_p, c_void_p],
    "nvfp4b200_quant_nvfp4_t": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_void_p, c_void_p],
    "nvfp4b200_global_scale": [c_void_p, c_i64, c_void_p, c_void_p, c_void_p, c_void_p],
    "nvfp4b200_global_scale_noalloc": [c_void_p, c_i64, c_void_p, c_void_p, c_void_p],
    "nvfp4b200_nvfp4_mm": [c_void_p] * 7 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_mxfp4_mm": [c_void_p] * 6 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_nvfp4_mm_relu": [c_void_p] * 7 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_nvfp4_mm_relu_2": [c_void_p] * 7 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_gemm": [c_void_p] * 9 + [c_int] * 3 + [c_i64] * 4 + [c_void_p],
    "nvfp4b200_swiglu_fwd": [c_void_p, c_void_p, c_i64, c_i64, c_int, c_void_p, c_void_p, c_void_p],
    "nvfp4b200_swiglu_bwd": [c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_int, c_void_p, c_void_p, c_void_p],
    "nvfp4b200_gemm_swiglu": [c_void_p] * 10 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_gemm_dswiglu": [c_void_p] * 10 + [c_i64] * 3 + [c_void_p],
    "nvfp4b200_rmsnorm_bwd": [c_void_p] * 7 + [c_i64, c_i64, c_void_p],
    "nvfp4b200_add_bf16": [c_void_p, c_void_p, c_void_p, c_i64, c_void_p],
    "nvfp4b200_adamw_step": [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_i64] + [c_float] * 8 + [c_void_p],
    "nvfp4b200_adamw_master_step": [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_i64] + [c_float] * 8
                                   + [c_void_p, c_void_p],
    "nvfp4b200_global_scale_from_amax": [c_void_p, c_void_p, c_i64, c_void_p],
}

_lock = threading.Lock()
_lib = None


class NVFP4Error(RuntimeError):
    pass


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = False):
    """Load the shared library (once).  Raises when it is not available."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if build_if_missing:
                _build.build()
            else:
                raise NVFP4Error(
                    f"NVFP4 B200 CUDA library not found at {path}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
        lib = ctypes.CDLL(path)
        lib.nvfp4b200_status_string.restype = ctypes.c_char_p
        lib.nvfp4b200_status_string.argtypes = [c_int]
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = c_int
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(rc: int) -> str:
    return load().nvfp4b200_status_string(rc).decode()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise NVFP4Error(f"{what} failed: {status_string(rc)} (status {rc})")


def call(name: str, *args) -> None:
    lib = load()
    check(getattr(lib, name)(*args), name)


def exported_symbols():
    return ["nvfp4b200_status_string"] + list(SIGNATURES)
