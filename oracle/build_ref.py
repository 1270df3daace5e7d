"""Build recipe for oracle/_ref/: the reference's quantizer kernels, compiled
from their source where it lies.  TEST INFRASTRUCTURE ONLY.

The reference ships its two quantizer kernels as CUDA C source strings inside
``float4utils.py`` (``_KERNEL_NVFP4_FUSED`` float4utils.py:62-150,
``_KERNEL_RMSNORM_NVFP4_SMEM`` float4utils.py:152-297), compiled at run time
by CuPy/NVRTC.  Neither CuPy nor the reference's ``gn_kernels`` dependency is
installed, so the module cannot be imported; instead this recipe parses the
file (``ast``, no import, no execution), writes each string to a temporary
directory outside the repository, and compiles it with nvcc for sm_100a
together with the host launchers in ``oracle/ref_launch.cu`` into
``oracle/_ref/libnvfp4_ref.so``.  Nothing from the reference is copied into
the repository; the shared object is git-ignored and only travels to the GPU
machine, where ``tests/golden/make_golden.py`` runs it to produce golden
vectors.

Usage:  python oracle/build_ref.py [--reference DIR]
The reference location is DIR, else the NVFP4_REFERENCE_DIR environment
variable, else this recipe's default (where this build reads it).
"""
from __future__ import annotations

import argparse
import ast
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT_SO = os.path.join(OUT_DIR, "libnvfp4_ref.so")
DEFAULT_REFERENCE = "/root/reference"


def reference_dir() -> str:
    """Where the reference tree is read from: $NVFP4_REFERENCE_DIR or the default."""
    return os.environ.get("NVFP4_REFERENCE_DIR") or DEFAULT_REFERENCE

KERNEL_STRINGS = {
    "REF_QUANT": "_KERNEL_NVFP4_FUSED",
    "REF_RMSNORM": "_KERNEL_RMSNORM_NVFP4_SMEM",
}


def extract_kernel_sources(float4utils_path: str) -> dict:
    with open(float4utils_path, "r", encoding="utf-8") as f:
        tree = ast.parse(f.read(), filename=float4utils_path)
    found = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1:
            tgt = node.targets[0]
            if isinstance(tgt, ast.Name) and isinstance(node.value, ast.Constant) \
                    and isinstance(node.value.value, str):
                found[tgt.id] = node.value.value
    out = {}
    for macro, name in KERNEL_STRINGS.items():
        if name not in found:
            raise RuntimeError(f"{name} not found in {float4utils_path}")
        out[macro] = found[name]
    return out


def build(reference: str = None, nvcc: str = "nvcc", quiet: bool = False) -> str:
    src = os.path.join(reference or reference_dir(), "float4utils.py")
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    sources = extract_kernel_sources(src)
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="nvfp4_ref_")
    try:
        objs = []
        for macro, code in sources.items():
            kfile = os.path.join(tmp, macro.lower() + ".cuh")
            with open(kfile, "w") as f:
                f.write(code)
            obj = os.path.join(tmp, macro.lower() + ".o")
            cmd = [nvcc, "-std=c++17", "-O3", "-Xcompiler", "-fPIC",
                   "-gencode", "arch=compute_100a,code=sm_100a",
                   f"-D{macro}", "-include", kfile, "-c",
                   os.path.join(HERE, "ref_launch.cu"), "-o", obj]
            if not quiet:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
            objs.append(obj)
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-o", OUT_SO] + objs + ["-lcudart"]
        if not quiet:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return OUT_SO


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=None, help="reference tree (default: $NVFP4_REFERENCE_DIR or the recipe default)")
    ap.add_argument("--nvcc", default="nvcc")
    args = ap.parse_args(argv)
    print(build(args.reference, args.nvcc))
    return 0


if __name__ == "__main__":
    sys.exit(main())
