"""CPU tests of the C ABI: the library loads, exports every symbol the header
declares, and rejects invalid arguments before touching any device."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nvfp4_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(nvfp4b200_\w+)\s*\(", text, re.M)))


def test_header_declares_the_api():
    names = _declared()
    for must in ("nvfp4b200_quant_nvfp4", "nvfp4b200_rmsnorm_quant_nvfp4", "nvfp4b200_nvfp4_mm",
                 "nvfp4b200_nvfp4_mm_relu", "nvfp4b200_nvfp4_mm_relu_2", "nvfp4b200_gemm",
                 "nvfp4b200_quant_nvfp4_t", "nvfp4b200_global_scale"):
        assert must in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in include/nvfp4_b200.h but not exported"
    # and the Python binding covers the same set
    assert set(_declared()) == set(pkg._lib.exported_symbols())


def test_api_version_matches_header(pkg):
    lib = pkg._lib.load()
    m = re.search(r"#define NVFP4B200_API_VERSION (\d+)", open(HEADER).read())
    assert lib.nvfp4b200_api_version() == int(m.group(1))


def test_status_strings(pkg):
    assert pkg._lib.status_string(0) == "ok"
    assert "shape" in pkg._lib.status_string(2)
    assert "aligned" in pkg._lib.status_string(3)
    assert pkg._lib.status_string(99) == "unknown status"


FAKE = 1 << 20            # 16-byte aligned, never dereferenced: validation fails first
MIS = FAKE + 4


@pytest.mark.parametrize("call,expected", [
    (lambda L: L.nvfp4b200_quant_nvfp4(None, FAKE, FAKE, 4, 32, None, None), 1),
    (lambda L: L.nvfp4b200_quant_nvfp4(FAKE, FAKE, FAKE, 4, 24, None, None), 2),      # k % 16
    (lambda L: L.nvfp4b200_quant_nvfp4(FAKE, FAKE, FAKE, -1, 32, None, None), 2),
    (lambda L: L.nvfp4b200_quant_nvfp4(MIS, FAKE, FAKE, 4, 32, None, None), 3),
    (lambda L: L.nvfp4b200_quant_nvfp4_t(FAKE, None, None, FAKE, FAKE, 24, 16, None, None), 2),  # rows % 16
    (lambda L: L.nvfp4b200_rmsnorm_quant_nvfp4(FAKE, None, FAKE, FAKE, None, 4, 32, 1e-6, None, None), 1),
    (lambda L: L.nvfp4b200_nvfp4_mm(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, 8, 8, 48, None), 2),  # k % 32
    (lambda L: L.nvfp4b200_nvfp4_mm(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, 8, 12, 64, None), 2),  # n % 8
    (lambda L: L.nvfp4b200_nvfp4_mm(FAKE, MIS, FAKE, FAKE, None, None, FAKE, 8, 8, 64, None), 3),
    (lambda L: L.nvfp4b200_nvfp4_mm(None, FAKE, FAKE, FAKE, None, None, FAKE, 8, 8, 64, None), 1),
    (lambda L: L.nvfp4b200_gemm(FAKE, FAKE, FAKE, FAKE, None, None, None, None, FAKE, 0, 1, 0, 8, 8, 64, 8, None), 1),
    (lambda L: L.nvfp4b200_gemm(FAKE, FAKE, FAKE, FAKE, None, None, None, None, FAKE, 0, 0, 7, 8, 8, 64, 8, None), 1),
    (lambda L: L.nvfp4b200_swiglu_fwd(FAKE, FAKE, 4, 12, 0, None, None, None), 2),       # ff % 8
    (lambda L: L.nvfp4b200_swiglu_fwd(FAKE, FAKE, 4, 64, 128, None, None, None), 2),     # interleaved ff % 128
    (lambda L: L.nvfp4b200_swiglu_bwd(FAKE, FAKE, FAKE, 4, 64, 7, None, None, None), 1),  # bad interleave
    (lambda L: L.nvfp4b200_gemm_swiglu(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, None, None, None, 8, 384, 64,
                                       None), 2),                                         # n % 256
    (lambda L: L.nvfp4b200_gemm_swiglu(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, None, FAKE, None, 8, 512, 64,
                                       None), 1),                                         # ws without g_out
    (lambda L: L.nvfp4b200_gemm_dswiglu(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, FAKE, None, None, 8, 384, 64,
                                        None), 2),                                        # n % 256
    (lambda L: L.nvfp4b200_gemm_dswiglu(FAKE, FAKE, FAKE, FAKE, None, None, None, FAKE, None, None, 8, 512, 64,
                                        None), 1),                                        # no gate/up input
    (lambda L: L.nvfp4b200_gemm_dswiglu(FAKE, FAKE, FAKE, FAKE, None, None, MIS, FAKE, None, None, 8, 512, 64,
                                        None), 3),                                        # misaligned gate/up
    (lambda L: L.nvfp4b200_gemm_dswiglu(FAKE, FAKE, FAKE, FAKE, None, None, FAKE, FAKE, None, FAKE, 8, 512, 64,
                                        None), 1),                                        # g_out without ws
    (lambda L: L.nvfp4b200_wait_selftest(0, None), 1),
    (lambda L: L.nvfp4b200_mxfp4_mm(FAKE, FAKE, FAKE, FAKE, None, FAKE, 8, 8, 48, None), 2),        # k % 32
    (lambda L: L.nvfp4b200_mxfp4_mm(None, FAKE, FAKE, FAKE, None, FAKE, 8, 8, 64, None), 1),                                  # limit out of range
    (lambda L: L.nvfp4b200_adamw_step(FAKE, FAKE, 5, FAKE, FAKE, 8, 1e-3, .9, .95, 1e-8, 0., 1., 1., 1., None), 1),
    (lambda L: L.nvfp4b200_adamw_master_step(FAKE, None, FAKE, 0, FAKE, FAKE, 8, 1., .1, .95, .05, 1e-8, 1e-3, 1.,
                                             1., None, None), 1),                          # no master
    (lambda L: L.nvfp4b200_adamw_master_step(FAKE, MIS, FAKE, 0, FAKE, FAKE, 8, 1., .1, .95, .05, 1e-8, 1e-3, 1.,
                                             1., None, None), 3),                          # misaligned master
    (lambda L: L.nvfp4b200_adamw_master_step(FAKE, FAKE, FAKE, 0, FAKE, FAKE, -1, 1., .1, .95, .05, 1e-8, 1e-3,
                                             1., 1., None, None), 2),
    (lambda L: L.nvfp4b200_adamw_master_step(FAKE, FAKE, FAKE, 0, FAKE, FAKE, 8, 1., .1, .95, .05, 1e-8, 1e-3,
                                             1., 1., FAKE + 2, None), 3),                  # misaligned amax word
    (lambda L: L.nvfp4b200_global_scale_from_amax(None, FAKE, 4, None), 1),
    (lambda L: L.nvfp4b200_global_scale_from_amax(FAKE, FAKE, -1, None), 2),
])
def test_argument_validation_without_device(pkg, call, expected):
    assert call(pkg._lib.load()) == expected


def test_python_binding_fails_loudly_without_library(pkg, monkeypatch, tmp_path):
    monkeypatch.setattr(pkg._lib, "_lib", None)
    monkeypatch.setattr(pkg._lib, "lib_path", lambda: str(tmp_path / "missing.so"))
    with pytest.raises(pkg.NVFP4Error):
        pkg._lib.load()


def test_gn_kernels_ops_trace_with_fake_tensors(pkg):
    """The torch custom ops (NVFP4 and MXFP4 GEMMs) have fake implementations:
    under FakeTensorMode they give the bf16 [M, N] result without a device,
    which is what torch.compile tracing needs."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    from nvfp4_b200 import gn_kernels as g
    with FakeTensorMode():
        a = torch.empty(300, 256, dtype=torch.uint8, device="cuda")
        b = torch.empty(264, 256, dtype=torch.uint8, device="cuda")
        s = torch.empty(384, 16, dtype=torch.uint8, device="cuda")
        one = torch.empty((), dtype=torch.float32, device="cuda")
        outs = [g.cutlass_mxfp4_mm(a, b.mT, s, s)] + [op(a, b.mT, s, s, one) for op in
                                                      (g.cutlass_nvfp4_mm, g.cutlass_nvfp4_mm_relu,
                                                       g.cutlass_nvfp4_mm_relu_2)]
    for d in outs:
        assert tuple(d.shape) == (300, 264) and d.dtype == torch.bfloat16
