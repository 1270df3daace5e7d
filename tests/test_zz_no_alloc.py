"""GPU test of nvfp4b200_global_scale_noalloc, the global-scale entry point
for callers that cannot allocate device memory (pool- or arena-managed
memory, plugin hosts, code that must not trigger a cudaMalloc).  It is
called through the C ABI and must give the same global scale and amax as
nvfp4b200_global_scale (exact equality: both are a maximum) on two calls in
a row, the second smaller than the first, so stale scratch contents from the
first call would show.  Collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(lib, x):
    g = torch.empty(1, device=x.device, dtype=torch.float32)
    amax = torch.empty(1, device=x.device, dtype=torch.float32)
    rc = lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), x.numel(), g.data_ptr(), amax.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.nvfp4b200_status_string(rc)
    return g, amax


def test_global_scale_noalloc_matches_workspace_entry_point(pkg):
    lib = pkg._lib.load()
    gen = torch.Generator(device="cuda").manual_seed(5)
    big = (torch.randn(3 * (1 << 18) + 77, device="cuda", generator=gen) * 3).to(torch.bfloat16)
    big[12345] = float("nan")
    big[-3] = -1000.0                     # the maximum sits in the scalar tail of the last CTA
    small = (torch.randn(1000, device="cuda", generator=gen) * 0.5).to(torch.bfloat16)
    for x in (big, small):                # two calls in a row, largest amax first
        g, amax = _noalloc(lib, x)
        g_ref, amax_ref = pkg.ops.global_scale(x, with_amax=True)
        torch.cuda.synchronize()
        assert amax.item() == amax_ref.item()
        assert g.item() == g_ref.item()
        assert np.isfinite(g.item()) and g.item() > 0
    assert _noalloc(lib, big)[1].item() == 1000.0


def test_global_scale_noalloc_rejects_oversized_input(pkg):
    lib = pkg._lib.load()
    x = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    g = torch.empty(1, device="cuda", dtype=torch.float32)
    rc = lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), (1 << 30) + 1, g.data_ptr(), None, None)
    assert rc == 2 and "shape" in lib.nvfp4b200_status_string(rc).decode()
