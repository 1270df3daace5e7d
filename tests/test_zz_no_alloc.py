"""GPU test of nvfp4b200_global_scale_noalloc, the global-scale entry point
for callers that cannot allocate device memory (pool- or arena-managed
memory, plugin hosts, code that must not trigger a cudaMalloc).  It is
called through the C ABI and must give the same global scale and amax as
nvfp4b200_global_scale (exact equality: both are a maximum) on two calls in
a row, the second smaller than the first, so stale scratch contents from the
first call would show; on an input large enough that the grid exceeds 256
CTAs with the maximum in a late CTA; and with amax_out NULL.  Repeated calls
must leave the device's free memory and torch's allocation unchanged.
Collected last on purpose."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(lib, x, with_amax=True):
    g = torch.empty(1, device=x.device, dtype=torch.float32)
    amax = torch.empty(1, device=x.device, dtype=torch.float32) if with_amax else None
    rc = lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), x.numel(), g.data_ptr(),
                                            None if amax is None else amax.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.nvfp4b200_status_string(rc)
    return g, amax


def test_global_scale_noalloc_matches_workspace_entry_point(pkg):
    lib = pkg._lib.load()
    gen = torch.Generator(device="cuda").manual_seed(5)
    big = (torch.randn(3 * (1 << 18) + 77, device="cuda", generator=gen) * 3).to(torch.bfloat16)
    big[12345] = float("nan")
    big[-3] = -1000.0                     # the maximum sits in the scalar tail
    small = (torch.randn(1000, device="cuda", generator=gen) * 0.5).to(torch.bfloat16)
    for x in (big, small):                # two calls in a row, largest amax first
        g, amax = _noalloc(lib, x)
        g_ref, amax_ref = pkg.ops.global_scale(x, with_amax=True)
        torch.cuda.synchronize()
        assert amax.item() == amax_ref.item()
        assert g.item() == g_ref.item()
        assert np.isfinite(g.item()) and g.item() > 0
    assert _noalloc(lib, big)[1].item() == 1000.0


def test_global_scale_noalloc_many_ctas_and_no_amax_out(pkg):
    lib = pkg._lib.load()
    n = 300 * (1 << 18) + 5               # ~157 MB: the grid is capped at 8 CTAs per SM, well above 256
    gen = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(n, device="cuda", generator=gen).to(torch.bfloat16)
    x[n - 9] = 77.0                       # last vector: read by a late CTA of the grid stride
    g, amax = _noalloc(lib, x)
    g_ref, amax_ref = pkg.ops.global_scale(x, with_amax=True)
    torch.cuda.synchronize()
    assert amax.item() == amax_ref.item() == 77.0
    assert g.item() == g_ref.item()
    g2, none = _noalloc(lib, x, with_amax=False)
    torch.cuda.synchronize()
    assert none is None and g2.item() == g_ref.item()


def test_global_scale_noalloc_allocates_nothing(pkg):
    lib = pkg._lib.load()
    x = torch.randn(1 << 20, device="cuda").to(torch.bfloat16)
    g = torch.empty(1, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), x.numel(), g.data_ptr(), None, stream) == 0
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(5):
        assert lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), x.numel(), g.data_ptr(), None, stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_global_scale_noalloc_rejects_oversized_input(pkg):
    lib = pkg._lib.load()
    x = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    g = torch.empty(1, device="cuda", dtype=torch.float32)
    rc = lib.nvfp4b200_global_scale_noalloc(x.data_ptr(), (1 << 30) + 1, g.data_ptr(), None, None)
    assert rc == 2 and "shape" in lib.nvfp4b200_status_string(rc).decode()
