"""Failure detection on the GPU without a fault: a bounded device wait that
runs out reports NVFP4B200_ERR_TIMEOUT to the host, and the context stays
usable for the next launch."""
import pytest
import torch

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = 6


def test_bounded_wait_runs_out_and_reports(pkg):
    assert pkg.ops.device_error() == 0          # clears anything left by earlier tests
    stream = torch.cuda.current_stream().cuda_stream
    pkg._lib.call("nvfp4b200_wait_selftest", 2_000_000, stream)   # ~1 ms at B200 clocks
    torch.cuda.synchronize()
    assert pkg.ops.device_error() == ERR_TIMEOUT
    assert pkg.ops.device_error() == 0          # read-and-clear
    # the context still runs kernels correctly
    x = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    q, s = pkg.ops.quantize(x)
    q2, s2 = pkg.ops.quantize(x)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(s, s2)
    assert pkg.ops.device_error() == 0
