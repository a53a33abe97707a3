"""Failure detection on the GPU without a fault: a bounded device wait that nothing satisfies
runs out, the kernel reports it through the device error word and returns, and the context
stays usable (the same path every mbarrier wait in the attention and delta-rule kernels takes)."""
import time

import pytest
import torch

from fastdecisions_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    _lib.load()
    assert _lib.poll_device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    _lib.call("fdk_selftest_bounded_wait", 2_000_000, stream)  # about a millisecond of SM clock
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert _lib.poll_device_error() == 4   # bit 2: the self-test's wait gave up
    assert _lib.poll_device_error() == 0   # read and cleared


def test_context_usable_after_a_wait_ran_out():
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("fdk_selftest_bounded_wait", 1_000_000, stream)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 4
    g = torch.Generator(device="cuda").manual_seed(5)
    gu = torch.randn(37, 2 * 256, generator=g, device="cuda").bfloat16()
    out = ops.swiglu(gu, 256)
    ref = (torch.nn.functional.silu(gu[:, :256].float()) * gu[:, 256:].float()).bfloat16()
    torch.testing.assert_close(out.float(), ref.float(), rtol=0.008, atol=0.002)
    assert _lib.poll_device_error() == 0
