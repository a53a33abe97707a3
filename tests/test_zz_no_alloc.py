"""The allocation-free delta-rule entry point, called through the C ABI.

``fdk_chunk_gated_delta_rule_fwd_noalloc`` serves callers that cannot allocate device memory (a
host binding only the C ABI with no device allocator of its own, or a request path that must not
call cudaMalloc / cudaFree because they synchronise the device): its scratch is a fixed 32 MiB
array inside the library.  This file checks that two calls in a row (different shapes, the second
reusing the scratch the first left behind) match the workspace entry point within the delta
rule's test tolerance, and that an oversized call is refused before any launch.  It is collected
last and builds all its inputs itself, so it runs the same alone or after the other tests.
"""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from fastdecisions_b200 import _lib, ops

MAX_ABS = 2e-2  # the delta-rule parity bound of tests/test_kernels_gpu.py


def _inputs(lens, H, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.randn(1, T, H, 128, generator=g).bfloat16().cuda()
    k = torch.randn(1, T, H, 128, generator=g).bfloat16().cuda()
    v = (0.5 * torch.randn(1, T, H, 128, generator=g)).bfloat16().cuda()
    gg = (-torch.rand(1, T, H, generator=g) * 2.0).cuda()
    beta = torch.rand(1, T, H, generator=g).bfloat16().cuda()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32).cuda()
    return q, k, v, gg, beta, cu


def _noalloc(q, k, v, gg, beta, cu, init=None):
    T, H = q.shape[1], q.shape[2]
    nseg = cu.numel() - 1
    out = torch.empty((1, T, H, 128), device="cuda", dtype=torch.bfloat16)
    final = torch.empty((nseg, H, 128, 128), device="cuda", dtype=torch.float32)
    _lib.call("fdk_chunk_gated_delta_rule_fwd_noalloc", q.data_ptr(), k.data_ptr(), H * 128, v.data_ptr(), H * 128,
              gg.data_ptr(), beta.data_ptr(), cu.data_ptr(), nseg, T, H, 128, 128, 128 ** -0.5,
              None if init is None else init.data_ptr(), out.data_ptr(), final.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return out, final


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    # the second call fills ~29.5 MiB of scratch; the third repeats the first, so every tile region
    # it reads still holds the larger call's stale tiles (nothing in the scratch may start at zero)
    cases = [([1, 64, 65, 170, 3], 16, 1), ([1536], 16, 2), ([1, 64, 65, 170, 3], 16, 1)]
    for lens, H, seed in cases:
        q, k, v, gg, beta, cu = _inputs(lens, H, seed)
        ref_o, ref_s = ops.chunk_gated_delta_rule(q, k, v, gg, beta, output_final_state=True, cu_seqlens=cu)
        got_o, got_s = _noalloc(q, k, v, gg, beta, cu)
        torch.cuda.synchronize()
        assert _lib.poll_device_error() == 0
        assert (got_o.float() - ref_o.float()).abs().max().item() < MAX_ABS
        assert (got_s - ref_s).abs().max().item() < MAX_ABS * max(1.0, ref_s.abs().max().item())
        assert torch.isfinite(got_o.float()).all()


def test_noalloc_matches_the_oracle():
    """The same call against the float32 CPU restatement of the chunked delta rule."""
    lens, H = [1, 64, 65, 170, 3], 4
    q, k, v, gg, beta, cu = _inputs(lens, H, 4)
    got_o, got_s = _noalloc(q, k, v, gg, beta, cu)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    ref_o, ref_s = O.chunk_gated_delta_rule(q.cpu(), k.cpu(), v.cpu(), gg.cpu(), beta.cpu().float(),
                                            output_final_state=True, cu_seqlens=cu.cpu())
    assert (got_o.float().cpu() - ref_o).abs().max().item() < MAX_ABS
    assert (got_s.cpu() - ref_s).abs().max().item() < 5e-2 * max(1.0, ref_s.abs().max().item())


def test_noalloc_rejects_calls_beyond_its_scratch():
    q, k, v, gg, beta, cu = _inputs([8], 16, 3)
    T = 4096  # needs ~77 MiB of scratch: refused before any launch
    with pytest.raises(ValueError, match="32 MiB"):
        _lib.call("fdk_chunk_gated_delta_rule_fwd_noalloc", q.data_ptr(), k.data_ptr(), 16 * 128, v.data_ptr(),
                  16 * 128, gg.data_ptr(), beta.data_ptr(), cu.data_ptr(), 1, T, 16, 128, 128, 128 ** -0.5, None,
                  q.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
