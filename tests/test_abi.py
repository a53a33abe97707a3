"""C-ABI checks that need no GPU: the library loads, exports every declared symbol, and the
Python signatures cover the header.  No compute entry point is called here."""
import ctypes
import os

import pytest

from fastdecisions_b200 import _lib


def test_library_built():
    assert os.path.exists(_lib.LIB_PATH), "run `python -m fastdecisions_b200.build` first"


def test_every_header_symbol_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = _lib.header_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_header():
    assert set(_lib.header_functions()) == set(_lib.SIGNATURES)


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.fdk_version().decode().startswith("fastdecisions-b200")
    assert isinstance(lib.fdk_get_last_error_string(), bytes)


def test_workspace_size_host_only():
    lib = _lib.load()
    n = lib.fdk_chunk_gated_delta_rule_workspace_size(1536, 1, 16, 128, 128)
    # (1536/64 + 1) chunks x 16 heads x (4 x 16 KiB + 8 KiB + 16 B) + table
    assert n >= 25 * 16 * (4 * 16384 + 8192)
    assert lib.fdk_chunk_gated_delta_rule_workspace_size(1536, 1, 16, 64, 128) == 0


def test_ops_refuse_cpu_tensors():
    import torch
    from fastdecisions_b200 import ops
    x = torch.zeros(4, 2048, dtype=torch.bfloat16)
    w = torch.zeros(2048, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.residual_rmsnorm(x, x, w)
    with pytest.raises(ValueError):
        ops.packed_conv_qkv(torch.zeros(1, 8, 6144, dtype=torch.bfloat16), torch.zeros(6144, 4, dtype=torch.bfloat16))


def test_selftest_budget_validated_before_launch():
    # argument checks run on the host before any CUDA call, so this needs no GPU
    for bad in (0, -5, 5_000_000_000):
        with pytest.raises(ValueError, match="budget_cycles"):
            _lib.call("fdk_selftest_bounded_wait", bad, None)
