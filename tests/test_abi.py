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


def test_plain_c_host_compiles_links_and_calls(tmp_path):
    """A C program (no C++, no CUDA headers) includes include/fdk.h, links libfdk.so and calls the
    host-only entry points and one argument-checking failure path -- what a cgo / JNI host does."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "host.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "fdk.h"
int main(void) {
  const char* v = fdk_version();
  size_t ws = fdk_chunk_gated_delta_rule_workspace_size(1536, 1, 16, 128, 128);
  int st = fdk_selftest_bounded_wait(0, NULL);  /* rejected on the host, before any CUDA call */
  printf("%s|%zu|%d|%s\n", v, ws, st, fdk_get_last_error_string());
  return (strncmp(v, "fastdecisions-b200", 18) == 0 && ws > 0 && st == FDK_ERR_INVALID_ARGUMENT) ? 0 : 1;
}
''')
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    libdir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "host"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", inc, str(src), "-o", str(exe), "-L", libdir,
                    "-l:libfdk.so", f"-Wl,-rpath,{libdir}"], check=True, capture_output=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    version, ws, st, msg = r.stdout.strip().split("|")
    assert int(ws) == _lib.load().fdk_chunk_gated_delta_rule_workspace_size(1536, 1, 16, 128, 128)
    assert int(st) == _lib.FDK_ERR_INVALID_ARGUMENT and "budget_cycles" in msg
