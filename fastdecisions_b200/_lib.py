"""ctypes binding of ``libfdk.so`` (the C ABI in ``include/fdk.h``).

The library is loaded from the package directory (built in-tree by ``fastdecisions_b200.build``).
There is no fallback: if the shared library is missing every op raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libfdk.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "fdk.h")

FDK_OK = 0
FDK_ERR_INVALID_ARGUMENT = 1
FDK_ERR_ALIGNMENT = 2
FDK_ERR_UNSUPPORTED = 3
FDK_ERR_LAUNCH = 4
FDK_ERR_DEVICE = 5

vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); must cover every function declared in include/fdk.h
SIGNATURES = {
    "fdk_version": (C.c_char_p, []),
    "fdk_get_last_error_string": (C.c_char_p, []),
    "fdk_residual_rmsnorm": (i32, [vp, i64, vp, i64, i32, vp, i32, vp, i64, vp, i64, i64, i64, f32, f32, vp]),
    "fdk_packed_conv_silu": (i32, [vp, i64, vp, i64, i64, i64, i32, vp, i64, i64, i64, vp, vp, vp, vp]),
    "fdk_gdn_gates": (i32, [vp, i64, vp, i64, vp, vp, vp, vp, i64, i64, vp]),
    "fdk_chunk_gated_delta_rule_workspace_size": (sz, [i64, i64, i64, i64, i64]),
    "fdk_chunk_gated_delta_rule_fwd": (i32, [vp, vp, i64, vp, i64, vp, vp, vp, i64, i64, i64, i64, i64, f32,
                                             vp, vp, vp, vp, sz, vp]),
    "fdk_chunk_gated_delta_rule_fwd_noalloc": (i32, [vp, vp, i64, vp, i64, vp, vp, vp, i64, i64, i64, i64, i64,
                                                     f32, vp, vp, vp, vp]),
    "fdk_gdn_fused_delta_rule_fwd": (i32, [vp, i64, vp, i32, i64, i64, i64, i64, vp, vp, vp, i64, i64, i64, f32, vp,
                                           vp, vp, vp, sz, vp]),
    "fdk_gated_rmsnorm": (i32, [vp, vp, i64, vp, i32, vp, i64, i64, i64, f32, vp]),
    "fdk_attn_qk_norm_rope": (i32, [vp, i64, vp, vp, i32, vp, vp, i64, i32, vp, vp, i64, i64, i64, i64, f32, vp]),
    "fdk_gqa_fwd": (i32, [vp, i64, vp, i64, vp, i64, vp, i64, i64, i64, i64, i64, i64, f32, vp, i64, i32, vp, vp]),
    "fdk_poll_device_error": (i32, [C.POINTER(C.c_int)]),
    "fdk_selftest_bounded_wait": (i32, [i64, vp]),
    "fdk_embed": (i32, [vp, vp, i64, i64, vp, i64, vp]),
    "fdk_gemm_bf16": (i32, [vp, i64, vp, i64, vp, i64, i64, i64, i64, i32, vp]),
    "fdk_gemm_bf16_residual_add": (i32, [vp, i64, vp, i64, vp, i64, i64, i64, i64, i32, vp, vp]),
    "fdk_gemm_bf16_partials": (i32, [vp, i64, vp, i64, vp, i64, i64, i64, i32, vp]),
    "fdk_rmsnorm_add_partials": (i32, [vp, i32, vp, i64, vp, i32, vp, i64, i64, i64, f32, f32, vp]),
    "fdk_gemm_bf16_qk_norm_rope": (i32, [vp, i64, vp, i64, vp, i64, i64, i64, i64, i64, i64, i64, vp, vp, vp, vp, i64,
                                         i32, f32, vp, vp, vp]),
    "fdk_swiglu": (i32, [vp, i64, vp, i64, i64, vp]),
    "fdk_slot_readout": (i32, [vp, i32, vp, i64, vp, vp, i64, vp, i32, vp, i64, f32, f32, vp, vp, vp]),
}

_lib = None


class FdkError(RuntimeError):
    pass


def header_functions() -> list[str]:
    """Names of every function declared in include/fdk.h."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"\b(fdk_[a-z0-9_]+)\s*\(", txt)))


def load(path: str = LIB_PATH):
    """Load libfdk.so (once) and attach the C signatures.  Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FdkError(f"{path} is missing: build it with `python -m fastdecisions_b200.build` "
                       "(there is no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def poll_device_error() -> int:
    """Device-side error word (non-zero when a bounded in-kernel wait ran out); clears it."""
    code = C.c_int(0)
    call("fdk_poll_device_error", C.byref(code))
    return code.value


# kernels each compute entry point launches (used to count device launches in a timed region)
KERNELS_PER_CALL = {"fdk_chunk_gated_delta_rule_fwd": 3, "fdk_chunk_gated_delta_rule_fwd_noalloc": 3,
                    "fdk_gdn_fused_delta_rule_fwd": 3}
call_counts: dict = {}


def launches_since(snapshot: dict) -> int:
    """Kernel launches issued through the C ABI since ``snapshot`` (a copy of ``call_counts``)."""
    n = 0
    for name, c in call_counts.items():
        if name.startswith("fdk_") and name not in ("fdk_poll_device_error",):
            n += (c - snapshot.get(name, 0)) * KERNELS_PER_CALL.get(name, 1)
    return n


def call(name: str, *args):
    """Call an fdk_* entry point and map a non-zero status to an exception."""
    lib = load()
    call_counts[name] = call_counts.get(name, 0) + 1
    st = getattr(lib, name)(*args)
    if st != FDK_OK:
        msg = lib.fdk_get_last_error_string().decode()
        if st in (FDK_ERR_INVALID_ARGUMENT, FDK_ERR_ALIGNMENT, FDK_ERR_UNSUPPORTED):
            raise ValueError(f"{name}: {msg}")
        raise FdkError(f"{name} failed (status {st}): {msg}")
    return st
