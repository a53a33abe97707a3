"""Build ``libfdk.so`` (the C-ABI CUDA library) in-tree for sm_100a with nvcc.

``python -m fastdecisions_b200.build`` compiles every ``csrc/*.cu`` to an object file under
``fastdecisions_b200/_build/`` (in parallel, skipped when up to date) and links
``fastdecisions_b200/libfdk.so``.  No GPU is needed: nvcc cross-compiles for sm_100a.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libfdk.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _flags(extra=()):
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I", os.path.join(ROOT, "include"), "-I", CSRC]
    f += list(extra)
    return f


def _compile(src: str, obj: str, verbose_ptxas: bool) -> str:
    deps = [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "fdk.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps) and not verbose_ptxas:
        return ""
    cmd = [nvcc(), "-c", src, "-o", obj] + _flags(["-Xptxas", "-v"] if verbose_ptxas else [])
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose_ptxas else ""


def build(verbose_ptxas: bool = False, jobs: int | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        logs = list(ex.map(lambda so: _compile(so[0], so[1], verbose_ptxas), zip(srcs, objs)))
    if verbose_ptxas:
        for s, log in zip(srcs, logs):
            print(f"== {os.path.basename(s)}\n{log}")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-Xcompiler", "-fPIC", "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


PHASES_LIB = os.path.join(PKG, "libfdk_phases.so")


def build_phase_stamps() -> str:
    """A profiling copy of the library, libfdk_phases.so: the delta-rule prep compiled with
    FDK_PHASE_STAMPS (per-phase SM-cycle counters, read with fdk_phase_stamps_read); every other
    object is the normal build's."""
    build()
    obj = os.path.join(BUILD, "delta_rule_phases.o")
    _compile_with(os.path.join(CSRC, "delta_rule.cu"), obj, ["-DFDK_PHASE_STAMPS"])
    objs = [o for o in sorted(glob.glob(os.path.join(BUILD, "*.o"))) if os.path.basename(o) not in
            ("delta_rule.o", "delta_rule_phases.o")] + [obj]
    r = subprocess.run([nvcc(), "-shared", "-o", PHASES_LIB] + objs + ARCH + ["-Xcompiler", "-fPIC", "-lcudart"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return PHASES_LIB


def _compile_with(src: str, obj: str, extra) -> None:
    r = subprocess.run([nvcc(), "-c", src, "-o", obj] + _flags(extra), capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    if "--phase-stamps" in sys.argv:
        print(build_phase_stamps())
    else:
        print(build(verbose_ptxas="-v" in sys.argv))
