"""Where a delta-rule prep tile spends its time: SM cycles per phase, from the profiling build.

    python -m fastdecisions_b200.build --phase-stamps     # libfdk_phases.so (stamps compiled in)
    python -m fastdecisions_b200.prepphases [--batch 7] [--lens 1536]

Runs the fused GDN call (conv + gates + chunked delta rule from the projection) on config-5 batch
``--batch`` and on ``--lens`` through libfdk_phases.so, and prints the mean cycles per tile of each
phase, measured by thread 0 of every tile from stamp to stamp (waits at the phase's closing barrier
included), so phases are comparable within one run.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json

import torch

from . import _lib, build, opbench
from .workloads import ModelConfig

PHASES = ("TMA + gates + q/k conv", "normalise (+ Qg/Kg out)", "MMA1 wait", "v conv", "L / Aqk", "solve level 0",
          "solve level 1", "solve level 2", "solve level 3", "TU / TW", "MMA2", "U^T / W^T out")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--batch", type=int, default=7)
    ap.add_argument("--lens", default="1536")
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args(argv)
    lib = _lib.load(build.PHASES_LIB)
    buf = (C.c_ulonglong * 16)()
    cases = ((f"config-5 batch {args.batch}", opbench.batch_lengths(args.batch)),
             (f"lens {args.lens}", [int(x) for x in args.lens.split(",")]))
    for label, lens in cases:
        fn, _ = opbench.make_case("gdn_fused", lens, ModelConfig())
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        lib.fdk_phase_stamps_read(buf)
        for _ in range(args.iters):
            fn()
        torch.cuda.synchronize()
        lib.fdk_phase_stamps_read(buf)
        n = max(1, buf[15])
        per = {PHASES[k - 1]: round(buf[k] / n) for k in range(1, 13)}
        print(json.dumps({"case": label, "tiles": int(buf[15]), "cycles_per_tile": round(sum(per.values())),
                          "phases": per}), flush=True)


if __name__ == "__main__":
    main()
