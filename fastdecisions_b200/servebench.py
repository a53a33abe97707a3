"""Serving-path timing: decision requests scored one call at a time, eager vs bucketed CUDA graphs.

    python -m fastdecisions_b200.servebench [--requests 64] [--per-call 1]

The first ``--requests`` requests of the config-5 mix (synthetic config-4 model) go through
``DecisionEngine.score`` ``--per-call`` at a time, once with eager launches and once with
``graphs=True`` (after one warm-up pass that captures the buckets, then ``seal()``; batches of more
than ``GRAPH_MAX_REQUESTS`` requests launch eagerly either way).  Reports
wall-clock requests/s (host token ids to host probabilities, the synchronising D2H included) and
the device time of the same calls, so the host-dispatch share is visible.  One JSON line per mode.
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from . import workloads as W
from .engine import DecisionEngine


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--per-call", type=int, default=1)
    ap.add_argument("--max-len", type=int, default=8192)
    args = ap.parse_args(argv)
    cfg = W.ModelConfig()
    eng = DecisionEngine(cfg, W.synthetic_weights(cfg), "cuda")
    reqs = [r for r in W.config5_requests(256) if r.ids.size <= args.max_len][:args.requests]
    calls = [reqs[i:i + args.per_call] for i in range(0, len(reqs), args.per_call)]
    for graphs in (False, True):
        for c in calls:  # warm-up (captures every bucket the calls need)
            eng.score(c, graphs=graphs)
        if graphs:
            eng.seal()
        torch.cuda.synchronize()
        dev_ms = 0.0
        t0 = time.perf_counter()
        for c in calls:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            eng.score(c, graphs=graphs)
            e1.record()
            e1.synchronize()
            dev_ms += e0.elapsed_time(e1)
        wall = time.perf_counter() - t0
        print(json.dumps({"mode": "cuda graphs (bucketed)" if graphs else "eager launches",
                          "requests": len(reqs), "per_call": args.per_call,
                          "tokens": int(sum(r.ids.size for r in reqs)), "requests_per_s": round(len(reqs) / wall, 2),
                          "wall_ms_per_call": round(1000 * wall / len(calls), 3),
                          "stream_ms_per_call": round(dev_ms / len(calls), 3),
                          "graph_captures": eng.stats["graph_captures"]}), flush=True)


if __name__ == "__main__":
    main()
