"""Per-op timing of the decision forward's device ops on one packed config-5 batch.

``python -m fastdecisions_b200.opbench --op delta_rule --batch 0`` builds batch ``--batch`` of the
config-5 plan (256 seeded requests, longest-first packing into 32768-token batches), runs one op on
layer-shaped synthetic inputs (seeded), and prints one JSON line per op: CUDA-event time per call,
the algorithmic work of one call and the fraction of the measured peak in MEASURED_PEAKS.json.
This is the small, self-contained case used for kernel profiles (one op, a few hundred MB on the
device); ``bench.py`` is the end-to-end measurement.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os

import numpy as np
import torch

from . import ops
from .engine import plan_batches
from .workloads import ModelConfig, config5_requests

CUBLAS = False  # --cublas: time torch.matmul (cuBLAS) for the gemm_* ops instead of the own GEMM
OPS = ("resadd_out", "resadd_down", "gemm_qkv_norm_rope", "gemm_gdn_in", "gemm_attn_qkv", "gemm_out", "gemm_down", "gemm_gate_up", "gemm_swiglu", "gdn_fused", "delta_rule", "gqa_attention", "packed_conv", "qk_norm_rope", "gated_rmsnorm", "residual_rmsnorm",
       "swiglu", "gdn_gates")


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm": float(d["hbm_gbs"]), "tensor": float(d["bf16_tflops"]), "source": "measured (burst)"}
    except (OSError, KeyError, ValueError):
        return {"hbm": 6650.0, "tensor": 1590.0, "source": "fallback"}


def batch_lengths(index: int, requests: int = 256, max_tokens: int = 32768) -> list:
    lens = [r.ids.size for r in config5_requests(requests)]
    plan = plan_batches(lens, max_tokens)
    return [lens[i] for i in plan[index]]


def make_case(op: str, lens: list, cfg: ModelConfig, seed: int = 0):
    """Returns (callable, ("tensor", flops) | ("hbm", bytes)) for one call of ``op``."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = "cuda"
    T = int(sum(lens))
    L = np.asarray(lens, dtype=np.int64)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(L)]), dtype=torch.int32, device=dev)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]).to(dev)

    def rn(*shape, scale=1.0):
        return (scale * torch.randn(*shape, generator=g, device=dev)).bfloat16()

    Hk, Hv, Dk, Dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, \
        cfg.linear_value_head_dim
    kd, vd = Hk * Dk, Hv * Dv
    C = 2 * kd + vd
    hq, hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    if op in ("resadd_out", "resadd_down"):  # the projection into the residual stream + the next norm
        H, I = cfg.hidden_size, cfg.intermediate_size
        k = vd if op == "resadd_out" else I
        a, w = rn(T, k), rn(H, k, scale=0.02)
        h = torch.randn(T, H, generator=g, device=dev)
        nw = rn(H, scale=0.02)
        flops = 2.0 * T * H * k
        if CUBLAS:  # cuBLAS GEMM (bf16 out), then the fused residual add + RMSNorm
            return (lambda: ops.residual_rmsnorm(torch.matmul(a, w.t()), h, nw, cfg.rms_norm_eps, residual_out=h)), \
                ("tensor", flops)
        return (lambda: ops.rmsnorm_stream(ops.gemm_residual_add(a, w, h), nw, cfg.rms_norm_eps)), ("tensor", flops)
    if op.startswith("gemm_"):  # own tcgen05 GEMM ("gemm_*") or, with --cublas, torch.matmul (cuBLAS)
        H, I = cfg.hidden_size, cfg.intermediate_size
        n, k = {"gemm_gdn_in": (C + vd + 2 * Hv, H), "gemm_attn_qkv": ((2 * hq + 2 * hkv) * D, H),
                "gemm_qkv_norm_rope": ((2 * hq + 2 * hkv) * D, H),
                "gemm_out": (H, vd), "gemm_down": (H, I), "gemm_gate_up": (2 * I, H), "gemm_swiglu": (2 * I, H)}[op]
        a, w = rn(T, k), rn(n, k, scale=0.02)
        flops = 2.0 * T * n * k
        if CUBLAS:
            if op == "gemm_swiglu":  # the unfused pair: cuBLAS GEMM then the SwiGLU kernel
                return (lambda: ops.swiglu(torch.matmul(a, w.t()), I)), ("tensor", flops)
            return (lambda: torch.matmul(a, w.t())), ("tensor", flops)
        if op == "gemm_qkv_norm_rope":  # the attention projection with q/k norm + RoPE
            qn, kn = rn(D, scale=0.02), rn(D, scale=0.02)
            rope = ops.rope_table(ops.rope_inv_freq(D, cfg.partial_rotary_factor, cfg.rope_theta).to(dev), int(L.max()))
            if CUBLAS:
                return (lambda: ops.attn_qk_norm_rope(torch.matmul(a, w.t()), qn, kn, pos, rope, hq, hkv, D,
                                                      cfg.rms_norm_eps)), ("tensor", flops)
            return (lambda: ops.gemm_qk_norm_rope(a, w, qn, kn, pos, rope, hq, hkv, D, cfg.rms_norm_eps)), ("tensor", flops)
        epi = ops.GEMM_SWIGLU if op == "gemm_swiglu" else ops.GEMM_PLAIN
        return (lambda: ops.gemm(a, w, epi)), ("tensor", flops)
    if op == "delta_rule":
        q, k, v = rn(1, T, Hk, Dk), rn(1, T, Hk, Dk), rn(1, T, Hv, Dv, scale=0.5)
        gg = -torch.rand(1, T, Hv, generator=g, device=dev) * 0.5
        beta = torch.rand(1, T, Hv, generator=g, device=dev).bfloat16()
        ws = torch.empty(ops.delta_rule_workspace_bytes(T, len(lens), Hv), dtype=torch.uint8, device=dev)
        fn = lambda: ops.chunk_gated_delta_rule(q, k, v, gg, beta, cu_seqlens=cu, workspace=ws)  # noqa: E731
        return fn, ("tensor", Hv * float(np.ceil(L / 64).sum()) * 11.7e6)
    if op == "gdn_fused":  # conv + gates + delta rule from the in-projection, as the engine runs them
        width = C + vd + 2 * Hv
        proj = rn(T, width + (-width) % 8)
        conv = rn(C, cfg.linear_conv_kernel_dim, scale=0.3)
        A_log = torch.log(torch.empty(Hv, device=dev).uniform_(1, 16))
        dt = torch.ones(Hv, device=dev)
        ws = torch.empty(ops.delta_rule_workspace_bytes(T, len(lens), Hv), dtype=torch.uint8, device=dev)
        fn = lambda: ops.gdn_fused_delta_rule(proj, conv, A_log, dt, Hv, C + vd + Hv, C + vd, cu, workspace=ws)  # noqa: E731
        return fn, ("tensor", Hv * float(np.ceil(L / 64).sum()) * 11.7e6)
    if op == "gqa_attention":
        q, k, v = rn(T, hq, D), rn(T, hkv, D), rn(T, hkv, D)
        fn = lambda: ops.gqa_attention_varlen_(q, k, v, cu, int(L.max()))  # noqa: E731
        return fn, ("tensor", 2.0 * hq * D * float((L * (L + 1)).sum()))
    if op == "packed_conv":
        x = rn(1, T, C)
        w = rn(C, cfg.linear_conv_kernel_dim, scale=0.3)
        fn = lambda: ops.packed_conv_qkv(x, w, kd, vd, Dk, cu)  # noqa: E731
        return fn, ("hbm", T * C * 2.0 * 2)
    if op == "qk_norm_rope":
        proj = rn(T, (2 * hq + 2 * hkv) * D)
        qn, kn = rn(D, scale=0.02), rn(D, scale=0.02)
        rope = ops.rope_table(ops.rope_inv_freq(D, cfg.partial_rotary_factor, cfg.rope_theta).to(dev), int(L.max()))
        fn = lambda: ops.attn_qk_norm_rope(proj, qn, kn, pos, rope, hq, hkv, D, cfg.rms_norm_eps)  # noqa: E731
        return fn, ("hbm", T * (hq + hkv) * D * 2.0 * 2)
    if op == "gated_rmsnorm":
        o, z = rn(T, Hv, Dv), rn(T, vd)
        w = rn(Dv, scale=0.1) + 1.0
        fn = lambda: ops.gated_rmsnorm(o, z, w, cfg.rms_norm_eps)  # noqa: E731
        return fn, ("hbm", T * vd * 6.0)
    if op == "residual_rmsnorm":
        H = cfg.hidden_size
        x = rn(T, H)
        h = torch.randn(T, H, generator=g, device=dev)
        w = rn(H, scale=0.02)
        fn = lambda: ops.residual_rmsnorm(x, h, w, cfg.rms_norm_eps, residual_out=h)  # noqa: E731
        return fn, ("hbm", T * H * (2 + 4 + 4 + 2.0))
    if op == "swiglu":
        I = cfg.intermediate_size
        gu = rn(T, 2 * I)
        fn = lambda: ops.swiglu(gu, I)  # noqa: E731
        return fn, ("hbm", T * I * 6.0)
    if op == "gdn_gates":
        a, b = rn(T, Hv), rn(T, Hv)
        A_log = torch.log(torch.empty(Hv, device=dev).uniform_(1, 16))
        dt = torch.ones(Hv, device=dev)
        fn = lambda: ops.gdn_gates(a, b, A_log, dt)  # noqa: E731
        return fn, ("hbm", T * Hv * 10.0)
    raise ValueError(f"unknown op {op!r}")


def time_op(fn, iters: int, warmup: int) -> float:
    """Mean milliseconds per call (CUDA events on the current stream, L2 flushed between calls)."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        total += e0.elapsed_time(e1)
    return total / iters


def time_rotating(fns, passes: int, warmup: int) -> float:
    """Mean milliseconds per call over back-to-back calls that cycle through independent buffer
    sets (their total far above L2, so every call streams from HBM).  One pass over the sets is
    captured in a CUDA graph (warm-up on a side stream first) and replayed ``passes`` times between
    two CUDA events: host dispatch is out of the measurement, as in the engine's graph replays."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            for f in fns:
                f()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in fns:
            f()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(passes):
        graph.replay()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (passes * len(fns))
    del graph
    return ms


def forward_cfg4(replays: int, **engine_opts) -> None:
    """Config 4 (batch 1, 1536 tokens) through the engine's CUDA graph: ``replays`` replays inside
    an NVTX range named ``replay`` (profilers select the graph's kernels by it), p50 printed."""
    import statistics
    from .engine import DecisionEngine, pack
    from .workloads import config4_request, synthetic_weights
    cfg = ModelConfig()
    split = engine_opts.pop("residual_split_k", 0)
    eng = DecisionEngine(cfg, synthetic_weights(cfg), "cuda", **engine_opts)
    eng.residual_split_k = split
    b = pack([config4_request()])
    key = eng.capture(b.tokens, 1, b.max_seqlen)
    d, _ = eng.to_device(b)
    eng.replay(key, *d)
    torch.cuda.synchronize()
    times = []
    torch.cuda.nvtx.range_push("replay")
    for _ in range(replays):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.replay(key)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"op": "forward_cfg4 (graph replay)", "tokens": b.tokens, "replays": replays, "opts": engine_opts,
                      "residual_split_k": split,
                      "p50_ms": round(statistics.median(times), 4), "min_ms": round(min(times), 4)}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--op", default="all", help="one of %s, or all" % ", ".join(OPS))
    ap.add_argument("--batch", type=int, default=0, help="index into the config-5 batch plan")
    ap.add_argument("--lens", default=None,
                    help="comma-separated request lengths to pack instead of a config-5 batch (e.g. 4096)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--rotate-mb", type=int, default=0,
                    help="HBM-bound ops: time CUDA-graph replays of back-to-back calls over enough "
                         "independent buffer sets to move this many MB per pass (e.g. 1024, far above the "
                         "126 MB L2) instead of single calls with an L2 flush between them")
    ap.add_argument("--attn", default=None,
                    help="attention geometry hq,hkv,head_dim (e.g. 8,2,256: the reference kernel's own shape)")
    ap.add_argument("--cublas", action="store_true", help="gemm_* ops: time torch.matmul (cuBLAS) instead")
    ap.add_argument("--replays", type=int, default=30, help="--op forward_cfg4: graph replays")
    ap.add_argument("--split-k", type=int, default=0,
                    help="--op forward_cfg4: 1 = out / down projections as k-split partial GEMMs (default: cuBLAS)")
    args = ap.parse_args(argv)
    if args.op == "forward_cfg4":
        forward_cfg4(args.replays, split_residual_gemm=args.split_k != 0, residual_split_k=0)
        return
    global CUBLAS
    CUBLAS = args.cublas
    cfg = ModelConfig()
    if args.attn:
        hq, hkv, d = (int(x) for x in args.attn.split(","))
        cfg = dataclasses.replace(cfg, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=d)
    lens = [int(x) for x in args.lens.split(",")] if args.lens else batch_lengths(args.batch)
    peaks = _peaks()
    for op in (OPS if args.op == "all" else (args.op,)):
        fn, (bound, work) = make_case(op, lens, cfg)
        timing = "single calls, L2 flushed between them"
        if args.rotate_mb and bound == "hbm":
            sets = max(2, math.ceil(args.rotate_mb * 2.0**20 / work))
            fns = [fn] + [make_case(op, lens, cfg, seed=i)[0] for i in range(1, sets)]
            ms = time_rotating(fns, args.iters, args.warmup)
            timing = f"CUDA-graph replays, back-to-back over {sets} buffer sets ({sets * work / 2**20:.0f} MB a pass)"
        else:
            ms = time_op(fn, args.iters, args.warmup)
        achieved = work / (ms * 1e-3) / (1e12 if bound == "tensor" else 1e9)
        print(json.dumps({"op": op + (" (cuBLAS)" if CUBLAS and op.startswith(("gemm_", "resadd_")) else ""), "batch": "lens" if args.lens else args.batch, "tokens": int(sum(lens)),
                          "attn": [cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim],
                          "segments": len(lens),
                          "max_len": int(max(lens)), "us": round(ms * 1e3, 2), "bound": bound,
                          "achieved": round(achieved, 1), "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
                          "frac": round(achieved / peaks[bound], 4), "peak_source": peaks["source"],
                          "timing": timing}), flush=True)


if __name__ == "__main__":
    main()
