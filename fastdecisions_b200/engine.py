"""Decision engine: the whole one-pass decision forward on one B200, over the C ABI.

Mirrors what the reference's ``Engine`` does around ``core(input_ids)`` (src/decider/engine.py:
77-181): embed -> 24 decoder layers -> final norm at the decision slots -> restricted logits ->
softmax, with the projections and MLP as cuBLAS GEMMs and every other op a kernel of
``libfdk.so``.  Differences that make it B200-native:

* requests are packed end to end (varlen ``cu_seqlens``) instead of right-padded to (B, T)
  buckets: the conv, delta rule and attention kernels restart at every segment boundary, so one
  forward serves any mix of request lengths without padding work;
* per-layer projections are fused into one GEMM each (GDN: qkv|z|b|a, attention: q|k|v, MLP:
  gate|up), the residual add is fused into the following RMSNorm, the attention output gate into
  the attention epilogue, and the last residual add into the slot readout (only slot rows);
* fixed shapes (e.g. batch-1 decisions of one length) are captured once into a CUDA graph and
  replayed, like the reference's bucketed graphs (engine.py:123-149).
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Optional, Sequence

import numpy as np
import torch

from . import ops
from .workloads import LETTER_IDS, ModelConfig, Request, letter_weight


_NULL = contextlib.nullcontext()


@dataclass
class PackedBatch:
    """Host-side packed varlen batch (int32 arrays) of ``len(slots)`` requests."""
    ids: np.ndarray
    cu_seqlens: np.ndarray
    positions: np.ndarray
    slots: np.ndarray        # absolute token row of each request's decision slot
    nopts: np.ndarray
    max_seqlen: int

    @property
    def tokens(self) -> int:
        return int(self.ids.size)

    @property
    def num_segments(self) -> int:
        return int(self.slots.size)


MAX_REQUEST_TOKENS = 32768
FUSED_SWIGLU_MIN_TOKENS = 4096  # packed batches at least this large use the SwiGLU-fused GEMM
FUSED_QKV_MIN_TOKENS = 4096     # ... and the attention projection with q/k norm + RoPE fused
FUSED_RESIDUAL_MIN_TOKENS = 4096  # ... and the out / down projections adding into the residual stream

# Bucketed CUDA graphs for small packed batches (EngineV2-style, src/decider/engine_v2.py:79-175):
# a batch is padded up to the smallest bucket of each kind and replayed from a graph captured once
# for that bucket.  Small batches are host-bound when launched eagerly (~250 launches a forward).
GRAPH_TOKEN_BUCKETS = (128, 160, 192, 256, 320, 384, 512, 640, 768, 1024, 1280, 1536, 1792, 2048, 2560, 3072, 3584,
                       4096, 5120, 6144, 7168, 8192)  # steps of at most 1.25x: padding stays under 25%
GRAPH_SEGMENT_BUCKETS = (1, 2, 4, 8, 16, 32, 64)
GRAPH_MAX_REQUESTS = 1  # score(graphs=True) graphs batches of this many requests at most


def _bucket(n: int, buckets) -> Optional[int]:
    for b in buckets:
        if n <= b:
            return b
    return None


def pack(requests: Sequence[Request]) -> PackedBatch:
    lens = np.array([r.ids.size for r in requests], dtype=np.int64)
    if (lens < 1).any():
        raise ValueError("every request needs at least one token")
    if (lens > MAX_REQUEST_TOKENS).any():
        raise ValueError(f"requests are limited to {MAX_REQUEST_TOKENS} tokens")
    cu = np.zeros(len(requests) + 1, dtype=np.int32)
    np.cumsum(lens, out=cu[1:])
    ids = np.concatenate([r.ids for r in requests]).astype(np.int32, copy=False)
    pos = (np.arange(ids.size, dtype=np.int64) - np.repeat(cu[:-1].astype(np.int64), lens)).astype(np.int32)
    slots = np.array([c + r.slot for c, r in zip(cu[:-1], requests)], dtype=np.int32)
    if any(not (0 <= r.slot < r.ids.size) for r in requests):
        raise ValueError("decision slot outside its request")
    nopts = np.array([r.nopts for r in requests], dtype=np.int32)
    return PackedBatch(ids, cu, pos, slots, nopts, int(lens.max()))


def plan_batches(lengths: Sequence[int], max_tokens: int) -> list:
    """Greedy packing of requests (longest first) into batches of at most ``max_tokens`` tokens
    (a request longer than the budget gets a batch of its own)."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    batches, cur, cur_t = [], [], 0
    for i in order:
        if cur and cur_t + lengths[i] > max_tokens:
            batches.append(cur)
            cur, cur_t = [], 0
        cur.append(i)
        cur_t += lengths[i]
    if cur:
        batches.append(cur)
    return batches


class DecisionEngine:
    def __init__(self, cfg: ModelConfig, weights: dict, device="cuda", letter_ids=LETTER_IDS,
                 temperature: float = 1.0, residual_fp32: bool = True, fuse_gdn_prologue: bool = True,
                 fused_swiglu_gemm: bool = True, fused_qkv_gemm: bool = False, fused_residual_gemm: bool = True,
                 split_residual_gemm: bool = False):
        """``residual_fp32`` keeps the residual stream in float32 (the sum of the layer outputs is
        never rounded); with False it is stored in bf16 like the eager bf16 model.
        ``fuse_gdn_prologue`` runs the Gated-DeltaNet conv, gates and delta rule as one call on the
        projection (same results as the three separate ops, without their HBM round trips).
        ``fused_swiglu_gemm`` runs the MLP's gate/up projection of packed batches of at least
        ``FUSED_SWIGLU_MIN_TOKENS`` tokens as the library's tcgen05 GEMM with the SwiGLU epilogue
        (the [T, 2 I] projection is never stored; silu(g) * u is formed from the fp32
        accumulators): measured 1.5% more requests/s on config 5.  Smaller batches (batch-1
        decisions) use cuBLAS and the separate SwiGLU kernel, measured faster there.
        ``fused_qkv_gemm`` likewise runs the attention projection of batches of at least
        ``FUSED_QKV_MIN_TOKENS`` tokens as the tcgen05 GEMM whose epilogue applies the q / k RMSNorm
        and the partial RoPE (no separate q / k norm kernel, no bf16 rounding of q / k before it).
        Off by default: measured 10% slower than cuBLAS + the separate kernel at 32k tokens (the
        GEMM's mainloop is ~7% behind cuBLAS at N = 5120).
        ``fused_residual_gemm`` (with the float32 residual stream) runs the out-projections and the
        MLP down-projection as the tcgen05 GEMM that adds its fp32 accumulators into the stream
        (TMA reduce-add; K split to fill the SMs at batch-1 sizes), followed by the RMSNorm of the
        stream alone, for packed batches of at least ``FUSED_RESIDUAL_MIN_TOKENS``: the layer
        outputs are never rounded to bf16 and the norm moves 6 bytes an element instead of 12.
        Measured at 32k tokens: out-projection + norm 423 -> 294 us, down-projection + norm
        741 -> 633 us, +1.1% requests/s on config 5; at batch 1 (1536 tokens) cuBLAS and the
        fused residual-add RMSNorm stay faster (5.21 vs 5.46 ms).
        ``split_residual_gemm`` (float32 stream) runs those projections of smaller batches, where
        the output tiles leave SMs idle, as K-split GEMMs writing fp32 partial planes that the next
        RMSNorm adds into the stream in a fixed order (reproducible; no bf16 rounding of the layer
        output).  Off by default: measured slower than cuBLAS + the residual-add RMSNorm in the
        config-4 graph (5.77 vs 5.30 ms)."""
        self.cfg = cfg
        self.fuse_gdn_prologue = bool(fuse_gdn_prologue)
        self.fused_swiglu_gemm = bool(fused_swiglu_gemm)
        self.fused_qkv_gemm = bool(fused_qkv_gemm)
        self.residual_fp32 = bool(residual_fp32)
        self.fused_residual_gemm = bool(fused_residual_gemm) and self.residual_fp32
        self.residual_split_k = 0  # k-slices of the residual-add GEMMs (0: the library's choice)
        self.split_residual_gemm = bool(split_residual_gemm) and self.residual_fp32
        self.dev = torch.device(device)
        self.temperature = float(temperature)
        dev = self.dev
        w = weights
        bf = torch.bfloat16

        def put(t, dtype=bf):
            return t.to(device=dev, dtype=dtype).contiguous()

        self.embed = put(w["embed_tokens.weight"])
        self.final_norm = put(w["norm.weight"])
        self.letters = put(letter_weight(w, letter_ids))
        self.inv_freq = ops.rope_inv_freq(cfg.head_dim, cfg.partial_rotary_factor, cfg.rope_theta, dev)
        self.max_positions = 32768  # requests up to the model's 32k-token context
        self.rope = ops.rope_table(self.inv_freq, self.max_positions)
        self.layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"layers.{i}."
            L = SimpleNamespace(kind=kind)
            L.in_norm = put(w[p + "input_layernorm.weight"])
            L.post_norm = put(w[p + "post_attention_layernorm.weight"])
            L.w_gu = put(torch.cat([w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]]))
            L.w_gu_il = None
            if self.fused_swiglu_gemm and cfg.intermediate_size % 128 == 0:
                L.w_gu_il = put(ops.interleave_gate_up(w[p + "mlp.gate_proj.weight"], w[p + "mlp.up_proj.weight"]))
            L.w_down = put(w[p + "mlp.down_proj.weight"])
            if kind == "linear_attention":
                la = p + "linear_attn."
                L.w_in = put(torch.cat([w[la + "in_proj_qkv.weight"], w[la + "in_proj_z.weight"],
                                        w[la + "in_proj_b.weight"], w[la + "in_proj_a.weight"]]))
                cw = w[la + "conv1d.weight"]
                L.conv = put(cw.reshape(cw.shape[0], cw.shape[-1]))
                L.A_log = put(w[la + "A_log"], torch.float32)
                L.dt_bias = put(w[la + "dt_bias"], torch.float32)
                L.gnorm = put(w[la + "norm.weight"])
                L.w_out = put(w[la + "out_proj.weight"])
            else:
                sa = p + "self_attn."
                L.w_qkv = put(torch.cat([w[sa + "q_proj.weight"], w[sa + "k_proj.weight"], w[sa + "v_proj.weight"]]))
                L.q_norm = put(w[sa + "q_norm.weight"])
                L.k_norm = put(w[sa + "k_norm.weight"])
                L.w_o = put(w[sa + "o_proj.weight"])
            self.layers.append(L)
        self._ws: dict = {}
        self._tk: dict = {}
        self._parts: dict = {}
        self._graphs = {}
        self._graph_pool = None
        self._sealed = False
        self._pinned_slots: list = []   # per stream: [pinned int32 host buffer, event after its H2D]
        self._streams: list = []
        self.stats = dict(forwards=0, graph_captures=0, graph_replays=0)
        self.kernel_timer = None  # optional callable(name) -> context manager, set by the bench

    # ------------------------------------------------------------------ workspace
    def _workspace(self, tokens: int, segments: int) -> torch.Tensor:
        """Delta-rule scratch of the current stream (one buffer per stream, so batches in flight on
        different streams never share it)."""
        need = ops.delta_rule_workspace_bytes(tokens, segments, self.cfg.linear_num_value_heads)
        key = torch.cuda.current_stream(self.dev).cuda_stream
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, device=self.dev, dtype=torch.uint8)
            self._ws[key] = ws
        return ws

    def _tickets(self, tokens: int) -> torch.Tensor:
        """Slice tickets of the residual-add GEMMs of the current stream (zero between calls)."""
        need = 4 * ((tokens + 127) // 128) * ((self.cfg.hidden_size + 255) // 256) + 2
        key = torch.cuda.current_stream(self.dev).cuda_stream
        tk = self._tk.get(key)
        if tk is None or tk.numel() < need:
            tk = torch.zeros(need, device=self.dev, dtype=torch.int32)
            self._tk[key] = tk
        return tk

    def _partials(self, tokens: int, slices: int) -> torch.Tensor:
        """float32 k-slice planes of the split projection GEMMs of the current stream."""
        need = slices * tokens * self.cfg.hidden_size
        key = torch.cuda.current_stream(self.dev).cuda_stream
        buf = self._parts.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(max(need, 4 * tokens * self.cfg.hidden_size), device=self.dev, dtype=torch.float32)
            self._parts[key] = buf
        return buf

    def reserve(self, tokens: int, segments: int):
        """Pre-size the delta-rule scratch and the GEMM tickets (call before graph capture)."""
        self._workspace(tokens, segments)
        self._tickets(tokens)

    # ------------------------------------------------------------------ forward
    def _timed(self, name):
        """Optional per-op CUDA-event timing (the benchmark sets ``kernel_timer``)."""
        if self.kernel_timer is None:
            return _NULL
        return self.kernel_timer(name)

    def _mixer_mlp(self, i: int, x: torch.Tensor, h: torch.Tensor, cu: torch.Tensor, pos: torch.Tensor,
                   max_seqlen: int, ws: torch.Tensor):
        """Layer ``i`` given its normalised input ``x`` (bf16) and the residual stream ``h``:
        token mixer, residual add fused into post_attention_layernorm, SwiGLU MLP.  Updates ``h`` in
        place to ``h + mixer`` and returns the MLP output (the caller adds it)."""
        c = self.cfg
        L = self.layers[i]
        T = x.shape[0]
        Hk, Hv = c.linear_num_key_heads, c.linear_num_value_heads
        Dk, Dv = c.linear_key_head_dim, c.linear_value_head_dim
        kd, vd = Hk * Dk, Hv * Dv
        C = 2 * kd + vd
        hq, hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        tm = self._timed
        if L.kind == "linear_attention":
            with tm("gemm"):
                proj = torch.matmul(x, L.w_in.t())                                       # [T, C + vd + 2 Hv]
            if self.fuse_gdn_prologue and Hk == Hv and Dk == Dv == 128:
                # conv + SiLU, gates and the chunked delta rule in one call on the projection
                with tm("delta_rule"):
                    o = ops.gdn_fused_delta_rule(proj, L.conv, L.A_log, L.dt_bias, Hv, C + vd + Hv, C + vd, cu,
                                                 workspace=ws)
            else:
                with tm("packed_conv"):
                    q, k, v = ops.packed_conv_qkv(proj[:, :C].unsqueeze(0), L.conv, kd, vd, Dk, cu)
                with tm("gdn_gates"):
                    g, beta = ops.gdn_gates(proj[:, C + vd + Hv:C + vd + 2 * Hv], proj[:, C + vd:C + vd + Hv],
                                            L.A_log, L.dt_bias)
                with tm("delta_rule"):
                    o, _ = ops.chunk_gated_delta_rule(q, k, v, g.unsqueeze(0), beta.unsqueeze(0), cu_seqlens=cu,
                                                      workspace=ws)
            with tm("gated_rmsnorm"):
                on = ops.gated_rmsnorm(o.view(T, Hv, Dv), proj[:, C:C + vd], L.gnorm, c.rms_norm_eps)
            mix_in, w_mix = on, L.w_out
        else:
            if (self.fused_qkv_gemm and T >= FUSED_QKV_MIN_TOKENS and D in (128, 256)
                    and self.rope.shape[1] == D // 4):
                with tm("gemm_qk_norm_rope"):  # projection + q/k norm + RoPE (own tcgen05 GEMM)
                    proj, q, k = ops.gemm_qk_norm_rope(x, L.w_qkv, L.q_norm, L.k_norm, pos, self.rope, hq, hkv, D,
                                                       c.rms_norm_eps)
            else:
                with tm("gemm"):
                    proj = torch.matmul(x, L.w_qkv.t())                                  # [T, (2 hq + 2 hkv) D]
                with tm("qk_norm_rope"):
                    q, k = ops.attn_qk_norm_rope(proj, L.q_norm, L.k_norm, pos, self.rope, hq, hkv, D, c.rms_norm_eps)
            v = proj[:, (2 * hq + hkv) * D:].view(T, hkv, D)
            with tm("gqa_attention"):
                o = ops.gqa_attention_varlen_(q, k, v, cu, max_seqlen, gate=proj[:, D:], gate_interleaved=True)
            mix_in, w_mix = o.view(T, hq * D), L.w_o
        fused_res = self.fused_residual_gemm and T >= FUSED_RESIDUAL_MIN_TOKENS
        H = c.hidden_size
        split_mix = 0 if fused_res or not self.split_residual_gemm else ops.split_slices(T, H, mix_in.shape[1])
        split_down = 0 if fused_res or not self.split_residual_gemm else ops.split_slices(T, H, c.intermediate_size)
        if split_mix > 1:  # k-split partial planes, added into the stream in order by the norm
            with tm("gemm_partials"):
                parts = ops.gemm_partials(mix_in, w_mix, self._partials(T, split_mix), split_mix)
            with tm("residual_rmsnorm"):
                x2 = ops.rmsnorm_add_partials(parts, split_mix, h, L.post_norm, c.rms_norm_eps)
        elif fused_res:  # out-projection adds into the fp32 stream; then its norm alone
            with tm("gemm_residual_add"):
                ops.gemm_residual_add(mix_in, w_mix, h, split_k=self.residual_split_k, tickets=self._tickets(T))
            with tm("residual_rmsnorm"):
                x2 = ops.rmsnorm_stream(h, L.post_norm, c.rms_norm_eps)
        else:
            with tm("gemm"):
                mix = torch.matmul(mix_in, w_mix.t())
            with tm("residual_rmsnorm"):
                x2, _ = ops.residual_rmsnorm(mix, h, L.post_norm, c.rms_norm_eps, residual_out=h)
        if L.w_gu_il is not None and T >= FUSED_SWIGLU_MIN_TOKENS:  # gate/up GEMM + SwiGLU epilogue (own kernel)
            with tm("gemm_swiglu"):
                act = ops.gemm(x2, L.w_gu_il, ops.GEMM_SWIGLU)
        else:
            with tm("gemm"):
                gu = torch.matmul(x2, L.w_gu.t())
            with tm("swiglu"):
                act = ops.swiglu(gu, c.intermediate_size)
        if split_down > 1:  # partial planes; the caller's norm (or the readout's add) sums them in
            with tm("gemm_partials"):
                ops.gemm_partials(act, L.w_down, self._partials(T, split_down), split_down)
            return ("partials", split_down)
        if fused_res:  # the MLP output goes straight into the stream: nothing returned
            with tm("gemm_residual_add"):
                ops.gemm_residual_add(act, L.w_down, h, split_k=self.residual_split_k, tickets=self._tickets(T))
            return None
        with tm("gemm"):
            return torch.matmul(act, L.w_down.t())

    @torch.no_grad()
    def forward_device(self, ids: torch.Tensor, cu: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor,
                       nopts: torch.Tensor, max_seqlen: int, probs: Optional[torch.Tensor] = None,
                       logits: Optional[torch.Tensor] = None, trace: Optional[list] = None):
        """All inputs int32 on the engine's device.  Returns ``(probs, logits)`` float32 ``[S, K]``.
        ``trace`` (a list, diagnostics only) receives the residual stream after every layer."""
        c = self.cfg
        ws = self._workspace(ids.numel(), cu.numel() - 1)
        self.stats["forwards"] += 1
        tm = self._timed
        with tm("embed"):
            e = ops.embed(ids, self.embed)
        with tm("residual_rmsnorm"):
            x, h = ops.residual_rmsnorm(e, None, self.layers[0].in_norm, c.rms_norm_eps,
                                        residual_fp32=self.residual_fp32)
        down = None
        for i in range(len(self.layers)):
            down = self._mixer_mlp(i, x, h, cu, pos, max_seqlen, ws)
            if isinstance(down, tuple):  # k-split partial planes of the down-projection
                parts = self._partials(h.shape[0], down[1])
                with tm("residual_rmsnorm"):
                    x = ops.rmsnorm_add_partials(parts, down[1], h, self.layers[i + 1].in_norm if i + 1 < len(
                        self.layers) else None, c.rms_norm_eps)
                down = None
                if i + 1 < len(self.layers):
                    if trace is not None:
                        trace.append(h.clone())
                    continue
            if i + 1 < len(self.layers):
                with tm("residual_rmsnorm"):
                    if down is None:  # already added into h by the down-projection
                        x = ops.rmsnorm_stream(h, self.layers[i + 1].in_norm, c.rms_norm_eps)
                    else:
                        x, _ = ops.residual_rmsnorm(down, h, self.layers[i + 1].in_norm, c.rms_norm_eps,
                                                    residual_out=h)
                if trace is not None:
                    trace.append(h.clone())
            elif trace is not None:
                last = h.float() + (0.0 if down is None else down.float())
                trace.append(last if self.residual_fp32 else last.bfloat16())
        with tm("slot_readout"):
            return ops.slot_readout(h, slots, nopts, self.final_norm, self.letters, c.rms_norm_eps, self.temperature,
                                    probs=probs, logits=logits, delta=down)

    @torch.no_grad()
    def layer_output(self, i: int, h_in: torch.Tensor, cu: torch.Tensor, pos: torch.Tensor, max_seqlen: int):
        """Residual stream after layer ``i`` alone, given the stream ``h_in [T, H]`` before it
        (parity tests feed the oracle's own stream here, so each layer is checked in isolation)."""
        c = self.cfg
        h = h_in.to(self.dev, torch.float32 if self.residual_fp32 else torch.bfloat16).contiguous().clone()
        zero = torch.zeros(h.shape, device=self.dev, dtype=torch.bfloat16)
        x, _ = ops.residual_rmsnorm(zero, h, self.layers[i].in_norm, c.rms_norm_eps, residual_out=h)
        down = self._mixer_mlp(i, x, h, cu, pos, max_seqlen, self._workspace(h.shape[0], cu.numel() - 1))
        if isinstance(down, tuple):
            ops.rmsnorm_add_partials(self._partials(h.shape[0], down[1]), down[1], h, None)
            down = None
        return h.float() + (0.0 if down is None else down.float())

    # ------------------------------------------------------------------ host API
    def to_device(self, batch: PackedBatch, pinned: Optional[torch.Tensor] = None):
        """One pinned host buffer -> one H2D copy; returns device views (ids, cu, pos, slots, nopts)."""
        parts = [batch.ids, batch.cu_seqlens, batch.positions, batch.slots, batch.nopts]
        n = sum(p.size for p in parts)
        if pinned is None or pinned.numel() < n:
            pinned = torch.empty(n, dtype=torch.int32, pin_memory=True)
        off = 0
        host = pinned.numpy()
        for p in parts:
            host[off:off + p.size] = p
            off += p.size
        dev = pinned[:n].to(self.dev, non_blocking=True)
        out, off = [], 0
        for p in parts:
            out.append(dev[off:off + p.size])
            off += p.size
        return out, n * 4

    def streams(self, n: int) -> list:
        """``n`` CUDA streams of this engine (created once); batches are spread over them."""
        while len(self._streams) < n:
            self._streams.append(torch.cuda.Stream(self.dev))
        return self._streams[:n]

    @torch.no_grad()
    def forward_batches(self, dev_batches: Sequence, max_seqlens: Sequence[int], probs: Sequence[torch.Tensor],
                        streams: int = 2):
        """Forward of several packed device batches, batch ``k`` on stream ``k % streams``: kernels
        of one batch fill the SMs another batch leaves idle (the delta-rule recurrence runs one chain
        per SM; short kernels have tails).  ``probs[k]`` receives batch ``k``'s answer rows.  The
        current stream waits for all of them on return."""
        main = torch.cuda.current_stream(self.dev)
        sts = self.streams(max(1, streams))
        for st in sts:
            st.wait_stream(main)
        for k, ((ids, cu, pos, slots, nopts), ms, pr) in enumerate(zip(dev_batches, max_seqlens, probs)):
            with torch.cuda.stream(sts[k % len(sts)]):
                self.forward_device(ids, cu, pos, slots, nopts, ms, probs=pr)
        for st in sts:
            main.wait_stream(st)

    @torch.no_grad()
    def score(self, requests: Sequence[Request], max_tokens: int = 32768, streams: int = 2,
              graphs: bool = False) -> np.ndarray:
        """Public API: decision probabilities ``[N, K]`` (numpy, request order) for host-side requests.

        Requests are packed longest-first into batches of at most ``max_tokens`` tokens
        (``plan_batches``); each batch is packed on the host while the previous ones run, copied in
        one pinned H2D transfer, run on stream ``k % streams``, and its answer rows come back in one
        D2H copy into pinned host memory.  With ``graphs`` every batch of at most
        ``GRAPH_MAX_REQUESTS`` requests that fits a graph bucket is replayed from its bucket's CUDA
        graph on one stream: host dispatch of ~250 launches is what bounds one request.  Measured
        (config-5 requests, one per call): 169 -> 203 requests/s; four per call the eager launches
        are faster (275 vs 252: the padding costs more than the dispatch it saves)."""
        if len(requests) == 0:
            return np.zeros((0, self.letters.shape[0]), dtype=np.float32)
        plan = plan_batches([r.ids.size for r in requests], max_tokens)
        K = self.letters.shape[0]
        sts = self.streams(1 if graphs else max(1, streams))  # graph replays share static buffers
        main = torch.cuda.current_stream(self.dev)
        for st in sts:
            st.wait_stream(main)
        host_out = torch.empty((len(requests), K), dtype=torch.float32, pin_memory=True)
        while len(self._pinned_slots) < len(sts):
            self._pinned_slots.append([None, torch.cuda.Event()])
        row = 0
        for k, b in enumerate(plan):
            batch = pack([requests[j] for j in b])  # host work overlaps the batches already queued
            slot = self._pinned_slots[k % len(sts)]
            n = batch.tokens * 2 + 3 * batch.num_segments + 1
            slot[1].synchronize()  # the previous H2D from this pinned buffer has finished
            if slot[0] is None or slot[0].numel() < n:
                slot[0] = torch.empty(max(n, 1 << 16), dtype=torch.int32, pin_memory=True)
            st = sts[k % len(sts)]
            with torch.cuda.stream(st):
                (ids, cu, pos, slots, nopts), _ = self.to_device(batch, slot[0])
                slot[1].record(st)
                graphed = graphs and batch.num_segments <= GRAPH_MAX_REQUESTS
                probs = self.forward_graphed(batch, (ids, cu, pos, slots, nopts)) if graphed else None
                if probs is None:
                    probs, _ = self.forward_device(ids, cu, pos, slots, nopts, batch.max_seqlen)
                host_out[row:row + len(b)].copy_(probs, non_blocking=True)
            row += len(b)
        for st in sts:
            main.wait_stream(st)
        main.synchronize()
        order = np.concatenate([np.asarray(b, dtype=np.int64) for b in plan])
        result = np.empty((len(requests), K), dtype=np.float32)
        result[order] = host_out.numpy()
        return result

    # ------------------------------------------------------------------ CUDA graphs
    @torch.no_grad()
    def capture(self, tokens: int, segments: int, max_seqlen: int):
        """Capture the forward for a fixed (tokens, segments, max_seqlen) shape; returns a key.
        All captures share one memory pool (replays of different graphs must not overlap: they run
        on one stream)."""
        key = (tokens, segments, max_seqlen)
        if key in self._graphs:
            return key
        if self._sealed:
            raise RuntimeError("DecisionEngine.capture: the engine is sealed (no new CUDA graphs)")
        dev = self.dev
        st = dict(ids=torch.zeros(tokens, dtype=torch.int32, device=dev),
                  cu=torch.tensor([0] * segments + [tokens], dtype=torch.int32, device=dev),
                  pos=torch.zeros(tokens, dtype=torch.int32, device=dev),
                  slots=torch.zeros(segments, dtype=torch.int32, device=dev),
                  nopts=torch.ones(segments, dtype=torch.int32, device=dev))
        self.reserve(tokens, segments)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                self.forward_device(st["ids"], st["cu"], st["pos"], st["slots"], st["nopts"], max_seqlen)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(graph, pool=self._graph_pool):
            probs, logits = self.forward_device(st["ids"], st["cu"], st["pos"], st["slots"], st["nopts"], max_seqlen)
        st.update(graph=graph, probs=probs, logits=logits)
        self._graphs[key] = st
        self.stats["graph_captures"] += 1
        return key

    def replay(self, key, ids=None, cu=None, pos=None, slots=None, nopts=None):
        """Copy new inputs (device tensors of the captured shapes) and replay; returns probs view."""
        st = self._graphs[key]
        for name, t in (("ids", ids), ("cu", cu), ("pos", pos), ("slots", slots), ("nopts", nopts)):
            if t is not None:
                st[name].copy_(t, non_blocking=True)
        st["graph"].replay()
        self.stats["graph_replays"] += 1
        return st["probs"]

    # ------------------------------------------------------------------ bucketed graphs
    def graph_key(self, batch: PackedBatch):
        """Bucket of a packed batch: (tokens, segments, max_seqlen) rounded up, or None when the
        batch is larger than the largest bucket.  Padding tokens form one extra segment."""
        tb = _bucket(batch.tokens, GRAPH_TOKEN_BUCKETS)
        if tb is None:
            return None
        pad = tb - batch.tokens
        sb = _bucket(batch.num_segments + (1 if pad else 0), GRAPH_SEGMENT_BUCKETS)
        if sb is None:
            return None
        need = max(batch.max_seqlen, pad, 1)
        mb = 128
        while mb < need:
            mb *= 2
        return tb, sb, min(mb, tb)

    def warm_buckets(self, keys):
        """Capture the given bucket keys ahead of serving (EngineV2's grid capture)."""
        for k in keys:
            self.capture(*k)

    def seal(self):
        """No new captures from now on: batches whose bucket was not captured run eagerly."""
        self._sealed = True

    @torch.no_grad()
    def forward_graphed(self, batch: PackedBatch, dev_inputs=None) -> Optional[torch.Tensor]:
        """Answer probabilities ``[S, K]`` (device) of a host batch through its bucket's CUDA graph,
        capturing the bucket on first use unless sealed; None when the batch has no usable bucket.
        ``dev_inputs``: the batch's device tensors (ids, cu, pos, slots, nopts) if already copied."""
        key = self.graph_key(batch)
        if key is None or (key not in self._graphs and self._sealed):
            return None
        if key not in self._graphs:
            self.capture(*key)
        tb, sb, _ = key
        st = self._graphs[key]
        T, S = batch.tokens, batch.num_segments
        ids, cu, pos, slots, nopts = dev_inputs if dev_inputs is not None else self.to_device(batch)[0]
        st["ids"][:T].copy_(ids, non_blocking=True)
        st["ids"][T:].zero_()
        st["pos"][:T].copy_(pos, non_blocking=True)
        if tb > T:  # the padding segment: positions 0, 1, ...
            st["pos"][T:].copy_(self._arange(tb - T))
        st["cu"][:S + 1].copy_(cu, non_blocking=True)
        st["cu"][S + 1:].fill_(tb)
        st["slots"][:S].copy_(slots, non_blocking=True)
        st["slots"][S:].zero_()
        st["nopts"][:S].copy_(nopts, non_blocking=True)
        st["nopts"][S:].fill_(1)
        st["graph"].replay()
        self.stats["graph_replays"] += 1
        return st["probs"][:S]

    def _arange(self, n: int) -> torch.Tensor:
        a = getattr(self, "_arange_buf", None)
        if a is None or a.numel() < n:
            a = torch.arange(max(n, 8192), dtype=torch.int32, device=self.dev)
            self._arange_buf = a
        return a[:n]
