"""Whole-forward CPU restatement of the hybrid decision model (TEST INFRASTRUCTURE ONLY).

Restates ``Qwen3_5TextModel.forward`` ([tf]:1227-1290) over ``Qwen3_5DecoderLayer`` ([tf]:744-783)
with the linear-attention mixer ``Qwen3_5GatedDeltaNet.forward`` ([tf]:422-533), the gated GQA
mixer ``Qwen3_5Attention.forward`` ([tf]:647-692) and the SwiGLU MLP ([tf]:706-708), followed by
the reference's slot readout (model.py:18-27, engine.py:48-56).  Weights are a dict keyed by the
transformers ``state_dict`` names, so the same dict loads into a real ``Qwen3_5TextModel`` for the
golden fixtures.  Packed varlen input (``cu_seqlens``) runs every segment as an independent
request, which is what right-padded batch rows are for the causal model (engine.py:1-6).
"""
from __future__ import annotations

import torch

from . import ops


def _lin(x, w):
    return x @ ops._f(w).t()


def layer_forward(cfg: dict, weights: dict, i: int, h, positions, cu_seqlens=None, round_dtype=None,
                  act_dtype=None):
    """One decoder layer ([tf]:744-783): returns the residual stream after layer ``i`` given the
    stream ``h [T, H]`` before it (float32).  Rounding options as in ``forward_hidden``."""
    T = h.shape[0]
    eps = cfg["rms_norm_eps"]
    kind = cfg["layer_types"][i]

    def rnd(x):
        return x if round_dtype is None else x.to(round_dtype).float()

    def a(x):
        return x if act_dtype is None else x.to(act_dtype).float()

    def lin(x, w):
        return a(_lin(x, w))

    p = f"layers.{i}."
    x = a(ops.rmsnorm_offset(h, weights[p + "input_layernorm.weight"], eps))   # [tf]:765
    if kind == "linear_attention":
        la = p + "linear_attn."
        Hk, Hv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        Dk, Dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
        mixed = lin(x, weights[la + "in_proj_qkv.weight"])                     # [tf]:442
        z = lin(x, weights[la + "in_proj_z.weight"]).reshape(T, Hv, Dv)          # [tf]:445-446
        b = lin(x, weights[la + "in_proj_b.weight"])                            # [tf]:448
        a_ = lin(x, weights[la + "in_proj_a.weight"])                           # [tf]:449
        q, k, v = (a(t) for t in ops.packed_conv_silu(mixed[None], weights[la + "conv1d.weight"], cu_seqlens,
                                                      key_dim=Hk * Dk, value_dim=Hv * Dv, head_dim=Dk))
        g, beta = ops.gdn_gates(a_, b, weights[la + "A_log"], weights[la + "dt_bias"])
        beta = a(beta)
        if Hv // Hk > 1:                                                       # [tf]:494-496
            q = q.repeat_interleave(Hv // Hk, dim=2)
            k = k.repeat_interleave(Hv // Hk, dim=2)
        o, _ = ops.chunk_gated_delta_rule(q, k, v, g[None], beta[None], cu_seqlens=cu_seqlens)
        o = a(ops.gated_rmsnorm(a(o[0]), z, weights[la + "norm.weight"], eps))    # [tf]:526-529
        out = lin(o.reshape(T, Hv * Dv), weights[la + "out_proj.weight"])        # [tf]:532
    else:
        sa = p + "self_attn."
        Hq, Hkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
        qg = lin(x, weights[sa + "q_proj.weight"]).reshape(T, Hq, 2 * D)          # [tf]:657-659
        q, gate = qg[..., :D], qg[..., D:].reshape(T, Hq * D)
        q = ops.rmsnorm_offset(q, weights[sa + "q_norm.weight"], eps)             # [tf]:662
        k = ops.rmsnorm_offset(lin(x, weights[sa + "k_proj.weight"]).reshape(T, Hkv, D),
                               weights[sa + "k_norm.weight"], eps)               # [tf]:663
        v = lin(x, weights[sa + "v_proj.weight"]).reshape(T, Hkv, D)             # [tf]:664
        cos, sin = ops.rope_cos_sin(positions, D, cfg["partial_rotary_factor"], cfg["rope_theta"])
        q = a(ops.apply_partial_rope(q, cos, sin))                               # [tf]:666-667
        k = a(ops.apply_partial_rope(k, cos, sin))
        o = ops.gqa_attention_varlen(q, k, v, cu_seqlens, scale=D ** -0.5)       # [tf]:676-685
        o = a(o.reshape(T, Hq * D) * torch.sigmoid(gate))                        # [tf]:687-689
        out = lin(o, weights[sa + "o_proj.weight"])                               # [tf]:691
    h = rnd(h + out)                                                           # [tf]:775
    x = a(ops.rmsnorm_offset(h, weights[p + "post_attention_layernorm.weight"], eps))  # [tf]:779
    m = p + "mlp."
    act = a(ops.swiglu(lin(x, weights[m + "gate_proj.weight"]), lin(x, weights[m + "up_proj.weight"])))
    h = rnd(h + lin(act, weights[m + "down_proj.weight"]))                     # [tf]:780-781
    return h


def positions_of(T, cu_seqlens=None):
    """Position ids restart at 0 for every packed request."""
    return torch.cat([torch.arange(s1 - s0) for s0, s1 in ops._segments(T, cu_seqlens)])


def forward_hidden(cfg: dict, weights: dict, ids, cu_seqlens=None, round_dtype=None, trace=None,
                   act_dtype=None):
    """Returns the float32 hidden state after the last decoder layer (before the final norm).

    ``cfg`` keys: hidden_size, layer_types, num_attention_heads, num_key_value_heads, head_dim,
    linear_num_key_heads, linear_num_value_heads, linear_key_head_dim, linear_value_head_dim,
    rms_norm_eps, partial_rotary_factor, rope_theta.  ``round_dtype`` (e.g. bfloat16) rounds the
    residual stream after every add, as the eager bf16 model stores it.  ``trace`` (a list)
    receives a copy of the residual stream after every decoder layer.  ``act_dtype`` (e.g.
    bfloat16) additionally rounds every stored activation (norm outputs, GEMM outputs, conv, delta
    rule, gated norm, q/k after RoPE, attention output, SwiGLU) to that dtype: a CPU emulation of
    the storage points of a bf16 GPU forward, used to separate kernel error from bf16 storage.
    """
    ids = torch.as_tensor(ids).reshape(-1)
    T = ids.numel()
    positions = positions_of(T, cu_seqlens)
    h = ops._f(weights["embed_tokens.weight"])[ids]                       # [tf]:1243

    def rnd(x):
        return x if round_dtype is None else x.to(round_dtype).float()

    h = rnd(h)
    for i in range(len(cfg["layer_types"])):
        h = layer_forward(cfg, weights, i, h, positions, cu_seqlens, round_dtype, act_dtype)
        if trace is not None:
            trace.append(h.clone())
    return h


def decide(cfg, weights, letter_weight, ids, cu_seqlens, slots, nopts, temperature=1.0):
    """Hidden states -> per-request answer probabilities ``[N, K]`` (engine.py:48-56)."""
    h = forward_hidden(cfg, weights, ids, cu_seqlens)
    return ops.slot_readout(h, weights["norm.weight"], letter_weight, slots, nopts,
                            cfg["rms_norm_eps"], temperature)
