"""Per-op CPU restatements of the forward hot path (TEST INFRASTRUCTURE ONLY, see package header).

Every function takes tensors of any floating dtype, computes in float32 on the CPU (float64 where
the reference's own check does) and returns float32 results; callers compare them with the CUDA
outputs at the tolerance stated in each test.  ``[tf]:N`` cites line N of transformers 5.5.0
``models/qwen3_5/modeling_qwen3_5.py``; other citations are files of the FastDecisions reference.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

F32 = torch.float32


def _f(x: torch.Tensor, dtype=F32) -> torch.Tensor:
    return x.detach().to("cpu", dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``x * rsqrt(sum(x^2) + eps)`` over the last dim ([tf]:228-231)."""
    x = _f(x)
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def rmsnorm_offset(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen3.5 RMSNorm: ``x * rsqrt(mean(x^2) + eps) * (1 + w)`` in float32 ([tf]:711-728)."""
    x = _f(x)
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + _f(weight))


def residual_rmsnorm(x, residual, weight, eps: float = 1e-6, sum_dtype=None):
    """Decoder residual add followed by the post-attention RMSNorm.

    ``s = residual + x`` ([tf]:775) then ``rmsnorm_offset(s)`` ([tf]:779, norm at :711-728).  When
    ``sum_dtype`` is given (e.g. bfloat16) the sum is rounded to it first, as the eager bf16 model
    does before the norm reads it.  Returns ``(normed, summed)`` in float32.  The reference's
    persistent kernel (persistent_residual_rms_kernel.py:64-72) drops eps and never writes ``s``;
    this restates the eager semantics instead, as the two-pass baseline does
    (residual_rms_baseline.py:74-84).
    """
    s = _f(x) if residual is None else _f(residual) + _f(x)
    if sum_dtype is not None:
        s = s.to(sum_dtype).to(F32)
    return rmsnorm_offset(s, weight, eps), s


def packed_conv_silu(x, weight, cu_seqlens=None, key_dim=None, value_dim=None, head_dim=128):
    """Depthwise causal conv1d (width K, left zero pad K-1) + SiLU, split into q/k/v.

    Restates the reference's independent fp64 token-major check
    (experiments/packed_conv/check_packed_output_conv.py:21-32) and the module path
    ``F.silu(conv1d(x)[..., :T])`` ([tf]:465-474, split at :476-489).  ``x`` is ``[B, T, C]``,
    ``weight`` ``[C, K]`` or ``[C, 1, K]``.  With ``cu_seqlens`` (packed varlen, B == 1) every segment
    starts with a zero history.  Returns float32 ``q, k, v`` of shape ``[B, T, H, head_dim]``.
    """
    xd = _f(x, torch.float64)
    B, T, C = xd.shape
    w = _f(weight, torch.float64).reshape(C, -1)
    K = w.shape[1]
    if cu_seqlens is None:
        bounds = [(b, 0, T) for b in range(B)]
    else:
        cs = [int(v) for v in cu_seqlens]
        assert B == 1, "packed varlen input has batch 1"
        bounds = [(0, cs[i], cs[i + 1]) for i in range(len(cs) - 1)]
    acc = torch.zeros_like(xd)
    for b, s0, s1 in bounds:
        seg = xd[b, s0:s1]
        L = s1 - s0
        out = torch.zeros_like(seg)
        for tap in range(K):
            lag = K - 1 - tap
            if lag < L:
                out[lag:] += seg[: L - lag] * w[:, tap]
        acc[b, s0:s1] = out
    y = (acc * torch.sigmoid(acc)).to(F32)
    if key_dim is None:
        key_dim = C // 3
    if value_dim is None:
        value_dim = C - 2 * key_dim
    q, k, v = y.split([key_dim, key_dim, value_dim], dim=-1)
    return (q.reshape(B, T, -1, head_dim), k.reshape(B, T, -1, head_dim),
            v.reshape(B, T, -1, head_dim))


def gdn_gates(a, b, A_log, dt_bias):
    """``beta = sigmoid(b)``; ``g = -exp(A_log) * softplus(a + dt_bias)`` ([tf]:491-493).

    Same arithmetic as the reference's fused kernel (unpack_gate_transform_kernel.py:69-75):
    softplus switches to the identity above 20, as ``F.softplus`` does.
    """
    beta = torch.sigmoid(_f(b))
    g = -torch.exp(_f(A_log)) * F.softplus(_f(a) + _f(dt_bias))
    return g, beta


def gated_rmsnorm(o, z, weight, eps: float = 1e-6, round_dtype=None):
    """Qwen3_5RMSNormGated: ``w * rmsnorm(o) * silu(z)`` per head row ([tf]:175-190).

    Normalises over the last dim in float32.  The module rounds the normalised row to the input
    dtype before the weight multiply ([tf]:187); pass ``round_dtype`` to reproduce that.
    """
    x = _f(o)
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    if round_dtype is not None:
        x = x.to(round_dtype).to(F32)
    return _f(weight) * x * F.silu(_f(z))


def _segments(T, cu_seqlens):
    if cu_seqlens is None:
        return [(0, T)]
    cs = [int(v) for v in cu_seqlens]
    return [(cs[i], cs[i + 1]) for i in range(len(cs) - 1)]


def _chunk_delta_one(q, k, v, g, beta, chunk_size, state):
    """One sequence of the chunked gated delta rule, float32, ``[H, T, D]`` inputs ([tf]:252-311)."""
    H, T, Dk = k.shape
    Dv = v.shape[-1]
    pad = (chunk_size - T % chunk_size) % chunk_size
    q = F.pad(q, (0, 0, 0, pad))
    k = F.pad(k, (0, 0, 0, pad))
    v = F.pad(v, (0, 0, 0, pad))
    beta = F.pad(beta, (0, pad))
    g = F.pad(g, (0, pad))
    Tp = T + pad
    q = q * (1.0 / math.sqrt(Dk))                                     # [tf]:266-267
    v_beta = v * beta.unsqueeze(-1)                                    # [tf]:269
    k_beta = k * beta.unsqueeze(-1)                                    # [tf]:270
    n = Tp // chunk_size
    q, k, v_beta, k_beta = (x.reshape(H, n, chunk_size, x.shape[-1]) for x in (q, k, v_beta, k_beta))
    g = g.reshape(H, n, chunk_size).cumsum(-1)                         # [tf]:276-279
    upper_incl = torch.triu(torch.ones(chunk_size, chunk_size, dtype=torch.bool), 0)
    decay = ((g.unsqueeze(-1) - g.unsqueeze(-2)).tril().exp()).tril()  # [tf]:280
    attn = -((k_beta @ k.transpose(-1, -2)) * decay).masked_fill(upper_incl, 0)   # [tf]:281
    for i in range(1, chunk_size):                                     # [tf]:282-285 forward substitution
        row = attn[..., i, :i].clone()
        sub = attn[..., :i, :i].clone()
        attn[..., i, :i] = row + (row.unsqueeze(-1) * sub).sum(-2)
    attn = attn + torch.eye(chunk_size)                                # [tf]:286
    u = attn @ v_beta                                                  # [tf]:287
    w = attn @ (k_beta * g.exp().unsqueeze(-1))                        # [tf]:288
    S = torch.zeros(H, Dk, Dv) if state is None else state.clone()
    out = torch.zeros(H, n, chunk_size, Dv)
    upper = torch.triu(torch.ones(chunk_size, chunk_size, dtype=torch.bool), 1)
    for c in range(n):                                                 # [tf]:297-309
        q_c, k_c = q[:, c], k[:, c]
        a = (q_c @ k_c.transpose(-1, -2) * decay[:, c]).masked_fill(upper, 0)
        v_new = u[:, c] - w[:, c] @ S
        out[:, c] = (q_c * g[:, c, :, None].exp()) @ S + a @ v_new
        S = S * g[:, c, -1, None, None].exp() + (
            k_c * (g[:, c, -1, None] - g[:, c]).exp()[..., None]).transpose(-1, -2) @ v_new
    return out.reshape(H, Tp, Dv)[:, :T], S


def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size: int = 64, initial_state=None,
                           output_final_state: bool = False, use_qk_l2norm_in_kernel: bool = True,
                           cu_seqlens=None):
    """Chunked gated delta rule, transformers' torch path ([tf]:234-311), float32 on CPU.

    Layout as the call site passes it ([tf]:499-508): ``query/key [B, T, H, Dk]``, ``value
    [B, T, H, Dv]``, ``g/beta [B, T, H]``.  ``cu_seqlens`` (packed varlen, B == 1) runs each segment
    independently from a zero (or ``initial_state[i]``) state, which is what the reference's
    packed call site asks for (packed_conv.py:55-59).  Returns ``(o [B, T, H, Dv] float32,
    final_state [N, H, Dk, Dv] or None)``.
    """
    q, k, v, gg, bb = (_f(t) for t in (query, key, value, g, beta))
    if use_qk_l2norm_in_kernel:                                        # [tf]:246-248
        q = l2norm(q)
        k = l2norm(k)
    B, T, H, _ = k.shape
    out = torch.zeros(B, T, H, v.shape[-1])
    states = []
    for b in range(B):
        segs = _segments(T, cu_seqlens) if cu_seqlens is not None else [(0, T)]
        for si, (s0, s1) in enumerate(segs):
            st = None
            if initial_state is not None:
                st = _f(initial_state[si if cu_seqlens is not None else b])
            if s1 <= s0:  # an empty request keeps its initial (or zero) state
                states.append(st if st is not None else torch.zeros(H, k.shape[-1], v.shape[-1]))
                continue
            o, S = _chunk_delta_one(q[b, s0:s1].transpose(0, 1), k[b, s0:s1].transpose(0, 1),
                                    v[b, s0:s1].transpose(0, 1), gg[b, s0:s1].transpose(0, 1),
                                    bb[b, s0:s1].transpose(0, 1), chunk_size, st)
            out[b, s0:s1] = o.transpose(0, 1)
            states.append(S)
    return out, (torch.stack(states) if output_final_state else None)


def recurrent_gated_delta_rule(query, key, value, g, beta, use_qk_l2norm_in_kernel: bool = True,
                               cu_seqlens=None):
    """Token-by-token form of the same rule ([tf]:314-353); used to cross-check the chunked form."""
    q, k, v, gg, bb = (_f(t) for t in (query, key, value, g, beta))
    if use_qk_l2norm_in_kernel:
        q = l2norm(q)
        k = l2norm(k)
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    q = q / math.sqrt(Dk)
    out = torch.zeros(B, T, H, Dv)
    for b in range(B):
        for s0, s1 in _segments(T, cu_seqlens):
            S = torch.zeros(H, Dk, Dv)
            for t in range(s0, s1):
                S = S * gg[b, t].exp()[:, None, None]
                kv_mem = (S * k[b, t][:, :, None]).sum(-2)
                delta = (v[b, t] - kv_mem) * bb[b, t][:, None]
                S = S + k[b, t][:, :, None] * delta[:, None, :]
                out[b, t] = (S * q[b, t][:, :, None]).sum(-2)
    return out


def rope_cos_sin(positions, head_dim: int, partial_rotary_factor: float = 0.25,
                 theta: float = 10000.0):
    """Text-only rotary tables: ``inv_freq`` ([tf]:106-135) and ``cat(freqs, freqs)`` ([tf]:139-155).

    For text input the three M-RoPE position rows are identical, so the interleave
    ([tf]:157-172) leaves the frequencies unchanged.  Returns float32 ``cos, sin [T, rot_dim]``.
    """
    dim = int(head_dim * partial_rotary_factor)
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    pos = torch.as_tensor(positions).to(F32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def apply_partial_rope(x, cos, sin):
    """Rotate the first ``rot_dim`` features of ``x [T, H, D]`` ([tf]:536-579), float32."""
    x = _f(x)
    r = cos.shape[-1]
    xr, xp = x[..., :r], x[..., r:]
    half = r // 2
    rot = torch.cat([-xr[..., half:], xr[..., :half]], dim=-1)
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([xr * c + rot * s, xp], dim=-1)


def gqa_attention_varlen(q, k, v, cu_seqlens=None, scale=None):
    """Causal GQA attention over packed segments, float32 softmax.

    Per segment this is the eager path ``softmax(q @ repeat_kv(k)^T * scale + causal) @ repeat_kv(v)``
    ([tf]:582-617), which is also the reference's fp32 math-SDPA check with ``enable_gqa``
    (experiments/native_gqa/bench_native_gqa.py:46-48).  ``q [T, Hq, D]``, ``k, v [T, Hkv, D]``;
    query head ``h`` reads KV head ``h // (Hq // Hkv)`` (native_gqa_kernel.py:41).
    """
    q, k, v = _f(q), _f(k), _f(v)
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    out = torch.zeros(T, Hq, v.shape[-1])
    for s0, s1 in _segments(T, cu_seqlens):
        L = s1 - s0
        if L <= 0:
            continue
        qs = q[s0:s1].transpose(0, 1)                                   # [Hq, L, D]
        ks = k[s0:s1].transpose(0, 1).repeat_interleave(rep, 0)
        vs = v[s0:s1].transpose(0, 1).repeat_interleave(rep, 0)
        sc = (qs @ ks.transpose(-1, -2)) * scale
        mask = torch.ones(L, L, dtype=torch.bool).triu(1)
        sc = sc.masked_fill(mask, float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s0:s1] = (p @ vs).transpose(0, 1)
    return out


def swiglu(gate, up):
    """``silu(gate) * up`` ([tf]:706-708), float32."""
    return F.silu(_f(gate)) * _f(up)


def slot_readout(hidden_last, final_norm_weight, letter_weight, slots, nopts, eps=1e-6,
                 temperature=1.0):
    """Final norm at the slot rows, restricted logits and masked softmax.

    ``h = norm(hidden)`` ([tf]:1285), ``logits = h[slots] @ W_letters^T`` (model.py:23-27 /
    engine.py:115-117), mask options ``>= nopts`` to -inf and ``softmax(logits / T)``
    (engine.py:48-56, temperature.py:136-144).  Returns ``(probs [N, K], logits [N, K])``.
    """
    h = rmsnorm_offset(_f(hidden_last)[torch.as_tensor(slots)], final_norm_weight, eps)
    logits = h @ _f(letter_weight).t()
    K = logits.shape[1]
    nop = torch.as_tensor(nopts)
    masked = logits.masked_fill(torch.arange(K)[None, :] >= nop[:, None], float("-inf"))
    return torch.softmax(masked / temperature, dim=-1), logits
