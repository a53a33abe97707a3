"""PyTorch operator surface over the C ABI, mirroring the reference's ``fastdecisions::*`` ops.

Each op validates its arguments in Python (``ValueError``, as the reference launchers do:
packed_conv_kernel.py:195-212, native_gqa_kernel.py:122-143, persistent_residual_rms_kernel.py:
76-89), allocates its outputs on the input's device, and launches on the current CUDA stream
through ``libfdk.so``.  Ops are ``torch.library.custom_op``s with ``register_fake`` shape contracts,
so ``torch.compile`` sees each as one graph node, and they are CUDA-graph capturable (no host
synchronisation, no allocation inside the library).  There is no CPU path: a CPU tensor raises.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

BF16 = torch.bfloat16


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("fastdecisions_b200 ops run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must share one CUDA device")


def _aligned(*ts):
    for t in ts:
        if t is not None and t.data_ptr() % 16:
            raise ValueError("tensors must be 16-byte aligned")


# ------------------------------------------------------------------------------------------------
# Residual add + RMSNorm  (persistent_residual_rms.py:7-14)
# ------------------------------------------------------------------------------------------------
def residual_rmsnorm(x: torch.Tensor, residual: Optional[torch.Tensor], weight: torch.Tensor,
                     eps: float = 1e-6, weight_offset: float = 1.0, write_residual: bool = True,
                     out: Optional[torch.Tensor] = None, residual_out: Optional[torch.Tensor] = None,
                     residual_fp32: Optional[bool] = None):
    """Returns ``(normed, summed)``: ``summed = x + residual`` (x when residual is None), stored in
    the residual stream's dtype (bf16, rounded, or float32 when ``residual_fp32``), and
    ``normed = bf16(summed * rsqrt(mean(summed^2) + eps) * (weight_offset + w))``."""
    _need_cuda(x, residual, weight)
    if residual_fp32 is None:
        residual_fp32 = residual is not None and residual.dtype == torch.float32
    rdt = torch.float32 if residual_fp32 else BF16
    if x.dtype != BF16 or (residual is not None and residual.dtype != rdt):
        raise ValueError("residual_rmsnorm: x must be bf16 and the residual bf16 or float32")
    if x.dim() < 1 or x.shape[-1] != weight.numel() or weight.dim() != 1:
        raise ValueError("residual_rmsnorm: weight must be a vector of the hidden size")
    if residual is not None and residual.shape != x.shape:
        raise ValueError("residual_rmsnorm: residual inputs must have identical shapes")
    if weight.dtype not in (BF16, torch.float32) or not weight.is_contiguous():
        raise ValueError("residual_rmsnorm: weight must be a contiguous bf16 or fp32 vector")
    H = x.shape[-1]
    x2 = x.reshape(-1, H)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, H)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
    rows = x2.shape[0]
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=BF16)
    if write_residual and residual_out is None:
        residual_out = torch.empty(x.shape, device=x.device, dtype=rdt)
    if write_residual and residual_out.dtype != rdt:
        raise ValueError("residual_rmsnorm: residual_out dtype must match the residual stream")
    o2 = out.reshape(-1, H)
    ro2 = residual_out.reshape(-1, H) if write_residual else None
    with torch.cuda.device(x.device):
        _lib.call("fdk_residual_rmsnorm", x2.data_ptr(), x2.stride(0) if rows > 1 else H,
                  _ptr(r2), (r2.stride(0) if rows > 1 else H) if r2 is not None else 0, int(residual_fp32),
                  weight.data_ptr(), int(weight.dtype == torch.float32), o2.data_ptr(),
                  o2.stride(0) if rows > 1 else H, _ptr(ro2),
                  (ro2.stride(0) if rows > 1 else H) if ro2 is not None else 0, rows, H,
                  float(eps), float(weight_offset), _stream(x))
    return out, (residual_out if write_residual else None)


def rmsnorm_stream(h: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, weight_offset: float = 1.0,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``bf16(h * rsqrt(mean(h^2) + eps) * (weight_offset + w))`` of the residual stream ``h`` itself
    (float32 or bf16, last dim contiguous): the norm after a GEMM that already added into ``h``."""
    _need_cuda(h, weight)
    if h.dtype not in (torch.float32, BF16) or h.shape[-1] != weight.numel() or h.stride(-1) != 1:
        raise ValueError("rmsnorm_stream: h must be float32 or bf16 with the hidden size last")
    H = h.shape[-1]
    h2 = h.reshape(-1, H)
    rows = h2.shape[0]
    if out is None:
        out = torch.empty(h.shape, device=h.device, dtype=BF16)
    o2 = out.reshape(-1, H)
    with torch.cuda.device(h.device):
        _lib.call("fdk_residual_rmsnorm", None, 0, h2.data_ptr(), h2.stride(0) if rows > 1 else H,
                  int(h.dtype == torch.float32), weight.data_ptr(), int(weight.dtype == torch.float32), o2.data_ptr(),
                  o2.stride(0) if rows > 1 else H, None, 0, rows, H, float(eps), float(weight_offset), _stream(h))
    return out


@torch.library.custom_op("fastdecisions::residual_rms", mutates_args=(), device_types="cuda")
def residual_rms(a: torch.Tensor, b: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Reference signature (persistent_residual_rms.py:7-9): RMSNorm(1+w, eps 1e-6) of a + b."""
    return residual_rmsnorm(a, b, weight, 1e-6, 1.0, write_residual=False)[0]


@residual_rms.register_fake
def _residual_rms_fake(a, b, weight):
    return a.new_empty(a.shape)


@torch.library.custom_op("fastdecisions::residual_rms2", mutates_args=(), device_types="cuda")
def residual_rms2(a: torch.Tensor, b: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Extended form: ``(normed, updated residual)`` written in one pass."""
    n, s = residual_rmsnorm(a, b, weight, 1e-6, 1.0, write_residual=True)
    return n, s


@residual_rms2.register_fake
def _residual_rms2_fake(a, b, weight):
    return a.new_empty(a.shape), a.new_empty(a.shape)


# ------------------------------------------------------------------------------------------------
# Packed causal conv + SiLU  (packed_conv.py:12-21, packed_conv_kernel.py:194-232)
# ------------------------------------------------------------------------------------------------
def packed_conv_qkv(x: torch.Tensor, weight: torch.Tensor, key_dim: Optional[int] = None,
                    value_dim: Optional[int] = None, head_dim: int = 128,
                    cu_seqlens: Optional[torch.Tensor] = None):
    """``x [B, T, C]`` (last dim contiguous, any row stride) -> ``q, k [B, T, Hk, D]``, ``v [B, T, Hv, D]``."""
    _need_cuda(x, weight, cu_seqlens)
    if x.dim() != 3:
        raise ValueError("packed_conv: expected x of shape [B, T, C]")
    B, T, C = x.shape
    if x.dtype != BF16 or weight.dtype != BF16:
        raise ValueError("packed_conv: x and weight must be bf16")
    if weight.dim() == 3:
        if weight.shape[1] != 1:
            raise ValueError("packed_conv: depthwise weight must be [C, 1, K]")
        weight = weight.reshape(weight.shape[0], weight.shape[2])
    if weight.dim() != 2 or weight.shape[0] != C or not weight.is_contiguous():
        raise ValueError("packed_conv: weight must be a contiguous [C, K] or [C, 1, K] tensor")
    K = weight.shape[1]
    if key_dim is None:
        key_dim = C // 3
    if value_dim is None:
        value_dim = C - 2 * key_dim
    if 2 * key_dim + value_dim != C or key_dim % head_dim or value_dim % head_dim:
        raise ValueError("packed_conv: C must equal 2*key_dim + value_dim with whole heads")
    if x.stride(2) != 1 or (B > 1 and x.stride(0) != T * x.stride(1)):
        x = x.contiguous()
    ldx = x.stride(1) if T > 1 else C
    _aligned(x, weight)
    nseg = 0
    if cu_seqlens is not None:
        if B != 1 or cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1:
            raise ValueError("packed_conv: cu_seqlens must be int32 [S+1] with batch 1")
        nseg = cu_seqlens.numel() - 1
    q = torch.empty((B, T, key_dim // head_dim, head_dim), device=x.device, dtype=BF16)
    k = torch.empty_like(q)
    v = torch.empty((B, T, value_dim // head_dim, head_dim), device=x.device, dtype=BF16)
    with torch.cuda.device(x.device):
        _lib.call("fdk_packed_conv_silu", x.data_ptr(), ldx, weight.data_ptr(), B, T, C, K,
                  _ptr(cu_seqlens), nseg, key_dim, value_dim, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                  _stream(x))
    return q, k, v


@torch.library.custom_op("fastdecisions::packed_conv", mutates_args=(), device_types="cuda")
def packed_conv(x: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Reference signature (packed_conv.py:12-14): C = 3 * 16 * 128 split evenly into q/k/v."""
    return packed_conv_qkv(x, weight)


@packed_conv.register_fake
def _packed_conv_fake(x, weight):
    B, T, C = x.shape
    shape = (B, T, C // 3 // 128, 128)
    return tuple(x.new_empty(shape) for _ in range(3))


@torch.library.custom_op("fastdecisions::packed_conv_varlen", mutates_args=(), device_types="cuda")
def packed_conv_varlen(x: torch.Tensor, weight: torch.Tensor, cu_seqlens: torch.Tensor,
                       key_dim: int, value_dim: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return packed_conv_qkv(x, weight, key_dim, value_dim, 128, cu_seqlens)


@packed_conv_varlen.register_fake
def _packed_conv_varlen_fake(x, weight, cu_seqlens, key_dim, value_dim):
    B, T, _ = x.shape
    return (x.new_empty((B, T, key_dim // 128, 128)), x.new_empty((B, T, key_dim // 128, 128)),
            x.new_empty((B, T, value_dim // 128, 128)))


# ------------------------------------------------------------------------------------------------
# Gate transform  (combined_gates.py:6-16, unpack_gate_transform_kernel.py:92-130)
# ------------------------------------------------------------------------------------------------
def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """``a, b [..., H]`` (bf16, last dim contiguous) -> ``g`` float32, ``beta`` bf16 of the same shape."""
    _need_cuda(a, b, A_log, dt_bias)
    if a.dtype != BF16 or b.dtype != BF16 or a.shape != b.shape:
        raise ValueError("gdn_gates: a and b must be bf16 tensors of one shape")
    H = a.shape[-1]
    if A_log.shape != (H,) or dt_bias.shape != (H,):
        raise ValueError(f"gdn_gates: A_log and dt_bias must have shape [{H}]")
    a2, b2 = a.reshape(-1, H), b.reshape(-1, H)
    if a2.stride(-1) != 1:
        a2 = a2.contiguous()
    if b2.stride(-1) != 1:
        b2 = b2.contiguous()
    al = A_log.float().contiguous()
    db = dt_bias.float().contiguous()
    g = torch.empty(a.shape, device=a.device, dtype=torch.float32)
    beta = torch.empty(a.shape, device=a.device, dtype=BF16)
    n = a2.shape[0]
    with torch.cuda.device(a.device):
        _lib.call("fdk_gdn_gates", a2.data_ptr(), a2.stride(0) if n > 1 else H, b2.data_ptr(),
                  b2.stride(0) if n > 1 else H, al.data_ptr(), db.data_ptr(), g.data_ptr(), beta.data_ptr(),
                  n, H, _stream(a))
    return g, beta


@torch.library.custom_op("fastdecisions::unpack_gate", mutates_args=(), device_types="cuda")
def unpack_gate(combined: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference signature (combined_gates.py:6-9): ``combined [B, T, 2H]`` holds a then b."""
    if combined.dim() != 3 or combined.shape[-1] % 2:
        raise ValueError("unpack_gate: combined must have shape [B, T, 2H]")
    H = combined.shape[-1] // 2
    return gdn_gates(combined[..., :H], combined[..., H:], a_log, dt_bias)


@unpack_gate.register_fake
def _unpack_gate_fake(combined, a_log, dt_bias):
    shape = (*combined.shape[:-1], combined.shape[-1] // 2)
    return combined.new_empty(shape, dtype=torch.float32), combined.new_empty(shape, dtype=BF16)


# ------------------------------------------------------------------------------------------------
# Chunked gated delta rule  ([tf]:234-311, call sites packed_conv.py:55-59, [tf]:499-508)
# ------------------------------------------------------------------------------------------------
def delta_rule_workspace_bytes(tokens: int, segments: int, heads: int, dk: int = 128, dv: int = 128) -> int:
    return int(_lib.load().fdk_chunk_gated_delta_rule_workspace_size(tokens, segments, heads, dk, dv))


def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size=64, initial_state=None,
                           output_final_state=False, use_qk_l2norm_in_kernel=True, cu_seqlens=None,
                           workspace: Optional[torch.Tensor] = None, **kwargs):
    """Drop-in for transformers' ``chunk_gated_delta_rule`` (same signature and layout):
    ``query/key [B, T, H, Dk]``, ``value [B, T, H, Dv]``, ``g [B, T, H]`` (log decay), ``beta [B, T, H]``.
    Returns ``(o [B, T, H, Dv] bf16, final_state [N, H, Dk, Dv] float32 or None)``; with
    ``cu_seqlens`` (int32 ``[N + 1]``, B == 1) each packed segment is an independent sequence.
    """
    _need_cuda(query, key, value, g, beta, initial_state, cu_seqlens)
    if chunk_size != 64:
        raise ValueError("chunk_gated_delta_rule: chunk_size must be 64")
    if not use_qk_l2norm_in_kernel:
        raise ValueError("chunk_gated_delta_rule: only use_qk_l2norm_in_kernel=True is implemented")
    if query.dim() != 4 or key.shape != query.shape or value.dim() != 4:
        raise ValueError("chunk_gated_delta_rule: expected [B, T, H, D] query/key/value")
    B, T, H, Dk = key.shape
    Dv = value.shape[-1]
    if value.shape[:3] != (B, T, H) or g.shape != (B, T, H) or beta.shape != (B, T, H):
        raise ValueError("chunk_gated_delta_rule: shape mismatch between q/k/v/g/beta")
    if Dk != 128 or Dv != 128:
        raise ValueError("chunk_gated_delta_rule: head dims must be 128")
    q = query if query.dtype == BF16 else query.to(BF16)
    k = key if key.dtype == BF16 else key.to(BF16)
    v = value if value.dtype == BF16 else value.to(BF16)
    # token-major [B*T, H, D] views with a common token stride for q and k
    if not (q.stride(3) == 1 and q.stride(2) == Dk and (B == 1 or q.stride(0) == T * q.stride(1))):
        q = q.contiguous()
    if not (k.stride(3) == 1 and k.stride(2) == Dk and k.stride(1) == q.stride(1) and (B == 1 or k.stride(0) == T * k.stride(1))):
        k = k.contiguous()
        if q.stride(1) != k.stride(1):
            q = q.contiguous()
    if not (v.stride(3) == 1 and v.stride(2) == Dv and (B == 1 or v.stride(0) == T * v.stride(1))):
        v = v.contiguous()
    gg = g.float().contiguous()
    bb = beta.to(BF16).contiguous()
    _aligned(q, k, v)
    if cu_seqlens is None:
        cu = torch.arange(0, (B + 1) * T, T, device=q.device, dtype=torch.int32)
        nseg = B
    else:
        if B != 1:
            raise ValueError("chunk_gated_delta_rule: cu_seqlens needs batch size 1")
        cu = cu_seqlens.to(torch.int32).contiguous()
        nseg = cu.numel() - 1
    tokens = B * T
    init = None
    if initial_state is not None:
        if initial_state.shape != (nseg, H, Dk, Dv):
            raise ValueError(f"chunk_gated_delta_rule: initial_state must be [{nseg}, {H}, {Dk}, {Dv}]")
        init = initial_state.float().contiguous()
    out = torch.empty((B, T, H, Dv), device=q.device, dtype=BF16)
    final = torch.empty((nseg, H, Dk, Dv), device=q.device, dtype=torch.float32) if output_final_state else None
    need = delta_rule_workspace_bytes(tokens, nseg, H, Dk, Dv)
    if workspace is None or workspace.numel() < need or workspace.data_ptr() % 256:
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    with torch.cuda.device(q.device):
        _lib.call("fdk_chunk_gated_delta_rule_fwd", q.data_ptr(), k.data_ptr(), q.stride(1) if T > 1 else H * Dk,
                  v.data_ptr(), v.stride(1) if T > 1 else H * Dv, gg.data_ptr(), bb.data_ptr(), cu.data_ptr(), nseg,
                  tokens, H, Dk, Dv, float(Dk ** -0.5), _ptr(init), out.data_ptr(), _ptr(final),
                  workspace.data_ptr(), workspace.numel(), _stream(q))
    return out, final


def gdn_fused_delta_rule(proj: torch.Tensor, conv_weight: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
                         heads: int, a_col: int, b_col: int, cu_seqlens: torch.Tensor,
                         workspace: Optional[torch.Tensor] = None, head_dim: int = 128) -> torch.Tensor:
    """The Gated-DeltaNet mixer core straight from the in-projection ``proj [T, >= C]`` (bf16, unit
    column stride): conv + SiLU of its q / k / v columns, the gates from columns ``a_col + h`` /
    ``b_col + h``, and the chunked delta rule over the packed segments of ``cu_seqlens`` -- the
    results of ``packed_conv_qkv``, ``gdn_gates`` and ``chunk_gated_delta_rule`` in one call.
    Returns ``o [T, heads, 128]`` bf16."""
    _need_cuda(proj, conv_weight, A_log, dt_bias, cu_seqlens)
    if proj.dim() != 2 or proj.dtype != BF16 or proj.stride(1) != 1:
        raise ValueError("gdn_fused_delta_rule: proj must be a bf16 [T, C] tensor with unit column stride")
    if head_dim != 128:
        raise ValueError("gdn_fused_delta_rule: head_dim must be 128")
    T = proj.shape[0]
    kd = vd = heads * head_dim
    w = conv_weight.reshape(conv_weight.shape[0], conv_weight.shape[-1])
    if w.dtype != BF16 or not w.is_contiguous() or w.shape != (2 * kd + vd, 4):
        raise ValueError("gdn_fused_delta_rule: conv weight must be a contiguous bf16 [C, 4] (or [C, 1, 4]) tensor")
    cu = cu_seqlens.to(torch.int32).contiguous()
    nseg = cu.numel() - 1
    ld = proj.stride(0) if T > 1 else proj.shape[1]
    out = torch.empty((T, heads, head_dim), device=proj.device, dtype=BF16)
    need = delta_rule_workspace_bytes(T, nseg, heads)
    if workspace is None or workspace.numel() < need or workspace.data_ptr() % 256:
        workspace = torch.empty(need, device=proj.device, dtype=torch.uint8)
    al = A_log.float().contiguous()
    dt = dt_bias.float().contiguous()
    with torch.cuda.device(proj.device):
        _lib.call("fdk_gdn_fused_delta_rule_fwd", proj.data_ptr(), ld, w.data_ptr(), 4, kd, vd, a_col, b_col,
                  al.data_ptr(), dt.data_ptr(), cu.data_ptr(), nseg,
                  T, heads, float(head_dim ** -0.5), None, out.data_ptr(), None, workspace.data_ptr(),
                  workspace.numel(), _stream(proj))
    return out


# ------------------------------------------------------------------------------------------------
# GDN gated norm, attention prologue, GQA attention, embedding, SwiGLU, readout
# ------------------------------------------------------------------------------------------------
def gated_rmsnorm(o: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                  out: Optional[torch.Tensor] = None):
    """``o [T, H, Dv]`` contiguous, ``z [T, H*Dv]`` (row stride free) -> ``[T, H*Dv]`` bf16."""
    _need_cuda(o, z, weight)
    T, H, Dv = o.shape
    if not o.is_contiguous() or o.dtype != BF16:
        o = o.contiguous().to(BF16)
    z2 = z.reshape(T, H * Dv) if z.dim() != 2 else z
    if z2.stride(-1) != 1:
        z2 = z2.contiguous()
    if out is None:
        out = torch.empty((T, H * Dv), device=o.device, dtype=BF16)
    with torch.cuda.device(o.device):
        _lib.call("fdk_gated_rmsnorm", o.data_ptr(), z2.data_ptr(), z2.stride(0) if T > 1 else H * Dv,
                  weight.data_ptr(), int(weight.dtype == torch.float32), out.data_ptr(), T, H, Dv, float(eps),
                  _stream(o))
    return out


def rope_inv_freq(head_dim: int, partial_rotary_factor: float = 0.25, theta: float = 10000.0,
                  device=None) -> torch.Tensor:
    """``inv_freq`` exactly as transformers computes it ([tf]:106-135), float32."""
    dim = int(head_dim * partial_rotary_factor)
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))
    return inv.to(device)


def rope_table(inv_freq: torch.Tensor, max_pos: int) -> torch.Tensor:
    """``[max_pos, rot_dim]`` float32: cos(p * inv_freq) then sin(p * inv_freq) per position,
    computed as transformers does (fp32 angle ``p * inv_freq``, then cos / sin; [tf]:139-155)."""
    pos = torch.arange(max_pos, device=inv_freq.device, dtype=torch.float32)
    ang = pos[:, None] * inv_freq.float()[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).contiguous()


def attn_qk_norm_rope(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                      positions: torch.Tensor, rope: torch.Tensor, hq: int, hkv: int, head_dim: int,
                      eps: float = 1e-6):
    """``qkv [T, >= (2*hq + hkv)*D]`` (q_proj then k_proj columns) -> ``q [T, hq, D]``, ``k [T, hkv, D]``.
    ``rope`` is the ``rope_table`` ([max_pos, rot_dim]); positions must be < max_pos."""
    _need_cuda(qkv, q_norm_w, k_norm_w, positions, rope)
    T = qkv.shape[0]
    if rope.dim() != 2 or rope.dtype != torch.float32 or not rope.is_contiguous():
        raise ValueError("attn_qk_norm_rope: rope must be a contiguous float32 [max_pos, rot_dim] table")
    rot = rope.shape[1]
    q = torch.empty((T, hq, head_dim), device=qkv.device, dtype=BF16)
    k = torch.empty((T, hkv, head_dim), device=qkv.device, dtype=BF16)
    with torch.cuda.device(qkv.device):
        _lib.call("fdk_attn_qk_norm_rope", qkv.data_ptr(), qkv.stride(0) if T > 1 else qkv.shape[1],
                  q_norm_w.data_ptr(), k_norm_w.data_ptr(), int(q_norm_w.dtype == torch.float32),
                  positions.data_ptr(), rope.data_ptr(), rope.shape[0], rot, q.data_ptr(), k.data_ptr(), T, hq, hkv,
                  head_dim, float(eps), _stream(qkv))
    return q, k


def gqa_attention_varlen_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                          max_seqlen: int, scale: Optional[float] = None, gate: Optional[torch.Tensor] = None,
                          gate_interleaved: bool = False, out: Optional[torch.Tensor] = None):
    """``q [T, Hq, D]``, ``k, v [T, Hkv, D]`` (token stride free, head stride D) -> ``[T, Hq, D]``."""
    _need_cuda(q, k, v, cu_seqlens, gate)
    if q.dtype != BF16 or k.dtype != BF16 or v.dtype != BF16:
        raise ValueError("gqa_attention: q, k, v must be bf16")
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    if k.shape != (T, Hkv, D) or v.shape != (T, Hkv, D):
        raise ValueError("gqa_attention: incompatible q/k/v shapes")
    if Hq % Hkv:
        raise ValueError("gqa_attention: query heads must be divisible by KV heads")
    for t in (q, k, v):
        if t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError("gqa_attention: head stride must equal head_dim and features be contiguous")
    if cu_seqlens.dtype != torch.int32:
        raise ValueError("gqa_attention: cu_seqlens must be int32")
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty((T, Hq, D), device=q.device, dtype=BF16)
    ldg = 0
    if gate is not None:
        ldg = gate.stride(0)
    with torch.cuda.device(q.device):
        _lib.call("fdk_gqa_fwd", q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                  cu_seqlens.data_ptr(), cu_seqlens.numel() - 1, int(max_seqlen), T, Hq, Hkv, D, float(scale),
                  _ptr(gate), ldg, int(gate_interleaved), out.data_ptr(), _stream(q))
    return out


@torch.library.custom_op("fastdecisions::gqa_attention_varlen", mutates_args=(), device_types="cuda")
def gqa_attention_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                         max_seqlen: int) -> torch.Tensor:
    return gqa_attention_varlen_(q, k, v, cu_seqlens, max_seqlen)


@gqa_attention_varlen.register_fake
def _gqa_varlen_fake(q, k, v, cu_seqlens, max_seqlen):
    return q.new_empty(q.shape)


def native_gqa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Reference signature (native_gqa_kernel.py:116-173): logical ``q [B, Hq, T, D]``,
    ``k, v [B, Hkv, T, D]``; returns logical ``[B, Hq, T, D]`` stored physically as ``[B, T, Hq, D]``."""
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("Q, K and V must be four-dimensional")
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    if min(B, Hq, Hkv, T) < 1:
        raise ValueError("Batch, head counts and sequence length must be positive")
    if Hq % Hkv:
        raise ValueError("Query heads must be divisible by KV heads")
    if k.shape != (B, Hkv, T, D) or v.shape != k.shape:
        raise ValueError("Incompatible Q/K/V shapes")
    _need_cuda(q, k, v)
    # token-major [B*T, H, D] views
    qt = q.transpose(1, 2).reshape(B * T, Hq, D)
    kt = k.transpose(1, 2).reshape(B * T, Hkv, D)
    vt = v.transpose(1, 2).reshape(B * T, Hkv, D)
    qt = qt if qt.stride(1) == D and qt.stride(2) == 1 else qt.contiguous()
    kt = kt if kt.stride(1) == D and kt.stride(2) == 1 else kt.contiguous()
    vt = vt if vt.stride(1) == D and vt.stride(2) == 1 else vt.contiguous()
    cu = torch.arange(0, (B + 1) * T, T, device=q.device, dtype=torch.int32)
    o = gqa_attention_varlen_(qt, kt, vt, cu, T)
    return o.reshape(B, T, Hq, D).permute(0, 2, 1, 3)


@torch.library.custom_op("fastdecisions::native_gqa", mutates_args=(), device_types="cuda")
def native_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return native_gqa_attention(q, k, v)


@native_gqa.register_fake
def _native_gqa_fake(q, k, v):
    b, h, t, d = q.shape
    return q.new_empty((b, t, h, d)).permute(0, 2, 1, 3)


def embed(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None):
    _need_cuda(ids, table)
    ids32 = ids.reshape(-1).to(torch.int32)
    T = ids32.numel()
    if out is None:
        out = torch.empty((T, table.shape[1]), device=table.device, dtype=BF16)
    with torch.cuda.device(table.device):
        _lib.call("fdk_embed", ids32.data_ptr(), table.data_ptr(), table.shape[0], table.shape[1], out.data_ptr(),
                  T, _stream(table))
    return out


def swiglu(gu: torch.Tensor, inter: int, out: Optional[torch.Tensor] = None):
    _need_cuda(gu)
    T = gu.shape[0]
    if out is None:
        out = torch.empty((T, inter), device=gu.device, dtype=BF16)
    with torch.cuda.device(gu.device):
        _lib.call("fdk_swiglu", gu.data_ptr(), gu.stride(0) if T > 1 else 2 * inter, out.data_ptr(), T, inter,
                  _stream(gu))
    return out


def slot_readout(hidden: torch.Tensor, slots: torch.Tensor, nopts: torch.Tensor, final_norm_w: torch.Tensor,
                 letters: torch.Tensor, eps: float = 1e-6, temperature: float = 1.0,
                 probs: Optional[torch.Tensor] = None, logits: Optional[torch.Tensor] = None,
                 delta: Optional[torch.Tensor] = None):
    """Final RMSNorm (1+w) of ``hidden[slots] (+ delta[slots])``, logits over ``letters`` rows and
    the masked softmax; ``slots`` are absolute token rows, ``nopts`` the options per slot."""
    _need_cuda(hidden, slots, nopts, final_norm_w, letters, delta)
    if delta is not None and (delta.shape != hidden.shape or not delta.is_contiguous()):
        raise ValueError("slot_readout: delta must be a contiguous tensor shaped like hidden")
    N, K = slots.numel(), letters.shape[0]
    if probs is None:
        probs = torch.empty((N, K), device=hidden.device, dtype=torch.float32)
    if logits is None:
        logits = torch.empty((N, K), device=hidden.device, dtype=torch.float32)
    with torch.cuda.device(hidden.device):
        _lib.call("fdk_slot_readout", hidden.data_ptr(), int(hidden.dtype == torch.float32), _ptr(delta),
                  hidden.shape[-1], slots.data_ptr(), nopts.data_ptr(), N,
                  final_norm_w.data_ptr(), int(final_norm_w.dtype == torch.float32), letters.data_ptr(), K,
                  float(eps), float(temperature), probs.data_ptr(), logits.data_ptr(), _stream(hidden))
    return probs, logits


# ------------------------------------------------------------------------------------------------
# Projection / MLP GEMMs on tcgen05 ([tf]:442-449, 532, 657-664, 691, 706-708)
# ------------------------------------------------------------------------------------------------
GEMM_PLAIN, GEMM_SWIGLU = 0, 1


def interleave_gate_up(gate_w: torch.Tensor, up_w: torch.Tensor, block: int = 128) -> torch.Tensor:
    """``[2 I, H]`` weight for the SwiGLU GEMM: gate / up rows interleaved in blocks of ``block``
    (block j: gate rows ``[block j, +block)`` then the same up rows)."""
    I, H = gate_w.shape
    if up_w.shape != (I, H) or I % block:
        raise ValueError(f"interleave_gate_up: gate and up must both be [I, H] with I a multiple of {block}")
    return torch.stack([gate_w.reshape(I // block, block, H), up_w.reshape(I // block, block, H)], 1).reshape(2 * I, H)


def gemm(a: torch.Tensor, w: torch.Tensor, epilogue: int = GEMM_PLAIN, out: Optional[torch.Tensor] = None):
    """``a [m, k] @ w[n, k]^T`` in bf16 with fp32 accumulation (``w`` in nn.Linear layout).
    ``epilogue=GEMM_SWIGLU``: ``w`` from ``interleave_gate_up`` and the result is
    ``silu(a gate^T) * (a up^T)`` of shape ``[m, n / 2]``."""
    _need_cuda(a, w, out)
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise ValueError("gemm: expected a [m, k] and w [n, k]")
    if a.dtype != BF16 or w.dtype != BF16 or a.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm: a and w must be bf16 with unit column stride")
    m, k = a.shape
    n = w.shape[0]
    nout = n // 2 if epilogue == GEMM_SWIGLU else n
    if out is None:
        out = torch.empty((m, nout), device=a.device, dtype=BF16)
    if out.shape != (m, nout) or out.dtype != BF16 or out.stride(1) != 1:
        raise ValueError("gemm: out must be a bf16 [m, n] (SwiGLU: [m, n / 2]) tensor with unit column stride")
    with torch.cuda.device(a.device):
        _lib.call("fdk_gemm_bf16", a.data_ptr(), a.stride(0) if m > 1 else k, w.data_ptr(),
                  w.stride(0) if n > 1 else k, out.data_ptr(), out.stride(0) if m > 1 else nout, m, n, k,
                  int(epilogue), _stream(a))
    return out


def gemm_qk_norm_rope(a: torch.Tensor, w: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor,
                      positions: torch.Tensor, rope: torch.Tensor, hq: int, hkv: int, head_dim: int,
                      eps: float = 1e-6):
    """Attention projection ``a [m, k] @ w[(2 hq + 2 hkv) D, k]^T`` with q/k RMSNorm (1 + w) and partial
    RoPE fused: returns ``(proj [m, n], q [m, hq, D], k [m, hkv, D])``; ``proj`` holds the output
    gate and v columns (its q / k columns are not written)."""
    _need_cuda(a, w, q_norm_w, k_norm_w, positions, rope)
    m, k = a.shape
    n = w.shape[0]
    if a.dtype != BF16 or w.dtype != BF16 or a.stride(1) != 1 or w.stride(1) != 1 or w.shape[1] != k:
        raise ValueError("gemm_qk_norm_rope: a [m, k] and w [n, k] must be bf16 with unit column stride")
    if q_norm_w.dtype != BF16 or k_norm_w.dtype != BF16 or positions.dtype != torch.int32:
        raise ValueError("gemm_qk_norm_rope: bf16 norm weights and int32 positions expected")
    if rope.dim() != 2 or rope.dtype != torch.float32 or not rope.is_contiguous():
        raise ValueError("gemm_qk_norm_rope: rope must be a contiguous float32 [max_pos, rot_dim] table")
    proj = torch.empty((m, n), device=a.device, dtype=BF16)
    q = torch.empty((m, hq, head_dim), device=a.device, dtype=BF16)
    kk = torch.empty((m, hkv, head_dim), device=a.device, dtype=BF16)
    with torch.cuda.device(a.device):
        _lib.call("fdk_gemm_bf16_qk_norm_rope", a.data_ptr(), a.stride(0) if m > 1 else k, w.data_ptr(),
                  w.stride(0) if n > 1 else k, proj.data_ptr(), n, m, n, k, hq, hkv, head_dim, q_norm_w.data_ptr(),
                  k_norm_w.data_ptr(), positions.data_ptr(), rope.data_ptr(), rope.shape[0], rope.shape[1], float(eps),
                  q.data_ptr(), kk.data_ptr(), _stream(a))
    return proj, q, kk


def residual_add_tickets(m: int, n: int, device) -> torch.Tensor:
    """Zeroed slice-ticket array for ``gemm_residual_add`` of an ``m x n`` output (reusable: every
    completed call leaves it zeroed; calls sharing it must not overlap on the GPU)."""
    return torch.zeros(4 * ((m + 127) // 128) * ((n + 255) // 256) + 2, dtype=torch.int32, device=device)


def gemm_residual_add(a: torch.Tensor, w: torch.Tensor, h: torch.Tensor, split_k: int = 0,
                      tickets: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``h += a @ w^T`` in place: ``a [m, k]`` bf16, ``w [n, k]`` bf16 (nn.Linear layout), ``h [m, n]``
    float32 (the residual stream).  The product is added from fp32 accumulators (never rounded to
    bf16); ``split_k`` slices K (0: chosen by the library to fill the SMs), the slices adding in a
    fixed order kept by ``tickets`` (``residual_add_tickets``; allocated here when not given).
    Returns ``h``."""
    _need_cuda(a, w, h)
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1] or h.shape != (a.shape[0], w.shape[0]):
        raise ValueError("gemm_residual_add: expected a [m, k], w [n, k] and h [m, n]")
    if a.dtype != BF16 or w.dtype != BF16 or h.dtype != torch.float32:
        raise ValueError("gemm_residual_add: a and w must be bf16 and h float32")
    if a.stride(1) != 1 or w.stride(1) != 1 or h.stride(1) != 1:
        raise ValueError("gemm_residual_add: unit column strides required")
    m, k = a.shape
    n = w.shape[0]
    need = 4 * ((m + 127) // 128) * ((n + 255) // 256) + 2
    if tickets is None:
        tickets = residual_add_tickets(m, n, a.device)
    elif tickets.dtype != torch.int32 or tickets.numel() < need:
        raise ValueError(f"gemm_residual_add: tickets must be int32 with at least {need} elements")
    with torch.cuda.device(a.device):
        _lib.call("fdk_gemm_bf16_residual_add", a.data_ptr(), a.stride(0) if m > 1 else k, w.data_ptr(),
                  w.stride(0) if n > 1 else k, h.data_ptr(), h.stride(0) if m > 1 else n, m, n, k, int(split_k),
                  tickets.data_ptr(), _stream(a))
    return h


def split_slices(m: int, n: int, k: int, sms: int = 148, max_slices: int = 4) -> int:
    """K-slices for ``gemm_partials``: the count (every slice non-empty) minimising waves of
    (tile, slice) units over the SMs x (k-steps a unit + 2 for its epilogue); 1 when the
    128 x 256 output tiles alone fill the SMs."""
    tiles = ((m + 127) // 128) * ((n + 255) // 256)
    steps = (k + 63) // 64
    best, best_cost = 1, None
    for s in range(1, min(max_slices, steps) + 1):
        kps = -(-steps // s)
        if -(-steps // kps) != s:
            continue
        cost = -(-tiles * s // sms) * (kps + 2)
        if best_cost is None or cost < best_cost:
            best, best_cost = s, cost
    return best


def gemm_partials(a: torch.Tensor, w: torch.Tensor, partials: torch.Tensor, slices: int) -> torch.Tensor:
    """``partials[s] = a[:, K_s] @ w[:, K_s]^T`` (float32 planes ``[slices, m, n]``) for the ``slices``
    parts of K; ``rmsnorm_add_partials`` adds them into the residual stream in order."""
    _need_cuda(a, w, partials)
    m, k = a.shape
    n = w.shape[0]
    if a.dtype != BF16 or w.dtype != BF16 or w.shape[1] != k or a.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm_partials: a [m, k] and w [n, k] must be bf16 with unit column stride")
    if partials.dtype != torch.float32 or not partials.is_contiguous() or partials.numel() < slices * m * n:
        raise ValueError("gemm_partials: partials must be contiguous float32 with room for [slices, m, n]")
    with torch.cuda.device(a.device):
        _lib.call("fdk_gemm_bf16_partials", a.data_ptr(), a.stride(0) if m > 1 else k, w.data_ptr(),
                  w.stride(0) if n > 1 else k, partials.data_ptr(), m, n, k, int(slices), _stream(a))
    return partials


def rmsnorm_add_partials(partials: torch.Tensor, slices: int, h: torch.Tensor, weight: Optional[torch.Tensor],
                         eps: float = 1e-6, weight_offset: float = 1.0) -> Optional[torch.Tensor]:
    """``h += partials[0] + ... + partials[slices - 1]`` (in that order), then the RMSNorm of ``h``
    (bf16, returned) -- or only the add when ``weight`` is None."""
    _need_cuda(partials, h, weight)
    rows, H = h.shape
    if h.dtype != torch.float32 or h.stride(1) != 1 or partials.dtype != torch.float32:
        raise ValueError("rmsnorm_add_partials: float32 h and partials expected")
    out = None if weight is None else torch.empty((rows, H), device=h.device, dtype=BF16)
    with torch.cuda.device(h.device):
        _lib.call("fdk_rmsnorm_add_partials", partials.data_ptr(), int(slices), h.data_ptr(),
                  h.stride(0) if rows > 1 else H, _ptr(weight), int(weight is not None and weight.dtype == torch.float32),
                  _ptr(out), H, rows, H, float(eps), float(weight_offset), _stream(h))
    return out
