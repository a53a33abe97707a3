"""Drop-in installers: put the B200 kernels into a transformers ``Qwen3_5TextModel`` in place.

Same pattern and names as the reference (src/decider/packed_conv.py:65-75,
persistent_residual_rms.py:36-49, experiments/native_gqa/bench_native_gqa_model.py:43-56,
114-118): each installer patches module instances with ``types.MethodType``, keeps the original
forward under ``_..._original_forward`` (idempotent), returns the number of modules patched, and
the patched forward falls back to the original for anything it does not handle (KV/conv caches,
training/autograd, non-CUDA or non-bf16 input, unsupported geometry).
"""
from __future__ import annotations

from types import MethodType

import torch

from . import ops


# ------------------------------------------------------------------ GDN mixer: packed conv path
def _gdn_supported(self, hidden_states, cache_params):
    return (cache_params is None and not self.training and not torch.is_grad_enabled()
            and hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
            and self.head_k_dim == 128 and self.head_v_dim == 128 and self.num_k_heads == self.num_v_heads
            and self.conv1d.bias is None and self.activation == "silu")


def _gdn_forward(self, hidden_states, cache_params=None, attention_mask=None, **kwargs):
    """Qwen3_5GatedDeltaNet.forward ([tf]:422-533) with packed conv, fused gates, the chunked
    delta-rule kernel and the gated-norm kernel; projections stay the module's own GEMMs."""
    if not _gdn_supported(self, hidden_states, cache_params) or attention_mask is not None:
        return self._packed_original_forward(hidden_states, cache_params=cache_params,
                                             attention_mask=attention_mask, **kwargs)
    B, T, _ = hidden_states.shape
    mixed = self.in_proj_qkv(hidden_states)
    q, k, v = ops.packed_conv_qkv(mixed, self.conv1d.weight, self.key_dim, self.value_dim, self.head_k_dim,
                                  kwargs.get("cu_seq_lens_q"))
    z = self.in_proj_z(hidden_states)
    g, beta = ops.gdn_gates(self.in_proj_a(hidden_states), self.in_proj_b(hidden_states), self.A_log, self.dt_bias)
    o, _ = ops.chunk_gated_delta_rule(q, k, v, g, beta, cu_seqlens=kwargs.get("cu_seq_lens_q"))
    on = ops.gated_rmsnorm(o.reshape(B * T, self.num_v_heads, self.head_v_dim), z.reshape(B * T, -1),
                           self.norm.weight, self.layer_norm_epsilon)
    return self.out_proj(on.reshape(B, T, -1))


def install_packed_conv(core) -> int:
    """Patch this model's GDN modules; returns the number installed (packed_conv.py:65-75)."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5GatedDeltaNet
    n = 0
    for m in core.modules():
        if isinstance(m, Qwen3_5GatedDeltaNet):
            if not hasattr(m, "_packed_original_forward"):
                m._packed_original_forward = m.forward
                m.forward = MethodType(_gdn_forward, m)
            n += 1
    return n


def install_chunk_gated_delta_rule(core) -> int:
    """Only swap the delta-rule function of each GDN module ([tf]:407) for the CUDA kernel."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5GatedDeltaNet
    n = 0
    for m in core.modules():
        if isinstance(m, Qwen3_5GatedDeltaNet):
            m.chunk_gated_delta_rule = ops.chunk_gated_delta_rule
            n += 1
    return n


# ------------------------------------------------------------------ decoder: residual + RMSNorm
def _decoder_forward(self, hidden_states, position_embeddings, attention_mask=None, position_ids=None,
                     past_key_values=None, **kwargs):
    """Decoder layer ([tf]:744-783) with the residual add fused into post_attention_layernorm."""
    if (past_key_values is not None or self.training or torch.is_grad_enabled() or not hidden_states.is_cuda
            or hidden_states.dtype != torch.bfloat16 or not hidden_states.is_contiguous()):
        return self._persistent_original_forward(hidden_states, position_embeddings, attention_mask=attention_mask,
                                                 position_ids=position_ids, past_key_values=past_key_values, **kwargs)
    residual = hidden_states
    x = self.input_layernorm(hidden_states)
    if self.layer_type == "linear_attention":
        mix = self.linear_attn(hidden_states=x, cache_params=None, attention_mask=attention_mask)
    else:
        mix, _ = self.self_attn(hidden_states=x, attention_mask=attention_mask, position_ids=position_ids,
                                past_key_values=None, position_embeddings=position_embeddings, **kwargs)
    normed, summed = ops.residual_rmsnorm(mix.contiguous(), residual, self.post_attention_layernorm.weight,
                                          self.post_attention_layernorm.eps)
    return summed + self.mlp(normed)


def install_persistent_residual_rms(core) -> int:
    """Patch decoder layers (persistent_residual_rms.py:36-49); all layer types are handled here."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5DecoderLayer
    n = 0
    for m in core.modules():
        if isinstance(m, Qwen3_5DecoderLayer):
            if not hasattr(m, "_persistent_original_forward"):
                m._persistent_original_forward = m.forward
                m.forward = MethodType(_decoder_forward, m)
            n += 1
    return n


# ------------------------------------------------------------------ attention: native GQA
def _gqa_geometry_supported(self) -> bool:
    """head_dim 256 (the reference kernel's only shape, native_gqa_kernel.py:132-133) with any head
    ratio, or head_dim 128 with an even number of query heads per KV head."""
    ratio = self.config.num_attention_heads // self.config.num_key_value_heads
    return self.head_dim == 256 or (self.head_dim == 128 and ratio % 2 == 0)


def _attn_forward(self, hidden_states, position_embeddings, attention_mask, past_key_values=None, **kwargs):
    """Qwen3_5Attention.forward ([tf]:647-692) with the native GQA kernel (bench_native_gqa_model.py:43-56).

    Only plain causal masks are accepted: the reference validates that before its patch
    (bench_native_gqa_model.py:86-98); here a non-None 4-D mask that is not causal falls back."""
    if (past_key_values is not None or self.training or torch.is_grad_enabled() or not hidden_states.is_cuda
            or hidden_states.dtype != torch.bfloat16 or not _gqa_geometry_supported(self)):
        return self._gqa_original_forward(hidden_states, position_embeddings, attention_mask,
                                          past_key_values=past_key_values, **kwargs)
    shape = hidden_states.shape[:-1]
    hshape = (*shape, -1, self.head_dim)
    q, gate = torch.chunk(self.q_proj(hidden_states).view(*shape, -1, self.head_dim * 2), 2, dim=-1)
    gate = gate.reshape(*shape, -1)
    q = self.q_norm(q.reshape(hshape)).transpose(1, 2)
    k = self.k_norm(self.k_proj(hidden_states).view(hshape)).transpose(1, 2)
    v = self.v_proj(hidden_states).view(hshape).transpose(1, 2)
    from transformers.models.qwen3_5.modeling_qwen3_5 import apply_rotary_pos_emb
    q, k = apply_rotary_pos_emb(q, k, *position_embeddings)
    out = ops.native_gqa_attention(q, k, v).transpose(1, 2).reshape(*shape, -1)
    return self.o_proj(out * torch.sigmoid(gate)), None


def install_native_gqa(core) -> int:
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Attention
    n = 0
    for m in core.modules():
        if isinstance(m, Qwen3_5Attention):
            if not hasattr(m, "_gqa_original_forward"):
                m._gqa_original_forward = m.forward
                m.forward = MethodType(_attn_forward, m)
            n += 1
    return n


def install_all(core) -> dict:
    return dict(packed_conv=install_packed_conv(core), native_gqa=install_native_gqa(core),
                residual_rms=install_persistent_residual_rms(core))
