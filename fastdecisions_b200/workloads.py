"""Synthetic model configuration, seeded weights and the seeded request workloads of the
benchmark configurations (random init: no checkpoint or dataset is needed or read).

* ``ModelConfig`` is the 2B-class hybrid decoder of config 4: hidden 2048, 24 layers in the
  repeating pattern (linear, linear, linear, full), 16 q / 4 kv heads of 128, 16 x 128 GDN heads,
  conv width 4, SwiGLU 6144, eps 1e-6, vocab 151936.  Layer semantics are transformers 5.5.0
  Qwen3.5 (models/qwen3_5/modeling_qwen3_5.py), which the reference's engine calls.
* ``synthetic_weights`` draws every weight N(0, 0.02) from per-tensor seeds derived from 17 (norm
  weights too, as offsets of the (1 + w) RMSNorms; the GDN gated norm multiplies by
  1 + N(0, 0.02); A_log = log U(1, 16); dt_bias = 1), stored in bf16 under the transformers
  ``state_dict`` names.
* ``config4_request`` / ``config5_requests`` generate the decision requests.
"""
from __future__ import annotations

import concurrent.futures as cf
import math
import os
from dataclasses import dataclass, field

import numpy as np
import torch

# Candidate-answer token ids of the readout (rows of the tied embedding); config 4 reads the first
# four, config 5 the first ``nopts`` (2..8) of them.
LETTER_IDS = (32, 33, 34, 35, 36, 37, 38, 39)


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 24
    full_attention_interval: int = 4
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 16
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    intermediate_size: int = 6144
    rms_norm_eps: float = 1e-6
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10000.0

    @property
    def layer_types(self) -> tuple:
        k = self.full_attention_interval
        return tuple("linear_attention" if (i + 1) % k else "full_attention" for i in range(self.num_hidden_layers))

    def as_dict(self) -> dict:
        d = {f: getattr(self, f) for f in self.__dataclass_fields__}
        d["layer_types"] = list(self.layer_types)
        return d

    def to_transformers(self):
        from transformers import Qwen3_5TextConfig
        c = Qwen3_5TextConfig(
            vocab_size=self.vocab_size, hidden_size=self.hidden_size, num_hidden_layers=self.num_hidden_layers,
            num_attention_heads=self.num_attention_heads, num_key_value_heads=self.num_key_value_heads,
            head_dim=self.head_dim, linear_num_key_heads=self.linear_num_key_heads,
            linear_num_value_heads=self.linear_num_value_heads, linear_key_head_dim=self.linear_key_head_dim,
            linear_value_head_dim=self.linear_value_head_dim, linear_conv_kernel_dim=self.linear_conv_kernel_dim,
            intermediate_size=self.intermediate_size, rms_norm_eps=self.rms_norm_eps,
            layer_types=list(self.layer_types))
        c._attn_implementation = "eager"
        return c

    # ---- work per token / request (used for roofline numerators and load balancing) ----
    def linear_params(self) -> int:
        """Weights multiplied per token by the projection/MLP GEMMs (embedding excluded)."""
        H, I = self.hidden_size, self.intermediate_size
        kd = self.linear_num_key_heads * self.linear_key_head_dim
        vd = self.linear_num_value_heads * self.linear_value_head_dim
        gdn = H * (2 * kd + vd) + H * vd + 2 * H * self.linear_num_value_heads + vd * H
        att = H * (2 * self.num_attention_heads * self.head_dim) + 2 * H * self.num_key_value_heads * self.head_dim \
            + self.num_attention_heads * self.head_dim * H
        mlp = 3 * H * I
        n_lin = sum(1 for t in self.layer_types if t == "linear_attention")
        n_att = self.num_hidden_layers - n_lin
        return n_lin * (gdn + mlp) + n_att * (att + mlp)

    def request_flops(self, L: int) -> float:
        """Forward FLOPs of one request of L tokens: GEMMs, causal attention (QK^T + PV) and the
        chunked delta rule (about 11.7 MFLOP per 64-token chunk and head)."""
        n_att = sum(1 for t in self.layer_types if t == "full_attention")
        n_lin = self.num_hidden_layers - n_att
        lin = 2.0 * self.linear_params() * L
        attn = n_att * 2.0 * self.num_attention_heads * self.head_dim * L * (L + 1)
        delta = n_lin * self.linear_num_value_heads * math.ceil(L / 64) * 11.7e6
        return lin + attn + delta


def _row_blocks(shape, seed, chunk_rows=16384):
    """Empty float32 tensor plus its row blocks ``(flat, r0, r1, block_seed)``; every block has its
    own seed so large tensors are filled in parallel and the values do not depend on threading."""
    out = torch.empty(shape, dtype=torch.float32)
    flat = out.view(shape[0], -1) if len(shape) > 1 else out.view(-1, 1)
    blocks = [(flat, r0, min(flat.shape[0], r0 + chunk_rows), seed * 1009 + r0 // chunk_rows)
              for r0 in range(0, flat.shape[0], chunk_rows)]
    return out, blocks


def synthetic_weights(cfg: ModelConfig = ModelConfig(), seed: int = 17, std: float = 0.02,
                      threads: int | None = None) -> dict:
    """Seeded random weights under transformers ``state_dict`` names (bf16; A_log/dt_bias fp32)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    Hv = cfg.linear_num_value_heads
    specs = [("embed_tokens.weight", (cfg.vocab_size, H), std, 0.0), ("norm.weight", (H,), std, 0.0)]
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        specs += [(p + "input_layernorm.weight", (H,), std, 0.0), (p + "post_attention_layernorm.weight", (H,), std, 0.0),
                  (p + "mlp.gate_proj.weight", (I, H), std, 0.0), (p + "mlp.up_proj.weight", (I, H), std, 0.0),
                  (p + "mlp.down_proj.weight", (H, I), std, 0.0)]
        if kind == "linear_attention":
            la = p + "linear_attn."
            specs += [(la + "in_proj_qkv.weight", (2 * kd + vd, H), std, 0.0), (la + "in_proj_z.weight", (vd, H), std, 0.0),
                      (la + "in_proj_b.weight", (Hv, H), std, 0.0), (la + "in_proj_a.weight", (Hv, H), std, 0.0),
                      (la + "conv1d.weight", (2 * kd + vd, 1, cfg.linear_conv_kernel_dim), std, 0.0),
                      (la + "norm.weight", (cfg.linear_value_head_dim,), std, 1.0),
                      (la + "out_proj.weight", (H, vd), std, 0.0)]
        else:
            sa = p + "self_attn."
            D = cfg.head_dim
            specs += [(sa + "q_proj.weight", (2 * cfg.num_attention_heads * D, H), std, 0.0),
                      (sa + "k_proj.weight", (cfg.num_key_value_heads * D, H), std, 0.0),
                      (sa + "v_proj.weight", (cfg.num_key_value_heads * D, H), std, 0.0),
                      (sa + "o_proj.weight", (H, cfg.num_attention_heads * D), std, 0.0),
                      (sa + "q_norm.weight", (D,), std, 0.0), (sa + "k_norm.weight", (D,), std, 0.0)]
    tensors, jobs = {}, []
    for idx, (name, shape, s, mean) in enumerate(specs):
        out, blocks = _row_blocks(shape, seed * 100003 + idx)
        tensors[name] = out
        jobs += [(flat, r0, r1, bseed, s, mean) for flat, r0, r1, bseed in blocks]

    def fill(job):
        flat, r0, r1, bseed, s_, m_ = job
        g = torch.Generator().manual_seed(bseed)
        flat[r0:r1].normal_(m_, s_, generator=g)

    with cf.ThreadPoolExecutor(max_workers=threads or min(32, os.cpu_count() or 8)) as ex:
        list(ex.map(fill, jobs))
    w = {k: v.to(torch.bfloat16) for k, v in tensors.items()}
    g = torch.Generator().manual_seed(seed)
    for i, kind in enumerate(cfg.layer_types):
        if kind == "linear_attention":
            la = f"layers.{i}.linear_attn."
            w[la + "A_log"] = torch.log(torch.empty(Hv).uniform_(1.0, 16.0, generator=g))
            w[la + "dt_bias"] = torch.ones(Hv)
    return w


def letter_weight(weights: dict, ids=LETTER_IDS) -> torch.Tensor:
    """Readout rows: the (tied) embedding rows of the candidate-answer tokens, ``[K, H]``."""
    return weights["embed_tokens.weight"][list(ids)].clone()


@dataclass
class Request:
    ids: np.ndarray          # int32 token ids
    slot: int                # decision slot position (the readout row)
    nopts: int               # number of candidate answers


def config4_request(seed: int = 17, length: int = 1536, vocab: int = 151936, nopts: int = 4) -> Request:
    """Config 4: batch 1, 1536 uniform random token ids, readout at the last position over 4 options."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (length,), generator=g).numpy().astype(np.int32)
    return Request(ids=ids, slot=length - 1, nopts=nopts)


def config5_requests(n: int = 256, seed: int = 17, vocab: int = 151936, median: float = 800.0,
                     sigma: float = 1.0, lo: int = 64, hi: int = 8192) -> list:
    """Config 5: lengths lognormal(median 800, sigma 1.0) clipped to [64, 8192], candidate counts
    uniform in [2, 8], uniform random ids.  Requests come in blocks of 256 with seeds 17, 18, ...
    so the first 256 are the same for every request count (weak scaling keeps config 5 as rank
    0's share at one GPU)."""
    out = []
    for b in range((n + 255) // 256):
        rng = np.random.default_rng(seed + b)
        m = min(256, n - 256 * b)
        lens = np.clip(np.round(rng.lognormal(math.log(median), sigma, size=256)), lo, hi).astype(np.int64)[:m]
        nopts = rng.integers(2, 9, size=256)[:m]
        for L, k in zip(lens, nopts):
            ids = rng.integers(0, vocab, size=int(L)).astype(np.int32)
            out.append(Request(ids=ids, slot=int(L) - 1, nopts=int(k)))
    return out
