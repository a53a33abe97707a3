"""Generate the golden fixtures that pin the CPU oracle to the reference's own arithmetic.

Run in a container that has transformers 5.5.0 (and, optionally, the FastDecisions sources on
``--reference``): ``python tests/golden/make_golden.py --reference <path to FastDecisions>``.
Every fixture is produced by the third-party code the reference calls (transformers' Qwen3.5
modules, CPU torch fallbacks, float32) or by the reference's own helper where one exists
(``decider.engine.fused_causal_conv1d_fn``, engine.py:25-40).  The outputs are small ``.pt`` files
committed next to this script; nothing here runs at test time.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def small_text_config(**over):
    from transformers import Qwen3_5TextConfig
    kw = dict(vocab_size=128, hidden_size=64, num_hidden_layers=4, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, linear_num_key_heads=2, linear_num_value_heads=2,
              linear_key_head_dim=32, linear_value_head_dim=32, intermediate_size=128,
              rms_norm_eps=1e-6)
    kw.update(over)
    cfg = Qwen3_5TextConfig(**kw)
    cfg._attn_implementation = "eager"
    return cfg


def perturb_norms(module, gen):
    """Give every (1 + w) norm a non-zero offset and every gated norm a non-unit weight."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("q_norm.weight") \
                    or name.endswith("k_norm.weight") or name == "norm.weight":
                p.copy_(torch.randn(p.shape, generator=gen) * 0.1)
            elif name.endswith("linear_attn.norm.weight"):
                p.copy_(1.0 + torch.randn(p.shape, generator=gen) * 0.1)
            elif name.endswith("dt_bias"):
                p.copy_(1.0 + torch.randn(p.shape, generator=gen) * 0.3)


def cfg_dict(cfg):
    return dict(hidden_size=cfg.hidden_size, layer_types=list(cfg.layer_types),
                num_attention_heads=cfg.num_attention_heads,
                num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                linear_num_key_heads=cfg.linear_num_key_heads,
                linear_num_value_heads=cfg.linear_num_value_heads,
                linear_key_head_dim=cfg.linear_key_head_dim,
                linear_value_head_dim=cfg.linear_value_head_dim, rms_norm_eps=cfg.rms_norm_eps,
                partial_rotary_factor=cfg.rope_parameters.get("partial_rotary_factor", 1.0),
                rope_theta=cfg.rope_parameters["rope_theta"], vocab_size=cfg.vocab_size)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="FastDecisions checkout (for src/decider)")
    args = ap.parse_args()
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    import transformers
    assert mq.chunk_gated_delta_rule is None or True
    gen = torch.Generator().manual_seed(17)
    out = {"transformers_version": transformers.__version__}

    # 1. Residual add + Qwen3_5RMSNorm (config 1 distribution, fewer rows).
    x = torch.randn(1, 8, 2048, generator=gen)
    res = torch.randn(1, 8, 2048, generator=gen)
    w = 1.0 + 0.02 * torch.randn(2048, generator=gen)
    norm = mq.Qwen3_5RMSNorm(2048, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(w)
        s = res + x                                          # decoder residual add ([tf]:775)
        out["rmsnorm"] = dict(x=x, residual=res, weight=w, eps=1e-6, summed=s, normed=norm(s))

    # 2. Depthwise causal conv + SiLU: the module's conv1d path and the reference's shifted form.
    C, T = 96, 70
    xc = torch.randn(2, T, C, generator=gen)
    conv = torch.nn.Conv1d(C, C, 4, groups=C, padding=3, bias=False)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(C, 1, 4, generator=gen) * 0.5)
        y_module = F.silu(conv(xc.transpose(1, 2))[:, :, :T]).transpose(1, 2)      # [tf]:474
        fixture = dict(x=xc, weight=conv.weight.detach().clone(), y_module=y_module)
        if args.reference:
            sys.path.insert(0, os.path.join(args.reference, "src"))
            from decider.engine import fused_causal_conv1d_fn                     # engine.py:25-40
            fixture["y_reference_helper"] = fused_causal_conv1d_fn(
                xc.transpose(1, 2), conv.weight.squeeze(1), activation="silu").transpose(1, 2)
        # packed varlen: two requests concatenated; each is run on its own through the module.
        cu = torch.tensor([0, 23, T], dtype=torch.int32)
        xv = xc[:1]
        yv = torch.cat([F.silu(conv(xv[:, a:b].transpose(1, 2))[:, :, :b - a]).transpose(1, 2)
                        for a, b in ((0, 23), (23, T))], dim=1)
        fixture.update(x_varlen=xv, cu_seqlens=cu, y_varlen=yv)
    out["conv"] = fixture

    # 3. Gated delta rule: transformers' chunked torch path, with its recurrent form beside it.
    for name, (B, T, H, D) in {"delta_small": (1, 100, 2, 32), "delta_d128": (1, 130, 2, 128)}.items():
        q = torch.randn(B, T, H, D, generator=gen).bfloat16().float()
        k = torch.randn(B, T, H, D, generator=gen).bfloat16().float()
        v = (0.5 * torch.randn(B, T, H, D, generator=gen)).bfloat16().float()
        a = torch.randn(B, T, H, generator=gen)
        b = torch.randn(B, T, H, generator=gen)
        A_log = torch.log(torch.empty(H).uniform_(1, 16, generator=gen))
        dt_bias = 1.0 + 0.3 * torch.randn(H, generator=gen)
        beta = b.sigmoid()                                                   # [tf]:491
        g = -A_log.float().exp() * F.softplus(a.float() + dt_bias)           # [tf]:493
        o_chunk, s_chunk = mq.torch_chunk_gated_delta_rule(
            q, k, v, g=g, beta=beta, initial_state=None, output_final_state=True,
            use_qk_l2norm_in_kernel=True)
        o_rec, s_rec = mq.torch_recurrent_gated_delta_rule(
            q, k, v, g=g, beta=beta, initial_state=None, output_final_state=True,
            use_qk_l2norm_in_kernel=True)
        out[name] = dict(q=q, k=k, v=v, a=a, b=b, A_log=A_log, dt_bias=dt_bias, g=g, beta=beta,
                         o_chunk=o_chunk, state_chunk=s_chunk, o_recurrent=o_rec,
                         state_recurrent=s_rec)

    # 4. Gated RMSNorm (Qwen3_5RMSNormGated, [tf]:175-190).
    gn = mq.Qwen3_5RMSNormGated(128, eps=1e-6)
    with torch.no_grad():
        gn.weight.copy_(1.0 + 0.1 * torch.randn(128, generator=gen))
        o = torch.randn(40, 128, generator=gen)
        z = torch.randn(40, 128, generator=gen)
        out["gated_norm"] = dict(o=o, z=z, weight=gn.weight.detach().clone(), eps=1e-6, y=gn(o, z))

    # 5. Attention core (eager_attention_forward, [tf]:594-617) at head_dim 128, GQA 16/4.
    T = 48
    qa = torch.randn(1, 16, T, 128, generator=gen)
    ka = torch.randn(1, 4, T, 128, generator=gen)
    va = torch.randn(1, 4, T, 128, generator=gen)

    class _M:  # eager_attention_forward only reads these attributes
        num_key_value_groups = 4
        training = False
    mask = torch.full((T, T), float("-inf")).triu(1)[None, None]
    with torch.no_grad():
        attn, _ = mq.eager_attention_forward(_M(), qa, ka, va, mask, scaling=128 ** -0.5)
    out["attention"] = dict(q=qa, k=ka, v=va, o=attn)                     # o: [1, T, 16, 128]

    # 6. Whole small model (4 layers L,L,L,F): last hidden state, two requests run separately.
    cfg = small_text_config()
    torch.manual_seed(17)
    model = mq.Qwen3_5TextModel(cfg).eval()
    perturb_norms(model, gen)
    ids_a = torch.randint(0, cfg.vocab_size, (1, 40), generator=gen)
    ids_b = torch.randint(0, cfg.vocab_size, (1, 29), generator=gen)
    with torch.no_grad():
        ha = model(input_ids=ids_a, use_cache=False).last_hidden_state
        hb = model(input_ids=ids_b, use_cache=False).last_hidden_state
    out["model_small"] = dict(cfg=cfg_dict(cfg), state_dict={k: v.clone() for k, v in model.state_dict().items()},
                              ids_a=ids_a, ids_b=ids_b, hidden_a=ha, hidden_b=hb)

    path = os.path.join(HERE, "golden_v1.pt")
    torch.save(out, path)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
