"""Answer-probability parity of the decision forward against the reference's float32 path.

    python -m fastdecisions_b200.paritybench [--requests 64] [--out parity.md]

On one GPU, for the first ``--requests`` requests of the config-5 mix plus the config-4 request
(synthetic weights from seed 17), this compares with the reference's own float32 forward --
transformers 5.5.0 ``Qwen3_5TextModel`` (the module the reference's engine calls) with its torch
paths (chunked delta rule, conv1d, eager attention), TF32 off, on the GPU -- the answer
probabilities of:

* this engine (``DecisionEngine``), residual stream in float32 (the default) and in bf16;
* the reference's own bf16 GPU path (the same transformers module in bf16, with fla's Triton
  delta rule where fla imports, as the reference runs it);
* the float32 reference with ONE group of bf16 rounding points switched on at a time (an
  ablation that names which storage point produces the drift): the residual stream after every
  add ([tf]:775,781), the inputs of every linear layer (norm / gated-norm / SwiGLU / gated
  attention outputs), the outputs of every linear layer, the token mixers' internals (conv output
  into the delta rule, delta-rule output, attention q / k / v and output), and all of them.

Readout as the reference's engine (model.py:18-27, engine.py:48-56): final-normed hidden state at
the slot times the candidate rows, options past ``nopts`` masked, softmax.  Prints a JSON summary
and writes a Markdown table.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import types

import numpy as np
import torch

from . import workloads as W

BF = torch.bfloat16


def _rnd(t):
    return t.to(BF).to(t.dtype) if torch.is_tensor(t) and t.is_floating_point() else t


def reference_model(cfg, weights, dtype, dev, fast_paths: bool):
    """transformers Qwen3_5TextModel with the given weights.  ``fast_paths=False`` builds it with
    the torch implementations (the reference's CPU / fallback path); True keeps whatever fast
    kernels the environment binds (fla on a GPU host)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    names = ("FusedRMSNormGated", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule", "causal_conv1d_fn",
             "causal_conv1d_update")
    saved = {n: getattr(mq, n) for n in names}
    old = torch.get_default_dtype()
    try:
        if not fast_paths:
            for n in names:
                setattr(mq, n, None)
        torch.set_default_dtype(dtype)
        with torch.device(dev):
            model = mq.Qwen3_5TextModel(cfg.to_transformers())
    finally:
        torch.set_default_dtype(old)
        for n, v in saved.items():
            setattr(mq, n, v)
    model.load_state_dict({k: v.to(dtype) for k, v in weights.items()}, strict=True)
    for i, kind in enumerate(cfg.layer_types):  # gate parameters stay float32, as in the checkpoint
        if kind == "linear_attention":
            la = model.layers[i].linear_attn
            la.A_log.data = weights[f"layers.{i}.linear_attn.A_log"].float().to(dev)
            la.dt_bias.data = weights[f"layers.{i}.linear_attn.dt_bias"].float().to(dev)
    return model.eval()


@contextlib.contextmanager
def rounding(model, groups: set):
    """Round to bf16 at the storage points of ``groups`` (subset of residual, linear_in, linear_out,
    mixer) inside a float32 model, restoring it on exit."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    handles, patched = [], []
    if "linear_in" in groups or "linear_out" in groups:
        for m in model.modules():
            if isinstance(m, torch.nn.Linear):
                if "linear_in" in groups:
                    handles.append(m.register_forward_pre_hook(lambda mod, args: tuple(_rnd(a) for a in args)))
                if "linear_out" in groups:
                    handles.append(m.register_forward_hook(lambda mod, args, out: _rnd(out)))
    if "residual" in groups:
        def layer_forward(self, hidden_states, position_embeddings, attention_mask=None, position_ids=None,
                          past_key_values=None, **kwargs):  # [tf]:744-783 with both adds rounded
            residual = hidden_states
            h = self.input_layernorm(hidden_states)
            if self.layer_type == "linear_attention":
                h = self.linear_attn(hidden_states=h, cache_params=None, attention_mask=attention_mask)
            else:
                h, _ = self.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                                      past_key_values=None, position_embeddings=position_embeddings, **kwargs)
            h = _rnd(residual + h)
            return _rnd(h + self.mlp(self.post_attention_layernorm(h)))
        for lay in model.layers:
            patched.append((lay, "forward", lay.forward))
            lay.forward = types.MethodType(layer_forward, lay)
    if "mixer" in groups:
        for m in model.modules():
            if isinstance(m, mq.Qwen3_5GatedDeltaNet):
                inner = m.chunk_gated_delta_rule

                def delta(q, k, v, g=None, beta=None, _inner=inner, **kw):
                    o, st = _inner(_rnd(q), _rnd(k), _rnd(v), g=g, beta=_rnd(beta), **kw)
                    return _rnd(o), st
                patched.append((m, "chunk_gated_delta_rule", inner))
                m.chunk_gated_delta_rule = delta
        eager = mq.eager_attention_forward

        def attn(module, q, k, v, *a, **kw):
            o, w = eager(module, _rnd(q), _rnd(k), _rnd(v), *a, **kw)
            return _rnd(o), w
        patched.append((mq, "eager_attention_forward", eager))
        mq.eager_attention_forward = attn
    try:
        yield
    finally:
        for h in handles:
            h.remove()
        for obj, name, val in reversed(patched):
            setattr(obj, name, val)


@torch.no_grad()
def reference_probs(model, reqs, letters, dev):
    out = []
    for r in reqs:
        hs = model(input_ids=torch.tensor(r.ids[None].astype(np.int64), device=dev), use_cache=False).last_hidden_state
        lg = hs[0, r.slot].float() @ letters.t()
        lg = lg.masked_fill(torch.arange(letters.shape[0], device=dev) >= r.nopts, float("-inf"))
        out.append(torch.softmax(lg, -1).cpu().numpy())
    return np.stack(out)


def summarize(p, ref, margin_pp=5.0):
    dp = np.abs(p - ref).max(1) * 100
    top2 = np.sort(ref, 1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) * 100 >= margin_pp
    same = p.argmax(1) == ref.argmax(1)
    return {"mean_dp_pp": round(float(dp.mean()), 3), "median_dp_pp": round(float(np.median(dp)), 3),
            "max_dp_pp": round(float(dp.max()), 3), "argmax_agree": int(same.sum()), "n": int(len(dp)),
            "flips_on_clear": int((~same & clear).sum()), "clear": int(clear.sum())}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--out", default=None, help="write the Markdown report here")
    args = ap.parse_args(argv)
    from .engine import DecisionEngine
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    dev = torch.device("cuda")
    cfg = W.ModelConfig()
    weights = W.synthetic_weights(cfg)
    reqs = W.config5_requests(256)[:args.requests] + [W.config4_request()]
    names = [f"c5[{i}]" for i in range(args.requests)] + ["config 4"]
    letters = W.letter_weight(weights).float().to(dev)

    ref32 = reference_model(cfg, weights, torch.float32, dev, fast_paths=False)
    want = reference_probs(ref32, reqs, letters, dev)
    results = {}
    ablations = [("residual",), ("linear_in",), ("linear_out",), ("mixer",),
                 ("linear_in", "linear_out", "mixer"), ("residual", "linear_in", "linear_out", "mixer")]
    abl = {}
    for groups in ablations:
        with rounding(ref32, set(groups)):
            abl["+".join(groups)] = reference_probs(ref32, reqs, letters, dev)
    del ref32
    torch.cuda.empty_cache()

    per = {}
    for label, fp32res in (("engine (fp32 residual)", True), ("engine (bf16 residual)", False)):
        eng = DecisionEngine(cfg, weights, dev, residual_fp32=fp32res)
        per[label] = eng.score(reqs)
        del eng
        torch.cuda.empty_cache()
    ref16 = reference_model(cfg, weights, BF, dev, fast_paths=True)
    per["reference bf16 GPU path"] = reference_probs(ref16, reqs, letters, dev)
    del ref16
    for k, v in abl.items():
        per[f"fp32 reference, bf16 at: {k}"] = v
    for k, v in per.items():
        results[k] = summarize(v, want)
    print(json.dumps(results), flush=True)

    if args.out:
        lens = [r.ids.size for r in reqs]
        lines = ["| path | mean abs dp (pp) | median | max | argmax same | flips where fp32 margin >= 5 pp |",
                 "|---|---|---|---|---|---|"]
        for k, s in results.items():
            lines.append(f"| {k} | {s['mean_dp_pp']} | {s['median_dp_pp']} | {s['max_dp_pp']} | "
                         f"{s['argmax_agree']}/{s['n']} | {s['flips_on_clear']} of {s['clear']} |")
        main_keys = ["engine (fp32 residual)", "engine (bf16 residual)", "reference bf16 GPU path"]
        rows = ["| request | tokens | fp32 top-1 margin (pp) | " + " | ".join(f"{k}: dp (pp) / argmax" for k in main_keys) + " |",
                "|---" * (3 + len(main_keys)) + "|"]
        top2 = np.sort(want, 1)[:, -2:]
        for i, nm in enumerate(names):
            cells = []
            for k in main_keys:
                d = np.abs(per[k][i] - want[i]).max() * 100
                cells.append(f"{d:.2f} / {'=' if per[k][i].argmax() == want[i].argmax() else 'FLIP'}")
            rows.append(f"| {nm} | {lens[i]} | {(top2[i, 1] - top2[i, 0]) * 100:.2f} | " + " | ".join(cells) + " |")
        with open(args.out, "w") as f:
            f.write("\n".join(lines) + "\n\n" + "\n".join(rows) + "\n")


if __name__ == "__main__":
    main()
