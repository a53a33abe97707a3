"""Pin the CPU oracle to the reference's own arithmetic (transformers 5.5.0 Qwen3.5 modules).

The fixtures in ``tests/golden/golden_v1.pt`` were produced by ``tests/golden/make_golden.py``
running the real modules; these tests run without a GPU.
"""
import torch

from oracle import ops
from oracle import model as omodel


def close(a, b, atol=1e-5, rtol=1e-5):
    torch.testing.assert_close(a.float(), b.float(), atol=atol, rtol=rtol)


def test_fixture_version(golden):
    assert golden["transformers_version"] == "5.5.0"


def test_residual_rmsnorm(golden):
    f = golden["rmsnorm"]
    normed, summed = ops.residual_rmsnorm(f["x"], f["residual"], f["weight"], f["eps"])
    close(summed, f["summed"], 0, 0)
    close(normed, f["normed"])


def test_packed_conv_dense_and_reference_helper(golden):
    f = golden["conv"]
    C = f["x"].shape[-1]
    q, k, v = ops.packed_conv_silu(f["x"], f["weight"], head_dim=32)
    y = torch.cat([t.reshape(*t.shape[:2], -1) for t in (q, k, v)], dim=-1)
    close(y, f["y_module"])
    if "y_reference_helper" in f:
        close(y, f["y_reference_helper"])
    assert y.shape[-1] == C


def test_packed_conv_varlen(golden):
    f = golden["conv"]
    q, k, v = ops.packed_conv_silu(f["x_varlen"], f["weight"], cu_seqlens=f["cu_seqlens"], head_dim=32)
    y = torch.cat([t.reshape(*t.shape[:2], -1) for t in (q, k, v)], dim=-1)
    close(y, f["y_varlen"])


def test_gates(golden):
    f = golden["delta_small"]
    g, beta = ops.gdn_gates(f["a"], f["b"], f["A_log"], f["dt_bias"])
    close(g, f["g"])
    close(beta, f["beta"])


def test_chunk_delta_rule_matches_transformers(golden):
    for name in ("delta_small", "delta_d128"):
        f = golden[name]
        o, st = ops.chunk_gated_delta_rule(f["q"], f["k"], f["v"], f["g"], f["beta"],
                                           output_final_state=True)
        close(o, f["o_chunk"], 2e-5, 2e-5)
        close(st[0], f["state_chunk"][0], 2e-5, 2e-5)


def test_chunk_matches_recurrent(golden):
    for name in ("delta_small", "delta_d128"):
        f = golden[name]
        o = ops.recurrent_gated_delta_rule(f["q"], f["k"], f["v"], f["g"], f["beta"])
        close(o, f["o_recurrent"], 2e-5, 2e-5)
        close(o, f["o_chunk"], 1e-4, 1e-4)


def test_delta_rule_varlen_equals_separate_runs(golden):
    f = golden["delta_small"]
    cu = torch.tensor([0, 37, 100])
    o, _ = ops.chunk_gated_delta_rule(f["q"], f["k"], f["v"], f["g"], f["beta"], cu_seqlens=cu)
    for a, b in ((0, 37), (37, 100)):
        ref, _ = ops.chunk_gated_delta_rule(f["q"][:, a:b], f["k"][:, a:b], f["v"][:, a:b],
                                            f["g"][:, a:b], f["beta"][:, a:b])
        close(o[:, a:b], ref, 1e-6, 1e-6)


def test_gated_rmsnorm(golden):
    f = golden["gated_norm"]
    close(ops.gated_rmsnorm(f["o"], f["z"], f["weight"], f["eps"]), f["y"])


def test_attention(golden):
    f = golden["attention"]
    q = f["q"][0].transpose(0, 1)
    k = f["k"][0].transpose(0, 1)
    v = f["v"][0].transpose(0, 1)
    o = ops.gqa_attention_varlen(q, k, v)
    close(o, f["o"][0], 2e-5, 2e-5)


def test_small_model_forward(golden):
    f = golden["model_small"]
    cfg, sd = f["cfg"], f["state_dict"]
    for ids, want in ((f["ids_a"], f["hidden_a"]), (f["ids_b"], f["hidden_b"])):
        h = omodel.forward_hidden(cfg, sd, ids[0])
        hn = ops.rmsnorm_offset(h, sd["norm.weight"], cfg["rms_norm_eps"])
        close(hn, want[0], 1e-4, 1e-4)


def test_small_model_packed_varlen(golden):
    f = golden["model_small"]
    cfg, sd = f["cfg"], f["state_dict"]
    ids = torch.cat([f["ids_a"][0], f["ids_b"][0]])
    la = f["ids_a"].shape[1]
    cu = torch.tensor([0, la, ids.numel()])
    h = omodel.forward_hidden(cfg, sd, ids, cu)
    hn = ops.rmsnorm_offset(h, sd["norm.weight"], cfg["rms_norm_eps"])
    close(hn[:la], f["hidden_a"][0], 1e-4, 1e-4)
    close(hn[la:], f["hidden_b"][0], 1e-4, 1e-4)
