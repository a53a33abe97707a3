"""Host-side logic on the CPU: request packing, batch planning, the seeded workloads, the work
model used for rooflines and load balancing, and the reference-style installers (no GPU, no
kernel launches)."""
import numpy as np
import pytest
import torch

from fastdecisions_b200.engine import MAX_REQUEST_TOKENS, pack, plan_batches
from fastdecisions_b200.workloads import ModelConfig, Request, config4_request, config5_requests


def _req(n, slot=None, nopts=4, base=0):
    return Request(ids=(np.arange(n, dtype=np.int32) + base), slot=n - 1 if slot is None else slot, nopts=nopts)


def test_pack_offsets_positions_and_slots():
    reqs = [_req(3, base=100), _req(1, base=200), _req(5, slot=2, nopts=8, base=300)]
    b = pack(reqs)
    assert b.cu_seqlens.tolist() == [0, 3, 4, 9]
    assert b.ids.tolist() == [100, 101, 102, 200, 300, 301, 302, 303, 304]
    assert b.positions.tolist() == [0, 1, 2, 0, 0, 1, 2, 3, 4]  # restart per request
    assert b.slots.tolist() == [2, 3, 6]                         # absolute rows
    assert b.nopts.tolist() == [4, 4, 8]
    assert b.max_seqlen == 5 and b.tokens == 9 and b.num_segments == 3
    assert b.ids.dtype == np.int32 and b.cu_seqlens.dtype == np.int32 and b.positions.dtype == np.int32


@pytest.mark.parametrize("bad", [
    [_req(0)],                                       # empty request
    [_req(4, slot=4)],                               # slot past the end
    [_req(4, slot=-1)],                              # negative slot
    [_req(MAX_REQUEST_TOKENS + 1)],                  # longer than a request may be
])
def test_pack_rejects_bad_requests(bad):
    with pytest.raises(ValueError):
        pack(bad)


def test_plan_batches_covers_every_request_within_budget():
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(1, 9000, size=300)]
    budget = 32768
    plan = plan_batches(lens, budget)
    flat = [i for b in plan for i in b]
    assert sorted(flat) == list(range(len(lens)))                       # each request exactly once
    for b in plan:
        assert sum(lens[i] for i in b) <= budget or len(b) == 1          # oversize only when alone
    assert [lens[i] for i in flat] == sorted(lens, reverse=True)         # longest first
    assert plan == plan_batches(lens, budget)                            # deterministic


def test_plan_batches_oversized_request_alone():
    plan = plan_batches([50, 10, 40], 45)
    assert plan == [[0], [2], [1]]


def test_config5_requests_are_seeded_and_prefix_stable():
    a = config5_requests(256)
    b = config5_requests(512)
    assert len(a) == 256 and len(b) == 512
    for x, y in zip(a, b[:256]):  # weak scaling: rank 0's share is the same request set
        assert np.array_equal(x.ids, y.ids) and x.slot == y.slot and x.nopts == y.nopts
    lens = np.array([r.ids.size for r in b])
    assert lens.min() >= 64 and lens.max() <= 8192
    assert 500 < np.median(lens) < 1200                                  # lognormal, median ~800
    assert all(2 <= r.nopts <= 8 and r.slot == r.ids.size - 1 for r in b)
    assert not np.array_equal(b[0].ids[:64], b[256].ids[:64])           # the second block is new


def test_config4_request():
    r = config4_request()
    assert r.ids.size == 1536 and r.slot == 1535 and r.nopts == 4
    assert np.array_equal(r.ids, config4_request().ids)
    assert r.ids.min() >= 0 and r.ids.max() < 151936


def test_work_model_matches_the_config4_figures():
    cfg = ModelConfig()
    assert cfg.linear_params() == 1_372_717_056
    assert cfg.layer_types.count("full_attention") == 6 and cfg.layer_types.count("linear_attention") == 18
    f = cfg.request_flops(1536)
    assert abs(f - 4.36e12) / 4.36e12 < 0.01                             # GEMMs + attention + delta rule
    # attention grows quadratically, the rest linearly
    assert cfg.request_flops(4096) - 2 * cfg.request_flops(2048) > 0


def _tiny_cpu_model():
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    cfg = ModelConfig(vocab_size=64, hidden_size=64, num_hidden_layers=8, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, linear_num_key_heads=2, linear_num_value_heads=2,
                      linear_key_head_dim=16, linear_value_head_dim=16, intermediate_size=96)
    torch.manual_seed(0)
    return mq.Qwen3_5TextModel(cfg.to_transformers())


def test_installers_count_and_are_idempotent():
    from fastdecisions_b200 import patches
    model = _tiny_cpu_model()
    gdn = [m for m in model.modules() if type(m).__name__ == "Qwen3_5GatedDeltaNet"]
    att = [m for m in model.modules() if type(m).__name__ == "Qwen3_5Attention"]
    assert len(gdn) == 6 and len(att) == 2
    first = patches.install_all(model)
    assert first == {"packed_conv": 6, "native_gqa": 2, "residual_rms": 8}
    originals = [m._packed_original_forward for m in gdn]
    second = patches.install_all(model)                                  # idempotent: same counts,
    assert second == first                                               # originals kept, not re-wrapped
    assert [m._packed_original_forward for m in gdn] == originals
    assert all(m.forward.__func__ is patches._gdn_forward for m in gdn)
    assert all(m.forward.__func__ is patches._attn_forward for m in att)
    assert patches.install_chunk_gated_delta_rule(model) == 6
