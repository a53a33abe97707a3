"""Native GQA attention (tcgen05) parity against the CPU oracle (per-segment fp32 softmax with
repeat_kv), at the reference's tolerance atol = rtol = 0.02 (experiments/native_gqa/
bench_native_gqa.py:60) and the north-star bound max-abs 2e-2."""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from fastdecisions_b200 import _lib, ops


def make(T, hq, hkv, seed, D=128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(T, hq, D, generator=g).bfloat16()
    k = torch.randn(T, hkv, D, generator=g).bfloat16()
    v = torch.randn(T, hkv, D, generator=g).bfloat16()
    return q, k, v


def run(q, k, v, lens, gate=None, gate_interleaved=False):
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    o = ops.gqa_attention_varlen_(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), max(lens) if lens else 0,
                                  gate=None if gate is None else gate.cuda(), gate_interleaved=gate_interleaved)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    return o.cpu().float(), cu


def check(o, ref):
    err = (o - ref).abs().max().item()
    torch.testing.assert_close(o, ref, atol=0.02, rtol=0.02)
    assert err < 2e-2, err
    return err


@pytest.mark.parametrize("lens", [[1], [5], [127], [128], [129], [300], [1, 255, 2, 130]])
def test_small_segments(lens):
    q, k, v = make(sum(lens), 16, 4, seed=len(lens) * 31 + lens[0])
    o, cu = run(q, k, v, lens)
    check(o, O.gqa_attention_varlen(q, k, v, cu))


def test_many_short_segments_two_head_path():
    # 40 segments x 8 head pairs x 3 query tiles fill the SMs: the two-heads-a-CTA kernel (the small
    # cases above run one head a CTA)
    lens = [300, 257, 129, 384] * 10
    q, k, v = make(sum(lens), 16, 4, seed=41)
    o, cu = run(q, k, v, lens)
    check(o, O.gqa_attention_varlen(q, k, v, cu))


def test_config3_varlen():
    # 4 requests, lengths uniform in [256, 4096] from seed 17
    g = torch.Generator().manual_seed(17)
    lens = torch.randint(256, 4097, (4,), generator=g).tolist()
    T = sum(lens)
    q = torch.randn(T, 16, 128, generator=g).bfloat16()
    k = torch.randn(T, 4, 128, generator=g).bfloat16()
    v = torch.randn(T, 4, 128, generator=g).bfloat16()
    o, cu = run(q, k, v, lens)
    check(o, O.gqa_attention_varlen(q, k, v, cu))


def test_heads_8_2_and_fused_gate():
    lens = [200, 77]
    q, k, v = make(sum(lens), 8, 2, seed=5)
    gate = torch.randn(sum(lens), 8 * 128, generator=torch.Generator().manual_seed(6)).bfloat16()
    o, cu = run(q, k, v, lens, gate=gate)
    ref = O.gqa_attention_varlen(q, k, v, cu) * torch.sigmoid(gate.float()).reshape(-1, 8, 128)
    check(o, ref)


def test_native_gqa_reference_signature():
    # logical [B, H, T, D] views of [B, T, H, D] storage, as the model's transpose(1, 2) produces
    B, T = 2, 190
    g = torch.Generator().manual_seed(8)
    q = torch.randn(B, T, 16, 128, generator=g).bfloat16().cuda().transpose(1, 2)
    k = torch.randn(B, T, 4, 128, generator=g).bfloat16().cuda().transpose(1, 2)
    v = torch.randn(B, T, 4, 128, generator=g).bfloat16().cuda().transpose(1, 2)
    out = torch.ops.fastdecisions.native_gqa(q, k, v)
    assert out.shape == (B, 16, T, 128)
    assert out.transpose(1, 2).is_contiguous()
    for b in range(B):
        ref = O.gqa_attention_varlen(q[b].transpose(0, 1).cpu(), k[b].transpose(0, 1).cpu(), v[b].transpose(0, 1).cpu())
        check(out[b].transpose(0, 1).cpu().float(), ref)


# ------------------------------------------------------------------ head_dim 256 (the reference's shape)
@pytest.mark.parametrize("lens", [[1], [63], [64], [65], [127], [128], [129], [300], [1, 255, 2, 130, 64]])
def test_d256_small_segments(lens):
    # 8 query / 2 KV heads of 256: the only shape native_gqa_kernel.py:132-133 accepts
    q, k, v = make(sum(lens), 8, 2, seed=len(lens) * 7 + lens[0], D=256)
    o, cu = run(q, k, v, lens)
    check(o, O.gqa_attention_varlen(q, k, v, cu))


def test_d256_long_varlen():
    # segments long enough for many KV blocks through the two-stage rings and lazy O rescales
    g = torch.Generator().manual_seed(19)
    lens = [2048, 700, 1537]
    T = sum(lens)
    q = torch.randn(T, 8, 256, generator=g).bfloat16()
    k = torch.randn(T, 2, 256, generator=g).bfloat16()
    v = torch.randn(T, 2, 256, generator=g).bfloat16()
    o, cu = run(q, k, v, lens)
    check(o, O.gqa_attention_varlen(q, k, v, cu))


def test_d256_other_head_ratios_and_interleaved_gate():
    lens = [150, 70]
    T = sum(lens)
    for hq, hkv in ((4, 4), (6, 2), (16, 2)):
        q, k, v = make(T, hq, hkv, seed=hq * 10 + hkv, D=256)
        gate = torch.randn(T, hq, 2, 256, generator=torch.Generator().manual_seed(hq)).bfloat16()
        o, cu = run(q, k, v, lens, gate=gate.reshape(T, -1)[:, 256:], gate_interleaved=True)
        ref = O.gqa_attention_varlen(q, k, v, cu) * torch.sigmoid(gate[:, :, 1].float())
        check(o, ref)


def test_d256_native_gqa_reference_signature():
    # native_gqa_attention at the reference's own shape: [B, 8, T, 256] / [B, 2, T, 256]
    B, T = 2, 333
    g = torch.Generator().manual_seed(12)
    q = torch.randn(B, T, 8, 256, generator=g).bfloat16().cuda().transpose(1, 2)
    k = torch.randn(B, T, 2, 256, generator=g).bfloat16().cuda().transpose(1, 2)
    v = torch.randn(B, T, 2, 256, generator=g).bfloat16().cuda().transpose(1, 2)
    out = ops.native_gqa_attention(q, k, v)
    assert out.shape == (B, 8, T, 256) and out.transpose(1, 2).is_contiguous()
    for b in range(B):
        ref = O.gqa_attention_varlen(q[b].transpose(0, 1).cpu(), k[b].transpose(0, 1).cpu(), v[b].transpose(0, 1).cpu())
        check(out[b].transpose(0, 1).cpu().float(), ref)


def test_rejects_bad_shapes():
    q, k, v = make(10, 16, 4, 1)
    cu = torch.tensor([0, 10], dtype=torch.int32).cuda()
    with pytest.raises(ValueError):
        ops.gqa_attention_varlen_(q.cuda(), k.cuda()[:, :3], v.cuda()[:, :3], cu, 10)
    with pytest.raises(ValueError):
        ops.gqa_attention_varlen_(q.cuda().float(), k.cuda(), v.cuda(), cu, 10)
    q6, k6, v6 = make(10, 16, 4, 1, D=64)
    with pytest.raises(ValueError, match="head_dim"):
        ops.gqa_attention_varlen_(q6.cuda(), k6.cuda(), v6.cuda(), cu, 10)
