"""GPU parity of each CUDA kernel against the CPU oracle (called through the C ABI).

Tolerances are the reference's own (experiments/*): packed conv rtol .008 / atol .002
(check_packed_output_conv.py:45), residual RMSNorm rtol .008 / atol .002
(bench_persistent_residual_rms.py:47), gates (bench_unpack_gate.py:36-38), plus the
north-star bound of max-abs 2e-2 against the float32 oracle for every bf16 kernel output.
"""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from fastdecisions_b200 import _lib, ops

MAX_ABS = 2e-2


def gen(seed=17):
    return torch.Generator().manual_seed(seed)


def dev(t):
    return t.to("cuda")


def max_abs(a, b):
    return (a.float().cpu() - b.float().cpu()).abs().max().item()


# --------------------------------------------------------------------------- residual RMSNorm
def test_residual_rmsnorm_config1():
    g = gen()
    x = torch.randn(1, 1024, 2048, generator=g)
    r = torch.randn(1, 1024, 2048, generator=g)
    w = 1.0 + 0.02 * torch.randn(2048, generator=g)
    xb, rb = x.bfloat16(), r.bfloat16()
    normed, summed = ops.residual_rmsnorm(dev(xb), dev(rb), dev(w.bfloat16()))
    want_s = (xb.float() + rb.float()).bfloat16()
    assert torch.equal(summed.cpu(), want_s), "updated residual must be bf16(x + r) exactly"
    ref_n, _ = O.residual_rmsnorm(xb, rb, w.bfloat16(), 1e-6, sum_dtype=torch.bfloat16)
    torch.testing.assert_close(normed.cpu().float(), ref_n, rtol=0.008, atol=0.002)
    # against the fp32 oracle of config 1 (fp32 inputs, no bf16 rounding anywhere)
    ref32, _ = O.residual_rmsnorm(x, r, w, 1e-6)
    assert max_abs(normed, ref32) < 4 * MAX_ABS  # |out| reaches ~8: bf16 input+output rounding


def test_residual_rmsnorm_golden_and_variants(golden):
    f = golden["rmsnorm"]
    n, s = ops.residual_rmsnorm(dev(f["x"].bfloat16()), dev(f["residual"].bfloat16()), dev(f["weight"].float()))
    torch.testing.assert_close(n.cpu().float(), f["normed"], rtol=0.02, atol=0.05)
    # no residual, fp32 weight, odd row count, strided rows
    x = torch.randn(37, 3000, generator=gen(3))[:, :2048].bfloat16()
    w = torch.randn(2048, generator=gen(4)) * 0.1
    n, s = ops.residual_rmsnorm(dev(x), None, dev(w))
    torch.testing.assert_close(n.cpu().float(), O.rmsnorm_offset(x, w), rtol=0.008, atol=0.002)
    assert torch.equal(s.cpu(), x)
    # the reference's one-output op
    a = dev(torch.randn(2, 5, 2048, generator=gen(5)).bfloat16())
    b = dev(torch.randn(2, 5, 2048, generator=gen(6)).bfloat16())
    out = torch.ops.fastdecisions.residual_rms(a, b, dev(w.bfloat16()))
    ref, _ = O.residual_rmsnorm(a.cpu(), b.cpu(), w.bfloat16(), sum_dtype=torch.bfloat16)
    torch.testing.assert_close(out.cpu().float(), ref, rtol=0.008, atol=0.002)


def test_residual_rmsnorm_rejects_bad_input():
    w = dev(torch.zeros(2048, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.residual_rmsnorm(dev(torch.zeros(4, 2048)), None, w)          # fp32 input
    with pytest.raises(ValueError):
        ops.residual_rmsnorm(dev(torch.zeros(4, 2048, dtype=torch.bfloat16)),
                             dev(torch.zeros(4, 1024, dtype=torch.bfloat16)), w)


# --------------------------------------------------------------------------- packed conv
def conv_ref(x, w, cu=None):
    q, k, v = O.packed_conv_silu(x, w, cu_seqlens=cu)
    return q, k, v


def conv_compare(got, want):
    for name, a, b in zip("qkv", got, want):
        a = a.cpu().float()
        assert a.shape == b.shape, name
        assert torch.isfinite(a).all(), name
        torch.testing.assert_close(a, b.reshape(a.shape), rtol=0.008, atol=0.002, msg=lambda m: f"{name}: {m}")


def test_packed_conv_config2():
    g = gen()
    x = torch.randn(1, 2048, 6144, generator=g).bfloat16()
    w = (0.5 * torch.randn(6144, 4, generator=g)).bfloat16()
    got = torch.ops.fastdecisions.packed_conv(dev(x), dev(w))
    conv_compare(got, conv_ref(x, w))
    assert all(t.shape == (1, 2048, 16, 128) and t.is_contiguous() for t in got)


@pytest.mark.parametrize("batch", [1, 2, 4])
@pytest.mark.parametrize("wshape", [(6144, 4), (6144, 1, 4)])
def test_packed_conv_batches_and_weight_shapes(batch, wshape):
    g = gen(batch)
    x = (torch.randn(batch, 333, 6144, generator=g) * 0.5).bfloat16()
    w = (torch.randn(wshape, generator=g) * 0.25).bfloat16()
    conv_compare(ops.packed_conv_qkv(dev(x), dev(w)), conv_ref(x, w))


def test_packed_conv_each_tap_and_batch_boundaries():
    # distinct per-batch / per-region constants; the poisoned tail of batch 0 must not leak
    x = torch.empty(2, 2048, 6144)
    for b in range(2):
        for region in range(3):
            x[b, :, region * 2048:(region + 1) * 2048] = (b * 3 + region + 1) / 8
    x[0, -3:, :] = 3
    x = x.bfloat16()
    for tap in range(4):
        w = torch.zeros(6144, 4)
        w[:, tap] = 1
        w = w.bfloat16()
        conv_compare(ops.packed_conv_qkv(dev(x), dev(w)), conv_ref(x, w))


def test_packed_conv_zero_input():
    x = torch.zeros(1, 2048, 6144, dtype=torch.bfloat16)
    w = torch.randn(6144, 4, generator=gen()).bfloat16()
    for t in ops.packed_conv_qkv(dev(x), dev(w)):
        assert torch.count_nonzero(t).item() == 0


def test_packed_conv_varlen_and_strided_input():
    g = gen(9)
    lens = [1, 2, 3, 5, 64, 100, 17]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    big = torch.randn(1, T, 6144 + 2080, generator=g).bfloat16()   # fused-projection row stride
    x = big[..., :6144]
    w = torch.randn(6144, 4, generator=g).bfloat16()
    got = ops.packed_conv_qkv(dev(big)[..., :6144], dev(w), cu_seqlens=dev(cu))
    conv_compare(got, conv_ref(x, w, cu))


# up to 8192 tokens the direct kernel runs; above it the shared-memory staged kernel (1-4 tiles a CTA)
@pytest.mark.parametrize("lens", [[1500, 900, 700], [4000, 1, 1999, 64], [5000, 1, 3000, 4100, 63],
                                  [8192, 4000, 2]])
def test_packed_conv_tiles_per_cta(lens):
    g = gen(21)
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    x = (torch.randn(1, T, 6144, generator=g) * 0.5).bfloat16()
    w = (torch.randn(6144, 4, generator=g) * 0.25).bfloat16()
    got = ops.packed_conv_qkv(dev(x), dev(w), cu_seqlens=dev(cu))
    conv_compare(got, conv_ref(x, w, cu))


@pytest.mark.parametrize("T", [300, 9000])
@pytest.mark.parametrize("width", [1, 2, 3])
def test_packed_conv_narrow_kernels(T, width):
    # causal conv widths below 4 (the C ABI takes 1-4), through both kernels
    g = gen(40 + width)
    x = (torch.randn(1, T, 6144, generator=g) * 0.5).bfloat16()
    w = (torch.randn(6144, width, generator=g) * 0.4).bfloat16()
    conv_compare(ops.packed_conv_qkv(dev(x), dev(w)), conv_ref(x, w))


def test_packed_conv_dense_batch_above_direct_threshold():
    g = gen(23)
    x = (torch.randn(5, 2000, 6144, generator=g) * 0.5).bfloat16()
    w = (torch.randn(6144, 4, generator=g) * 0.25).bfloat16()
    conv_compare(ops.packed_conv_qkv(dev(x), dev(w)), conv_ref(x, w))


def test_packed_conv_golden(golden):
    f = golden["conv"]
    x, w = f["x"], f["weight"]
    got = ops.packed_conv_qkv(dev(x.bfloat16()), dev(w.bfloat16()), key_dim=32, value_dim=32, head_dim=32)
    y = torch.cat([t.reshape(*t.shape[:2], -1).cpu().float() for t in got], -1)
    assert max_abs(y, f["y_module"]) < MAX_ABS * 2


def test_packed_conv_cuda_graph_replay():
    g = gen(11)
    x = dev((torch.randn(1, 2048, 6144, generator=g) * 0.5).bfloat16())
    w = dev((torch.randn(6144, 4, generator=g) * 0.25).bfloat16())
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            ops.packed_conv_qkv(x, w)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = ops.packed_conv_qkv(x, w)
    x.copy_(dev((torch.randn(1, 2048, 6144, generator=g) * 0.5).bfloat16()))
    graph.replay()
    torch.cuda.synchronize()
    conv_compare(outs, conv_ref(x.cpu(), w.cpu()))


# --------------------------------------------------------------------------- gates, norms, misc
def test_gdn_gates():
    g = gen()
    ab = torch.randn(2, 50, 32, generator=g).bfloat16()
    A_log = torch.log(torch.empty(16).uniform_(1, 16, generator=g))
    dt = 1.0 + 0.3 * torch.randn(16, generator=g)
    gg, beta = torch.ops.fastdecisions.unpack_gate(dev(ab), dev(A_log), dev(dt))
    rg, rb = O.gdn_gates(ab[..., :16], ab[..., 16:], A_log, dt)
    torch.testing.assert_close(gg.cpu(), rg, rtol=0.02, atol=0.002)
    torch.testing.assert_close(beta.cpu().float(), rb, rtol=0.008, atol=0.001)


def test_gated_rmsnorm():
    g = gen()
    o = torch.randn(77, 16, 128, generator=g).bfloat16()
    zbig = torch.randn(77, 16 * 128 + 64, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(128, generator=g)).bfloat16()
    got = ops.gated_rmsnorm(dev(o), dev(zbig)[:, :2048], dev(w))
    ref = O.gated_rmsnorm(o, zbig[:, :2048].reshape(77, 16, 128), w).reshape(77, 2048)
    torch.testing.assert_close(got.cpu().float(), ref, rtol=0.008, atol=0.002)


def test_gated_rmsnorm_golden(golden):
    f = golden["gated_norm"]
    got = ops.gated_rmsnorm(dev(f["o"].bfloat16()).reshape(40, 1, 128), dev(f["z"].bfloat16()), dev(f["weight"].float()))
    # the fixture's float32 inputs are rounded to bf16 here (relative 2^-9 each), outputs reach ~10
    torch.testing.assert_close(got.cpu().float(), f["y"], rtol=0.016, atol=0.004)


@pytest.mark.parametrize("D", [128, 256])
def test_attn_qk_norm_rope(D):
    g = gen(D)
    T, hq, hkv = 45, 16, 4
    qkv = torch.randn(T, (2 * hq + 2 * hkv) * D, generator=g).bfloat16()
    qw = (0.1 * torch.randn(D, generator=g)).bfloat16()
    kw = (0.1 * torch.randn(D, generator=g)).bfloat16()
    pos = torch.cat([torch.arange(20), torch.arange(25)]).int()
    inv = ops.rope_inv_freq(D)
    q, k = ops.attn_qk_norm_rope(dev(qkv), dev(qw), dev(kw), dev(pos), ops.rope_table(dev(inv), 64), hq, hkv, D)
    qg = qkv[:, :2 * hq * D].reshape(T, hq, 2 * D)
    qr = O.rmsnorm_offset(qg[..., :D], qw)
    kr = O.rmsnorm_offset(qkv[:, 2 * hq * D:2 * hq * D + hkv * D].reshape(T, hkv, D), kw)
    cos, sin = O.rope_cos_sin(pos, D)
    torch.testing.assert_close(q.cpu().float(), O.apply_partial_rope(qr, cos, sin), rtol=0.008, atol=0.004)
    torch.testing.assert_close(k.cpu().float(), O.apply_partial_rope(kr, cos, sin), rtol=0.008, atol=0.004)


def test_embed_swiglu_readout():
    g = gen()
    table = torch.randn(1000, 2048, generator=g).bfloat16()
    ids = torch.randint(0, 1000, (33,), generator=g)
    h = ops.embed(dev(ids), dev(table))
    assert torch.equal(h.cpu(), table[ids])
    gu = torch.randn(33, 2 * 6144, generator=g).bfloat16()
    act = ops.swiglu(dev(gu), 6144)
    torch.testing.assert_close(act.cpu().float(), O.swiglu(gu[:, :6144], gu[:, 6144:]), rtol=0.008, atol=0.002)
    fw = (0.02 * torch.randn(2048, generator=g)).bfloat16()
    letters = (0.02 * torch.randn(8, 2048, generator=g)).bfloat16()
    slots = torch.tensor([0, 5, 32], dtype=torch.int32)
    nopts = torch.tensor([2, 8, 4], dtype=torch.int32)
    p, lg = ops.slot_readout(dev(h), dev(slots), dev(nopts), dev(fw), dev(letters))
    rp, rl = O.slot_readout(h.cpu(), fw, letters, slots.long(), nopts.long())
    assert (p.cpu() - rp).abs().max().item() < 1e-3
    assert torch.equal(p.cpu().argmax(1), rp.argmax(1))
    assert (p.cpu()[0, 2:] == 0).all() and torch.isinf(lg.cpu()[0, 2:]).all()


# --------------------------------------------------------------------------- delta rule
def delta_inputs(T, H, seed, D=128):
    g = gen(seed)
    q = torch.randn(1, T, H, D, generator=g).bfloat16()
    k = torch.randn(1, T, H, D, generator=g).bfloat16()
    v = (0.5 * torch.randn(1, T, H, D, generator=g)).bfloat16()
    a = torch.randn(1, T, H, generator=g)
    b = torch.randn(1, T, H, generator=g)
    A_log = torch.log(torch.empty(H).uniform_(1, 16, generator=g))
    dt = 1.0 + 0.3 * torch.randn(H, generator=g)
    gg, beta = O.gdn_gates(a, b, A_log, dt)
    return q, k, v, gg, beta.bfloat16()


def delta_check(T, H, seed, cu=None, init=False):
    q, k, v, gg, beta = delta_inputs(T, H, seed)
    nseg = 1 if cu is None else len(cu) - 1
    st = torch.randn(nseg, H, 128, 128, generator=gen(seed + 1)) * 0.1 if init else None
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.int32)
    o, fs = ops.chunk_gated_delta_rule(dev(q), dev(k), dev(v), dev(gg), dev(beta),
                                       initial_state=None if st is None else dev(st),
                                       output_final_state=True, cu_seqlens=None if cu_t is None else dev(cu_t))
    ro, rs = O.chunk_gated_delta_rule(q, k, v, gg, beta.float(), initial_state=st, output_final_state=True,
                                      cu_seqlens=cu_t)
    err = max_abs(o, ro)
    scale = ro.abs().max().item()
    assert err < MAX_ABS, (err, scale)
    assert (fs.cpu() - rs).abs().max().item() < 5e-2 * max(1.0, rs.abs().max().item())
    return err


def test_delta_rule_single_segment():
    delta_check(200, 4, 1)


def test_delta_rule_exact_chunks_and_tail():
    delta_check(128, 2, 2)
    delta_check(65, 2, 3)
    delta_check(1, 2, 4)


def test_delta_rule_single_request_initial_state():
    # one request: prep and recurrence pipelined in one launch; initial and final states
    delta_check(700, 8, 12, init=True)


def test_delta_rule_varlen_segments():
    delta_check(300, 4, 5, cu=[0, 1, 64, 65, 129, 200, 200, 300])


def test_delta_rule_initial_state():
    delta_check(150, 2, 6, cu=[0, 70, 150], init=True)


def test_delta_rule_empty_segments_keep_initial_state():
    # empty segments at both ends: their final state is the initial state, untouched
    delta_check(150, 2, 8, cu=[0, 0, 150, 150], init=True)


def test_delta_rule_long_segment_many_heads():
    # 40 chunks per (segment, head) through the 2-stage tile ring, plus a ragged short segment
    delta_check(2600, 8, 9, cu=[0, 2560, 2600], init=True)


def test_delta_rule_many_chains_whole_chain_path():
    # 10 segments x 8 heads = 80 (segment, head) chains, more than half of the 148 SMs: each chain
    # runs whole on one CTA (M = 128); the tests above, with few chains, run every chain as two
    # 64-row halves on two CTAs (M = 64)
    lens = [100, 1, 64, 65, 130, 7, 200, 63, 128, 50]
    delta_check(sum(lens), 8, 10, cu=[0] + list(torch.tensor(lens).cumsum(0).tolist()), init=True)


def test_delta_rule_golden(golden):
    f = golden["delta_d128"]
    o, st = ops.chunk_gated_delta_rule(dev(f["q"].bfloat16()), dev(f["k"].bfloat16()), dev(f["v"].bfloat16()),
                                       dev(f["g"]), dev(f["beta"].bfloat16()), output_final_state=True)
    assert max_abs(o, f["o_chunk"]) < MAX_ABS


def test_delta_rule_config4_layer_shape():
    # one GDN layer of config 4: T = 1536, 16 heads x 128
    err = delta_check(1536, 16, 7)
    assert err < MAX_ABS


def test_delta_rule_rejects_cu_seqlens_beyond_tokens_on_the_device():
    """cu_seqlens lives on the device: the chunk-table kernel checks it (cu[0] == 0, non-decreasing,
    cu[-1] == tokens); a mismatch reports bit 8 of the error word and leaves every output untouched
    (no tile or output row past the tokens is touched)."""
    T, H = 100, 2
    g = gen(31)
    q = dev(torch.randn(1, T, H, 128, generator=g).bfloat16())
    k = dev(torch.randn(1, T, H, 128, generator=g).bfloat16())
    v = dev(torch.randn(1, T, H, 128, generator=g).bfloat16())
    gg = dev(-torch.rand(1, T, H, generator=g))
    beta = dev(torch.rand(1, T, H, generator=g).bfloat16())
    assert _lib.poll_device_error() == 0
    for cu in ([0, 60, 300], [0, 80, 40, 100], [5, 100]):
        out = torch.full((1, T, H, 128), 7.0, device="cuda", dtype=torch.bfloat16)
        fin = torch.full((len(cu) - 1, H, 128, 128), 3.0, device="cuda")
        ws = torch.empty(ops.delta_rule_workspace_bytes(T, len(cu) - 1, H), device="cuda", dtype=torch.uint8)
        _lib.call("fdk_chunk_gated_delta_rule_fwd", q.data_ptr(), k.data_ptr(), H * 128, v.data_ptr(), H * 128,
                  gg.data_ptr(), beta.data_ptr(), dev(torch.tensor(cu, dtype=torch.int32)).data_ptr(), len(cu) - 1,
                  T, H, 128, 128, 128 ** -0.5, None, out.data_ptr(), fin.data_ptr(), ws.data_ptr(), ws.numel(),
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert _lib.poll_device_error() == 8, cu
        assert (out.float() == 7.0).all()
        assert (fin == 0).all()  # every segment treated as empty: its final state is the (zero) initial state
    assert _lib.poll_device_error() == 0


# --------------------------------------------------------------------------- fused GDN prologue
def gdn_proj_inputs(lens, H, seed):
    g = gen(seed)
    T = sum(lens)
    kd = vd = H * 128
    C = 2 * kd + vd
    width = C + vd + 2 * H
    proj = torch.randn(T, width + (-width) % 8 + 8, generator=g).bfloat16()   # q k v | z | b | a | pad (16 B rows)
    conv = (0.5 * torch.randn(C, 4, generator=g)).bfloat16()
    A_log = torch.log(torch.empty(H).uniform_(1, 16, generator=g))
    dt = 1.0 + 0.3 * torch.randn(H, generator=g)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    return proj, conv, A_log, dt, cu, C, vd


@pytest.mark.parametrize("lens", [[200], [1, 2, 3, 64, 65, 130, 7], [1536]])
def test_gdn_fused_matches_separate_ops(lens):
    H = 4
    proj, conv, A_log, dt, cu, C, vd = gdn_proj_inputs(lens, H, 21)
    P, W, AL, DT, CU = dev(proj), dev(conv), dev(A_log), dev(dt), dev(cu)
    fused = ops.gdn_fused_delta_rule(P, W, AL, DT, H, C + vd + H, C + vd, CU)
    q, k, v = ops.packed_conv_qkv(P[:, :C].unsqueeze(0), W, H * 128, vd, 128, CU)
    gg, beta = ops.gdn_gates(P[:, C + vd + H:C + vd + 2 * H], P[:, C + vd:C + vd + H], AL, DT)
    sep, _ = ops.chunk_gated_delta_rule(q, k, v, gg.unsqueeze(0), beta.unsqueeze(0), cu_seqlens=CU)
    assert (fused.float() - sep[0].float()).abs().max().item() <= 1e-6
    assert _lib.poll_device_error() == 0


@pytest.mark.parametrize("H,lens", [(2, [100, 1, 70]), (16, [1536])])
def test_gdn_fused_against_oracle(H, lens):
    # (16, [1536]): one GDN layer of config 4 through the single-launch pipelined path
    proj, conv, A_log, dt, cu, C, vd = gdn_proj_inputs(lens, H, 22)
    fused = ops.gdn_fused_delta_rule(dev(proj), dev(conv), dev(A_log), dev(dt), H, C + vd + H, C + vd, dev(cu))
    q, k, v = O.packed_conv_silu(proj[:, :C].unsqueeze(0), conv, cu_seqlens=cu, key_dim=H * 128, value_dim=vd)
    gg, beta = O.gdn_gates(proj[:, C + vd + H:C + vd + 2 * H].float(), proj[:, C + vd:C + vd + H].float(), A_log, dt)
    ro, _ = O.chunk_gated_delta_rule(q.bfloat16().float(), k.bfloat16().float(), v.bfloat16().float(),
                                     gg.unsqueeze(0), beta.bfloat16().float().unsqueeze(0), cu_seqlens=cu)
    assert max_abs(fused.unsqueeze(0), ro) < MAX_ABS
