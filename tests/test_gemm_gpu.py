"""The tcgen05 projection / MLP GEMM against a float32 PyTorch reference of the same op (and the
SwiGLU epilogue against the oracle's swiglu of [tf]:706-708), at the layer shapes of the decision
forward and ragged sizes."""
import pytest
import torch

from oracle import ops as O

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from fastdecisions_b200 import _lib, ops


def inputs(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).bfloat16()
    w = (0.02 * torch.randn(n, k, generator=g)).bfloat16()
    return a, w


def check(got, ref):
    # bf16 output of an fp32-accumulated product: within two bf16 ulps of the fp32 reference
    got = got.float().cpu()
    tol = 2.0 ** -7 * ref.abs() + 1e-3 * ref.abs().max().item()
    bad = (got - ref).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} outside tolerance, max err {(got - ref).abs().max():.3g}"


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (5, 8, 8), (127, 264, 72), (300, 2048, 2048), (1536, 8224, 2048),
                                   (1000, 5120, 2048), (777, 2048, 6144), (4097, 512, 128)])
def test_gemm_plain(m, n, k):
    a, w = inputs(m, n, k, m + n + k)
    got = ops.gemm(a.cuda(), w.cuda())
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    check(got, a.float() @ w.float().t())


@pytest.mark.parametrize("m,inter,k", [(1, 128, 64), (200, 256, 256), (1536, 6144, 2048), (333, 384, 136)])
def test_gemm_swiglu_epilogue(m, inter, k):
    a, gw = inputs(m, inter, k, 3 * m + k)
    uw = (0.02 * torch.randn(inter, k, generator=torch.Generator().manual_seed(m))).bfloat16()
    w = ops.interleave_gate_up(gw, uw)
    got = ops.gemm(a.cuda(), w.cuda(), ops.GEMM_SWIGLU)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    ref = O.swiglu(a.float() @ gw.float().t(), a.float() @ uw.float().t())
    check(got, ref)


def test_gemm_strided_rows_and_rejects():
    a, w = inputs(100, 256, 128, 7)
    big = torch.zeros(100, 200, dtype=torch.bfloat16)
    big[:, 40:168] = a
    out = torch.zeros(100, 264, dtype=torch.bfloat16, device="cuda")
    ops.gemm(big.cuda()[:, 40:168], w.cuda(), out=out[:, :256])
    check(out[:, :256], a.float() @ w.float().t())
    assert (out[:, 256:] == 0).all()
    with pytest.raises(ValueError):
        ops.gemm(a.cuda()[:, :100], w.cuda()[:, :100].contiguous()[:, :100], ops.GEMM_SWIGLU)  # k=100 % 8 != 0
    with pytest.raises(ValueError, match="multiple of 256"):
        ops.gemm(a.cuda(), w.cuda()[:136].contiguous(), ops.GEMM_SWIGLU)


@pytest.mark.parametrize("m,hq,hkv,D", [(45, 16, 4, 128), (300, 16, 4, 128), (1537, 16, 4, 128), (200, 8, 2, 256),
                                        (130, 6, 2, 128)])
def test_gemm_qk_norm_rope_epilogue(m, hq, hkv, D):
    """The attention projection with q / k RMSNorm (1 + w) and partial RoPE in the epilogue, against
    the oracle applied to the float32 product ([tf]:657-668)."""
    g = torch.Generator().manual_seed(m + D)
    k = 512
    n = (2 * hq + 2 * hkv) * D
    a = torch.randn(m, k, generator=g).bfloat16()
    w = (0.05 * torch.randn(n, k, generator=g)).bfloat16()
    qw = (0.1 * torch.randn(D, generator=g)).bfloat16()
    kw = (0.1 * torch.randn(D, generator=g)).bfloat16()
    pos = torch.cat([torch.arange(m // 2), torch.arange(m - m // 2)]).int()
    rope = ops.rope_table(ops.rope_inv_freq(D).cuda(), max(m, 64))
    proj, q, kk = ops.gemm_qk_norm_rope(a.cuda(), w.cuda(), qw.cuda(), kw.cuda(), pos.cuda(), rope, hq, hkv, D)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    full = a.float() @ w.float().t()
    qg = full[:, :2 * hq * D].reshape(m, hq, 2, D)
    cos, sin = O.rope_cos_sin(pos, D)
    q_ref = O.apply_partial_rope(O.rmsnorm_offset(qg[:, :, 0], qw), cos, sin)
    k_ref = O.apply_partial_rope(O.rmsnorm_offset(full[:, 2 * hq * D:(2 * hq + hkv) * D].reshape(m, hkv, D), kw), cos, sin)
    torch.testing.assert_close(q.cpu().float(), q_ref, rtol=0.008, atol=0.004)
    torch.testing.assert_close(kk.cpu().float(), k_ref, rtol=0.008, atol=0.004)
    # the output gate and v columns are the plain product
    check(proj.reshape(m, -1)[:, :2 * hq * D].reshape(m, hq, 2, D)[:, :, 1], qg[:, :, 1])
    check(proj[:, (2 * hq + hkv) * D:], full[:, (2 * hq + hkv) * D:])


@pytest.mark.parametrize("m,n,k,split", [(1536, 2048, 2048, 0), (1536, 2048, 6144, 0), (777, 2048, 2048, 1),
                                         (300, 264, 136, 3), (5, 256, 64, 0), (4097, 512, 1024, 2)])
def test_gemm_residual_add(m, n, k, split):
    """h (float32) += a w^T from the fp32 accumulators, k split into slices that each add their part;
    against the float32 product (the residual adds of [tf]:775, 781)."""
    a, w = inputs(m, n, k, m + 3 * n + k)
    h0 = torch.randn(m, n, generator=torch.Generator().manual_seed(m))
    h = h0.cuda()
    ops.gemm_residual_add(a.cuda(), w.cuda(), h, split_k=split)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    ref = h0 + a.float() @ w.float().t()
    err = (h.cpu() - ref).abs().max().item()
    assert err <= 1e-4 * max(1.0, ref.abs().max().item()), err


def test_rmsnorm_of_the_stream_alone():
    g = torch.Generator().manual_seed(3)
    h = torch.randn(100, 2048, generator=g)
    w = (0.02 * torch.randn(2048, generator=g)).bfloat16()
    got = ops.rmsnorm_stream(h.cuda(), w.cuda())
    torch.testing.assert_close(got.cpu().float(), O.rmsnorm_offset(h, w), rtol=0.008, atol=0.002)


def test_gemm_residual_add_is_reproducible_with_split_k():
    """The k-slices add into h in a fixed order: repeated calls give bit-identical results, and the
    ticket array is left zeroed."""
    a, w = inputs(1536, 2048, 6144, 77)
    a, w = a.cuda(), w.cuda()
    h0 = torch.randn(1536, 2048, generator=torch.Generator().manual_seed(78)).cuda()
    tk = ops.residual_add_tickets(1536, 2048, "cuda")
    outs = []
    for _ in range(3):
        h = h0.clone()
        ops.gemm_residual_add(a, w, h, split_k=4, tickets=tk)
        outs.append(h)
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert int(tk.abs().sum()) == 0


@pytest.mark.parametrize("m,n,k", [(1536, 2048, 2048), (1536, 2048, 6144), (300, 264, 136), (5, 2048, 6144)])
def test_gemm_partials_and_ordered_add(m, n, k):
    """k-split planes from the GEMM, added into the float32 stream in a fixed order by the norm
    kernel: h + a w^T against the float32 product, the norm against the oracle, and repeat calls
    bit-identical."""
    a, w = inputs(m, n, k, 5 * m + n + k)
    s = ops.split_slices(m, n, k)
    if n == 264:
        s = 2
    h0 = torch.randn(m, n, generator=torch.Generator().manual_seed(k))
    nw = (0.02 * torch.randn(n, generator=torch.Generator().manual_seed(n))).bfloat16()
    parts = torch.empty(s * m * n, device="cuda", dtype=torch.float32)
    outs = []
    for _ in range(2):
        h = h0.cuda()
        ops.gemm_partials(a.cuda(), w.cuda(), parts, s)
        x = ops.rmsnorm_add_partials(parts, s, h, nw.cuda())
        outs.append((h.clone(), x))
    torch.cuda.synchronize()
    assert _lib.poll_device_error() == 0
    ref = h0 + a.float() @ w.float().t()
    err = (outs[0][0].cpu() - ref).abs().max().item()
    assert err <= 1e-4 * max(1.0, ref.abs().max().item()), err
    torch.testing.assert_close(outs[0][1].cpu().float(), O.rmsnorm_offset(ref, nw), rtol=0.008, atol=0.002)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    h = h0.cuda()
    assert ops.rmsnorm_add_partials(parts, s, h, None) is None  # the add alone (last layer)
    assert torch.equal(h, outs[0][0])


def test_split_slices_choice():
    assert ops.split_slices(1536, 2048, 2048) == 3 and ops.split_slices(1536, 2048, 6144) == 3
    assert ops.split_slices(32768, 2048, 2048) == 1
