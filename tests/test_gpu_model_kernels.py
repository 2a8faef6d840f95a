"""The decoder's own kernels (include/gdn_model.h) against plain PyTorch restatements of the
reference's bf16 ops (qwen3_5.py:35-183), on the GPU.

Each comparison follows the reference's op order in torch (bf16 tensors, fp32 where
the reference upcasts); the kernels accumulate in fp32 in another order, so a result
may differ by one bf16 rounding step in rare elements.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
bf = torch.bfloat16


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulps_apart(a, b):
    """Elementwise distance in bf16 units of the larger magnitude."""
    a, b = a.float(), b.float()
    ulp = torch.maximum(a.abs(), b.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(ulp)) - 7)
    return ((a - b).abs() / ulp)


def test_add_rms_norm_matches_the_block_ops():
    from llms_from_scratch_b200.model import add_rms_norm
    torch.manual_seed(0)
    N, D = 37, 1024
    x = torch.randn(N, D, device="cuda").to(bf)
    r = torch.randn(N, D, device="cuda").to(bf)
    w = (torch.randn(D, device="cuda") * 0.02).to(bf)
    h = x + r  # bf16 add (qwen3_5.py:231)
    hf = h.float()
    want = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())).to(bf)  # :57-63
    r2 = r.clone()
    out, res = add_rms_norm(x, w, 1e-6, residual=r2)
    assert torch.equal(res, h)
    d = _ulps_apart(out, want)
    assert (d <= 1).all() and (d > 0).float().mean() < 0.01
    out0, _ = add_rms_norm(x, w, 1e-6)
    xf = x.float()
    want0 = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())).to(bf)
    assert (_ulps_apart(out0, want0) <= 1).all()


def test_silu_mul_matches_the_feed_forward_ops():
    from llms_from_scratch_b200.model import silu_mul
    torch.manual_seed(1)
    u = torch.randn(9, 2 * 3584, device="cuda").to(bf) * 3
    want = F.silu(u[:, :3584]) * u[:, 3584:]  # qwen3_5.py:45, bf16 ops
    got = silu_mul(u)
    d = _ulps_apart(got, want)
    assert (d <= 1).all() and (d > 0).float().mean() < 0.01


def _reference_attention(qkv_all, qn, kn, cos, sin, Hq=8, Hkv=2, Dh=256):
    """GroupedQueryAttention.forward's ops (qwen3_5.py:145-183) up to out_proj, over the whole sequence."""
    B, T, _ = qkv_all.shape
    qg = qkv_all[..., :Hq * 2 * Dh].view(B, T, Hq, 2 * Dh)
    queries, gate = torch.chunk(qg, 2, dim=-1)
    gate = gate.reshape(B, T, Hq * Dh)
    keys = qkv_all[..., Hq * 2 * Dh:Hq * 2 * Dh + Hkv * Dh].reshape(B, T, Hkv, Dh).transpose(1, 2)
    values = qkv_all[..., Hq * 2 * Dh + Hkv * Dh:].reshape(B, T, Hkv, Dh).transpose(1, 2)
    queries = queries.transpose(1, 2)

    def rms(x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())).to(x.dtype)

    def rope(x):
        rot = cos.shape[-1]
        xr, xp = x[..., :rot], x[..., rot:]
        x1, x2 = xr[..., :rot // 2], xr[..., rot // 2:]
        c, s = cos[:T][None, None], sin[:T][None, None]
        out = torch.cat([xr * c + torch.cat((-x2, x1), -1) * s, xp], -1)
        return out.to(x.dtype)

    queries, keys = rope(rms(queries, qn)), rope(rms(keys, kn))
    keys = keys.repeat_interleave(Hq // Hkv, dim=1)
    values = values.repeat_interleave(Hq // Hkv, dim=1)
    mask = torch.triu(torch.ones(T, T, device=qkv_all.device, dtype=torch.bool), diagonal=1)
    sc = (queries @ keys.transpose(2, 3)).masked_fill(mask, -torch.inf)
    wts = torch.softmax(sc * (Dh ** -0.5), dim=-1, dtype=torch.float32).to(bf)
    ctx = (wts @ values).transpose(1, 2).reshape(B, T, Hq * Dh)
    return ctx * torch.sigmoid(gate)


def test_cached_attention_matches_full_recompute():
    """Prefill 5 tokens into the cache, then 3 more tokens in one call at position 5: the outputs of the
    later call equal the reference ops recomputed over all 8 positions."""
    import ctypes

    from llms_from_scratch_b200 import _lib
    from llms_from_scratch_b200.model import QWEN3_5_0_8B, rope_tables
    from llms_from_scratch_b200.ops import _desc
    torch.manual_seed(2)
    B, T1, T2, L, Hq, Hkv, Dh = 2, 5, 3, 64, 8, 2, 256
    W = (2 * Hq + 2 * Hkv) * Dh
    qkv = torch.randn(B, T1 + T2, W, device="cuda").to(bf)
    qn = (torch.randn(Dh, device="cuda") * 0.1).to(bf)
    kn = (torch.randn(Dh, device="cuda") * 0.1).to(bf)
    cos, sin, rot = rope_tables(QWEN3_5_0_8B, L)
    cos, sin = cos.cuda(), sin.cuda()
    kc = torch.zeros(B, Hkv, L, Dh, device="cuda", dtype=bf)
    vc = torch.zeros_like(kc)
    lib = _lib.load()
    outs = []
    for lo, hi in ((0, T1), (T1, T1 + T2)):
        part = qkv[:, lo:hi]
        pos = torch.tensor([lo], dtype=torch.int32, device="cuda")
        q = torch.empty(B, hi - lo, Hq, Dh, device="cuda", dtype=bf)
        st = torch.cuda.current_stream().cuda_stream
        d = [_desc(x) for x in (part, qn, kn, q, kc, vc)]
        _lib.check(lib.gdn_model_attn_prep(ctypes.byref(d[0]), ctypes.byref(d[1]), ctypes.byref(d[2]), cos.data_ptr(),
                                           sin.data_ptr(), rot, pos.data_ptr(), 1e-6, ctypes.byref(d[3]),
                                           ctypes.byref(d[4]), ctypes.byref(d[5]), st))
        gate = part[..., :Hq * 2 * Dh].unflatten(-1, (Hq, 2 * Dh))[..., Dh:]
        out = torch.empty(B, hi - lo, Hq * Dh, device="cuda", dtype=bf)
        dg, do = _desc(gate), _desc(out)
        _lib.check(lib.gdn_model_attention(ctypes.byref(d[3]), ctypes.byref(d[4]), ctypes.byref(d[5]),
                                           ctypes.byref(dg), pos.data_ptr(), ctypes.byref(do), st))
        outs.append(out)
    got = torch.cat(outs, 1).float()
    want = _reference_attention(qkv, qn, kn, cos, sin).float()
    err = (got - want).abs()
    scale = want.abs().max()
    assert err.max() <= 0.02 * scale, (err.max().item(), scale.item())
    assert (err / scale).mean() < 2e-3


@pytest.mark.parametrize("M", [1, 3, 8, 17, 32])
def test_decode_linear_matches_fp32_matmul(M):
    """gdn_model_linear (the decode projections) against the fp32 product of the same bf16 operands."""
    from llms_from_scratch_b200.model import EPI_PARTIAL, EPI_SILU_MUL, EPI_STORE, interleave_fc12, linear
    torch.manual_seed(10 + M)
    K, N = 1024, 272
    x = torch.randn(M, K, device="cuda").to(bf)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(bf)
    want = x.float() @ w.float().T
    got = linear(x, w, EPI_STORE)
    # one bf16 rounding step, or a tiny absolute slack for results near zero (fp32 sums in another order)
    near = (got.float() - want).abs() <= 1e-4 * want.abs().max()
    assert ((_ulps_apart(got, want.to(bf)) <= 1) | near).all()
    # split-K partials sum to the fp32 product
    K2 = 3584
    x2 = torch.randn(M, K2, device="cuda").to(bf)
    w2 = (torch.randn(N, K2, device="cuda") * 0.05).to(bf)
    part = linear(x2, w2, EPI_PARTIAL, ksplit=4).buf
    assert part.shape == (4, M, N)
    ref2 = x2.float() @ w2.float().T
    assert ((part.sum(0) - ref2).abs() <= 1e-4 * ref2.abs().max()).all()
    # the FFN epilogue on interleaved fc1 / fc2 rows: SiLU(fc1 x) * (fc2 x) with the reference's roundings
    F_ = 136
    fc1 = (torch.randn(F_, K, device="cuda") * 0.05).to(bf)
    fc2 = (torch.randn(F_, K, device="cuda") * 0.05).to(bf)
    act = linear(x, interleave_fc12(fc1, fc2), EPI_SILU_MUL)
    want_act = F.silu((x.float() @ fc1.float().T).to(bf)) * (x.float() @ fc2.float().T).to(bf)
    assert act.shape == (M, F_)
    near = (act.float() - want_act.float()).abs() <= 1e-3 * want_act.float().abs().max()
    assert ((_ulps_apart(act, want_act) <= 2) | near).all()


def test_fused_gdn_decode_matches_the_separate_kernels():
    """gdn_model_gdn_decode (conv update + gates + recurrent rule + gated norm for one token) equals the
    four separate kernels it replaces, on random states and projections."""
    from llms_from_scratch_b200 import fast_recurrent_gated_delta_rule, layer
    from llms_from_scratch_b200.model import gdn_decode
    torch.manual_seed(4)
    B, H, D = 5, 16, 128
    C = 3 * H * D
    proj = torch.randn(B, C + H * D + 2 * H, device="cuda").to(bf)
    conv_state = torch.randn(B, C, 4, device="cuda").to(bf)
    conv_w = (torch.randn(C, 4, device="cuda") * 0.5).to(bf)
    A_log = torch.log(torch.rand(H, device="cuda") * 15 + 0.5).to(bf)
    dt_bias = torch.randn(H, device="cuda").to(bf)
    state = torch.randn(B, H, D, D, device="cuda") * 0.05
    norm_w = (1 + 0.1 * torch.randn(D, device="cuda")).to(bf)
    # the separate kernels
    cs1, st1 = conv_state.clone(), state.clone()
    mixed = proj[:, :C].unsqueeze(1)
    conv = layer.causal_conv1d_update(mixed.transpose(1, 2), cs1, conv_w, None, "silu").transpose(1, 2)
    z = proj[:, C:C + H * D]
    b_, a_ = proj[:, C + H * D:C + H * D + H].unsqueeze(1), proj[:, C + H * D + H:].unsqueeze(1)
    g, beta = layer.gates(a_, b_, A_log, dt_bias)
    q, k, v = (conv[..., i * H * D:(i + 1) * H * D].unflatten(-1, (H, D)) for i in range(3))
    core, _ = fast_recurrent_gated_delta_rule(q, k, v, g, beta, st1, True, use_qk_l2norm_in_kernel=True, out_state=st1)
    want = layer.rms_norm_gated(core.reshape(B, H, D), z.reshape(B, H, D), norm_w, 1e-6).reshape(B, H * D)
    # fused
    cs2, st2 = conv_state.clone(), state.clone()
    got = gdn_decode(proj, cs2, conv_w, A_log, dt_bias, st2, norm_w, 1e-6)
    assert torch.equal(cs1, cs2)
    # the same arithmetic per state element; the kv / o sums over the 128 rows run in another order
    torch.testing.assert_close(st2, st1, rtol=1e-5, atol=1e-6)
    d = _ulps_apart(got, want)
    assert (d <= 1).all() and (d > 0).float().mean() < 0.01, (d.max().item(), (d > 0).float().mean().item())
