"""Parity of the layer kernels (gdn_layer.cu, through the C ABI) with the layer
oracle and the reference's fixtures.

16-bit results may differ from the oracle, rarely: the kernels sum in fp32 (the
conv's 16-bit products are exact there, their 4-term sum is not) and use the fast
exp, division and rsqrt for SiLU, sigmoid and the norm, which differ from the
oracle's fp32/fp64 values in their last bits and can flip a 16-bit rounding.  A
flip in the conv's intermediate rounding passes through SiLU, whose slope near
y = -4 turns one unit of a large y into several units of the small output.  The
bar written here: at most 0.1% of elements differ at all, and all of them within
the path's 16-bit tolerance (max-abs 2e-2, rel-L2 5e-3).  fp32 results within
1e-5 relative (the path's fp32 tolerance is 1e-4); g (accurate exp and log1p)
within 1e-6.  Pure copies (the conv state) are bit-exact.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import gdn_layer_oracle as L
from oracle import gdn_oracle as O
from oracle.gdn_oracle import round_bf16

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TDT = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(x, dtype="bf16"):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(TDT[dtype])


def host(t):
    return t.float().cpu().numpy()


def assert_close16(ours, ref, in_dtype="bf16", what=""):
    ours = np.asarray(ours, np.float32)
    ref = np.asarray(ref, np.float32)
    assert ours.shape == ref.shape, what
    if in_dtype == "fp32":
        np.testing.assert_allclose(ours, ref, rtol=1e-5, atol=1e-6, err_msg=what)
        return
    d = np.abs(ours - ref)
    frac = float(np.mean(d > 0))
    assert frac <= 1e-3, f"{what}: {frac:.2e} of elements differ"
    assert d.max() <= 2e-2, f"{what}: max-abs {d.max():.3e}"
    assert np.linalg.norm(d) <= 5e-3 * max(np.linalg.norm(ref), 1e-30), f"{what}: rel-L2 beyond 5e-3"


def _layer():
    from llms_from_scratch_b200 import layer
    return layer


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "layer_conv_T*.npz"))))
def test_prefill_conv_golden(path):
    z = np.load(path)
    st = torch.full((z["x"].shape[0], z["x"].shape[2], 4), 7.0, dtype=torch.bfloat16, device="cuda")
    y = _layer().causal_conv1d_silu(dev(z["x"]), dev(z["weight"]), conv_state=st)
    torch.cuda.synchronize()
    assert_close16(host(y), z["out"], what="conv out")
    np.testing.assert_array_equal(host(st), z["conv_state"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "layer_convupd_*.npz"))))
def test_decode_conv_update_golden(path):
    z = np.load(path)
    st = dev(z["conv_state"])
    y = _layer().causal_conv1d_update(dev(z["x"]).transpose(1, 2), st, dev(z["weight"]), None, "silu")
    torch.cuda.synchronize()
    assert y.shape == (z["x"].shape[0], z["x"].shape[2], z["x"].shape[1])
    assert_close16(host(y.transpose(1, 2)), z["out"], what="update out")
    np.testing.assert_array_equal(host(st), z["new_state"])


def test_gates_golden():
    z = np.load(os.path.join(GOLDEN, "layer_gates.npz"))
    g, beta = _layer().gates(dev(z["a"]), dev(z["b"]), dev(z["A_log"]), dev(z["dt_bias"]))
    torch.cuda.synchronize()
    assert g.dtype == torch.float32 and beta.dtype == torch.bfloat16
    np.testing.assert_allclose(host(g), z["g"], rtol=1e-6, atol=0)
    assert_close16(host(beta), z["beta"], what="beta")


def test_rms_norm_gated_golden():
    z = np.load(os.path.join(GOLDEN, "layer_rmsnorm_gated.npz"))
    o = _layer().rms_norm_gated(dev(z["x"]), dev(z["gate"]), dev(z["weight"]), float(z["eps"]))
    torch.cuda.synchronize()
    assert_close16(host(o), z["out"], what="norm")


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32", "fp16"])
@pytest.mark.parametrize("B,T,C", [(2, 1, 64), (1, 3, 128), (2, 17, 96), (1, 1000, 6144)])
def test_prefill_conv_vs_oracle(in_dtype, B, T, C):
    rng = np.random.default_rng(B * 7 + T + C)
    x = O.round_to(rng.standard_normal((B, T, C), dtype=np.float32), in_dtype)
    w = O.round_to(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5), in_dtype)
    st = torch.empty((B, C, 4), dtype=TDT[in_dtype], device="cuda")
    y = _layer().causal_conv1d_silu(dev(x, in_dtype), dev(w, in_dtype), conv_state=st)
    torch.cuda.synchronize()
    ry, rs = L.causal_conv1d_silu(x, w, in_dtype)
    assert_close16(host(y), ry, in_dtype, "conv out")
    np.testing.assert_array_equal(host(st), rs)


def test_decode_updates_reproduce_the_prefill():
    """Token-by-token decode from a zero state equals the prefill conv and leaves the same state."""
    B, T, C = 3, 12, 6144
    rng = np.random.default_rng(9)
    x = dev(round_bf16(rng.standard_normal((B, T, C), dtype=np.float32)))
    w = dev(round_bf16(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5)))
    lay = _layer()
    s_pre = torch.empty((B, C, 4), dtype=torch.bfloat16, device="cuda")
    y = lay.causal_conv1d_silu(x, w, conv_state=s_pre)
    s = torch.zeros((B, C, 4), dtype=torch.bfloat16, device="cuda")
    outs = [lay.causal_conv1d_update(x[:, t:t + 1].transpose(1, 2), s, w, None, "silu").transpose(1, 2)
            for t in range(T)]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(outs, dim=1), y)
    assert torch.equal(s, s_pre)
    # a two-token update equals two one-token updates
    s2 = torch.zeros_like(s)
    lay.causal_conv1d_update(x[:, :T - 2].transpose(1, 2), s2, w, None, "silu")
    y2 = lay.causal_conv1d_update(x[:, T - 2:].transpose(1, 2), s2, w, None, "silu").transpose(1, 2)
    torch.cuda.synchronize()
    assert torch.equal(y2, y[:, T - 2:])
    assert torch.equal(s2, s_pre)


def test_conv_fn_hook_takes_the_layers_layout():
    """causal_conv1d_fn receives mixed_qkv.transpose(1, 2) ([B, C, T]) as the layer passes it (:349-355)."""
    rng = np.random.default_rng(3)
    mixed = dev(round_bf16(rng.standard_normal((2, 40, 256), dtype=np.float32)))
    w = dev(round_bf16(rng.standard_normal((256, 4), dtype=np.float32) * np.float32(0.5)))
    lay = _layer()
    y_hook = lay.causal_conv1d_fn(x=mixed.transpose(1, 2), weight=w.unsqueeze(1).squeeze(1), bias=None,
                                  activation="silu", seq_idx=None)
    y = lay.causal_conv1d_silu(mixed, w)
    torch.cuda.synchronize()
    assert y_hook.shape == (2, 256, 40)
    assert torch.equal(y_hook.transpose(1, 2), y)


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32"])
def test_gates_vs_oracle(in_dtype):
    rng = np.random.default_rng(17)
    B, T, H = 3, 257, 16
    a = O.round_to(rng.standard_normal((B, T, H), dtype=np.float32) * np.float32(6.0), in_dtype)
    b = O.round_to(rng.standard_normal((B, T, H), dtype=np.float32) * np.float32(3.0), in_dtype)
    A_log = O.round_to(np.log(rng.uniform(0.5, 16.0, H).astype(np.float32)), in_dtype)
    dt = O.round_to(rng.standard_normal(H, dtype=np.float32), in_dtype)
    g, beta = _layer().gates(dev(a, in_dtype), dev(b, in_dtype), dev(A_log, in_dtype), dev(dt, in_dtype))
    torch.cuda.synchronize()
    rg, rb = L.gates(a, b, A_log, dt, in_dtype)
    np.testing.assert_allclose(host(g), rg, rtol=1e-6, atol=1e-30)
    assert_close16(host(beta), rb, in_dtype, "beta")


@pytest.mark.parametrize("in_dtype", ["bf16", "fp32"])
def test_rms_norm_gated_vs_oracle_and_strided_rows(in_dtype):
    rng = np.random.default_rng(23)
    N = 4096
    x = O.round_to(rng.standard_normal((N, 128), dtype=np.float32) * np.float32(2.0), in_dtype)
    z = O.round_to(rng.standard_normal((N, 128), dtype=np.float32) * np.float32(2.0), in_dtype)
    w = O.round_to(np.float32(1.0) + rng.standard_normal(128, dtype=np.float32) * np.float32(0.2), in_dtype)
    ref = L.rms_norm_gated(x, z, w, 1e-6, in_dtype)
    lay = _layer()
    o = lay.rms_norm_gated(dev(x, in_dtype), dev(z, in_dtype), dev(w, in_dtype), 1e-6)
    # rows taken from a wider buffer, as the layer's [B, T, H, D] -> [-1, D] reshape of a strided tensor
    wide = torch.zeros((N, 256), dtype=TDT[in_dtype], device="cuda")
    wide[:, 64:192] = dev(x, in_dtype)
    o2 = lay.rms_norm_gated(wide[:, 64:192], dev(z, in_dtype), dev(w, in_dtype), 1e-6)
    torch.cuda.synchronize()
    assert_close16(host(o), ref, in_dtype, "norm")
    assert torch.equal(o, o2)
    m = lay.RMSNormGated(128, eps=1e-6).cuda()
    with torch.no_grad():
        m.weight.copy_(dev(w, "fp32"))
        assert torch.equal(m(dev(x, in_dtype), dev(z, in_dtype)), o)


def test_layer_core_prefill_matches_the_oracle_pipeline():
    """conv -> q/k/v views of its output -> gates -> chunked rule -> gated norm, against the oracle's
    pipeline of the same steps (the core of Qwen3_5GatedDeltaNet.forward between its projections)."""
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    lay = _layer()
    B, T, H, D = 1, 300, 4, 128
    C = 3 * H * D
    rng = np.random.default_rng(31)
    mixed = round_bf16(rng.standard_normal((B, T, C), dtype=np.float32))
    w = round_bf16(rng.standard_normal((C, 4), dtype=np.float32) * np.float32(0.5))
    a = round_bf16(rng.standard_normal((B, T, H), dtype=np.float32))
    b = round_bf16(rng.standard_normal((B, T, H), dtype=np.float32))
    A_log = round_bf16(np.log(rng.uniform(0.5, 16.0, H).astype(np.float32)))
    dt = round_bf16(rng.standard_normal(H, dtype=np.float32))
    zg = round_bf16(rng.standard_normal((B, T, H, D), dtype=np.float32))
    nw = round_bf16(np.float32(1.0) + rng.standard_normal(D, dtype=np.float32) * np.float32(0.1))

    y = lay.causal_conv1d_silu(dev(mixed), dev(w))
    q, k, v = (y[..., i * H * D:(i + 1) * H * D].unflatten(-1, (H, D)) for i in range(3))  # strided views
    g, beta = lay.gates(dev(a), dev(b), dev(A_log), dev(dt))
    o, _ = fast_chunk_gated_delta_rule(q, k, v, g, beta, use_qk_l2norm_in_kernel=True)
    out = lay.rms_norm_gated(o, dev(zg), dev(nw), 1e-6)
    torch.cuda.synchronize()

    ry, _ = L.causal_conv1d_silu(mixed, w)
    rq, rk, rv = (ry[..., i * H * D:(i + 1) * H * D].reshape(B, T, H, D) for i in range(3))
    rg, rb = L.gates(a, b, A_log, dt)
    ro, _ = O.chunk_gated_delta_rule(rq, rk, rv, rg, rb, use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    ref = L.rms_norm_gated(np.asarray(ro, np.float32).reshape(-1, D), zg.reshape(-1, D), nw, 1e-6)
    ours = host(out).reshape(-1, D)
    err = float(np.abs(ours - ref).max())
    rel = float(np.linalg.norm(ours - ref) / np.linalg.norm(ref))
    assert err <= 5e-2 and rel <= 1e-2, (err, rel)  # the chunk rule's bf16 tolerance, through the norm
