"""Parity of the CUDA path (through the C ABI) with the CPU oracle and with the
reference's own golden vectors.

Tolerances are the ones the reference path is held to: for 16-bit inputs with
fp32 accumulation max-abs 2e-2 and relative-L2 5e-3; for fp32 inputs 1e-4
(max-abs).  Sizes the oracle cannot finish in seconds are checked through
size-independent properties instead (state passing, batch independence).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TDT = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
BF16_MAX_ABS, BF16_REL_L2, FP32_MAX_ABS = 2e-2, 5e-3, 1e-4


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_from_scratch_b200 import _lib
    _lib.load()


def ops():
    import llms_from_scratch_b200 as m
    return m


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda").to(dtype)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_parity(ours, ref, in_dtype, what=""):
    ours = np.asarray(ours, np.float32)
    ref = np.asarray(ref, np.float32)
    assert ours.shape == ref.shape, what
    assert np.all(np.isfinite(ours)), f"{what}: non-finite values"
    err = float(np.abs(ours - ref).max()) if ours.size else 0.0
    if in_dtype == "fp32":
        assert err <= FP32_MAX_ABS, f"{what}: max-abs {err:.3e} > {FP32_MAX_ABS}"
    else:
        r = rel_l2(ours, ref) if ours.size else 0.0
        assert err <= BF16_MAX_ABS and r <= BF16_REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {r:.3e}"


def run_chunk(q, k, v, g, beta, state, in_dtype, l2=True, ofs=True):
    m = ops()
    dt = TDT[in_dtype]
    o, s = m.fast_chunk_gated_delta_rule(dev(q, dt), dev(k, dt), dev(v, dt), dev(g), dev(beta), chunk_size=64,
                                         initial_state=dev(state), output_final_state=ofs,
                                         use_qk_l2norm_in_kernel=l2)
    assert o.dtype == dt
    return o.float().cpu().numpy(), (None if s is None else s.cpu().numpy())


def run_rec(q, k, v, g, beta, state, in_dtype, l2=True, ofs=True):
    m = ops()
    dt = TDT[in_dtype]
    o, s = m.fast_recurrent_gated_delta_rule(dev(q, dt), dev(k, dt), dev(v, dt), dev(g), dev(beta),
                                             dev(state), ofs, use_qk_l2norm_in_kernel=l2)
    return o.float().cpu().numpy(), (None if s is None else s.cpu().numpy())


GOLDEN_FILES = sorted(p for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                      if not os.path.basename(p).startswith(("config1", "layer_", "bwd_", "model_")))  # layer_*, bwd_*, model_*: own tests


@pytest.mark.parametrize("path", GOLDEN_FILES, ids=[os.path.basename(p)[:-4] for p in GOLDEN_FILES])
def test_against_reference_golden_vectors(path):
    z = np.load(path)
    d = {k: z[k] for k in z.files}
    kind, in_dtype = str(d["kind"]), str(d["in_dtype"])
    fn = run_chunk if kind == "chunk" else run_rec
    ref_o = O.from_bf16_bits(d["out"]) if in_dtype == "bf16" else d["out"]
    if "q_l2" in d:
        # 16-bit fixture: start from the reference's own normalised q/k (torch's CPU
        # bf16 rsqrt is a hardware estimate), which pins the rest of the arithmetic
        # at the full tolerance ...
        o, s = fn(d["q_l2"], d["k_l2"], d["v"], d["g"], d["beta"], d.get("initial_state"), in_dtype,
                  l2=False, ofs=bool(d["output_final_state"]))
        assert_parity(o, ref_o, in_dtype, "out (reference-normalised q/k)")
        if "final_state" in d:
            assert_parity(s, d["final_state"], in_dtype, "final_state (reference-normalised q/k)")
    # ... and end to end with the in-kernel l2norm
    o, s = fn(d["q"], d["k"], d["v"], d["g"], d["beta"], d.get("initial_state"), in_dtype,
              l2=bool(d["l2norm"]), ofs=bool(d["output_final_state"]))
    assert_parity(o, ref_o, in_dtype, "out")
    if "final_state" in d:
        if "q_l2" in d:
            # A one-ulp difference in the inverse norm of one recent key (the rsqrt
            # estimate above) moves the final state by up to ~0.5% rel-L2 when q/k
            # are far from unit norm; the oracle sees the same gap.
            assert rel_l2(s, d["final_state"]) < 1e-2
        else:
            assert_parity(s, d["final_state"], in_dtype, "final_state")
    else:
        assert s is None


def test_config1_golden_sample():
    z = np.load(os.path.join(GOLDEN, "config1_fp32_B1_T256_H16.npz"))
    q, k, v, g, beta, _ = O.make_inputs(int(z["B"]), int(z["T"]), int(z["H"]), seed=int(z["seed"]))
    o, s = run_chunk(q, k, v, g, beta, None, "fp32")
    st = int(z["stride"])
    assert_parity(o.reshape(-1)[::st], z["out_sample"], "fp32", "out sample")
    assert_parity(s.reshape(-1)[::st], z["state_sample"], "fp32", "state sample")


@pytest.mark.parametrize("in_dtype", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
@pytest.mark.parametrize("with_state", [False, True])
def test_chunk_edge_lengths_vs_oracle(in_dtype, T, with_state):
    q, k, v, g, beta, s0 = O.make_inputs(2, T, 3, seed=100 + T, in_dtype=in_dtype,
                                         init_state_std=0.02 if with_state else 0.0, normalize_qk=False)
    o, s = run_chunk(q, k, v, g, beta, s0, in_dtype)
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype=in_dtype)
    assert_parity(o, ro, in_dtype, "out")
    assert_parity(s, rs, in_dtype, "state")


@pytest.mark.parametrize("in_dtype", ["fp32", "bf16"])
def test_chunk_without_l2norm_and_without_final_state(in_dtype):
    q, k, v, g, beta, s0 = O.make_inputs(1, 130, 2, seed=7, in_dtype=in_dtype, init_state_std=0.02)
    o, s = run_chunk(q, k, v, g, beta, s0, in_dtype, l2=False, ofs=False)
    assert s is None
    ro, _ = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, use_qk_l2norm_in_kernel=False,
                                     in_dtype=in_dtype)
    assert_parity(o, ro, in_dtype, "out")


@pytest.mark.parametrize("T", [256, 512, 1024, 2048, 4096])
def test_config2_bf16_full_size_vs_oracle(T):
    """Benchmark config 2: B=1, H=16, bf16 q/k/v, fp32 g/beta, initial state ~ N(0, 0.02)."""
    q, k, v, g, beta, s0 = O.make_inputs(1, T, 16, seed=0, in_dtype="bf16", init_state_std=0.02)
    o, s = run_chunk(q, k, v, g, beta, s0, "bf16")
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    assert_parity(o, ro, "bf16", "out")
    assert_parity(s, rs, "bf16", "state")


def test_strided_views_like_the_model():
    """q/k/v as views into one packed projection (qwen3_5_transformers.py:363-375)."""
    m = ops()
    B, T, H = 2, 150, 4
    torch.manual_seed(0)
    mixed = torch.randn(B, T, 3 * H * 128, device="cuda", dtype=torch.bfloat16)
    q, k, v = torch.split(mixed, [H * 128] * 3, dim=-1)
    q, k, v = (x.reshape(B, T, H, 128) for x in (q, k, v))
    ab = torch.randn(B, T, 2 * H, device="cuda")
    g = (-torch.nn.functional.softplus(ab))[..., :H]
    beta = ab.sigmoid()[..., H:]
    assert not q.is_contiguous() and not g.is_contiguous()
    o1, s1 = m.fast_chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True)
    o2, s2 = m.fast_chunk_gated_delta_rule(q.contiguous(), k.contiguous(), v.contiguous(), g.contiguous(),
                                           beta.contiguous(), output_final_state=True, use_qk_l2norm_in_kernel=True)
    torch.testing.assert_close(o1, o2, rtol=0, atol=0)
    torch.testing.assert_close(s1, s2, rtol=0, atol=0)


def test_state_passing_property_full_size():
    """[0,T) in one call == [0,T1) then [T1,T) from the carried state (T=4096, T1 off a chunk boundary)."""
    m = ops()
    q, k, v, g, beta, s0 = O.make_inputs(1, 4096, 16, seed=3, in_dtype="bf16", init_state_std=0.02)
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, ts = dev(g), dev(beta), dev(s0)
    o_full, s_full = m.fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=ts, output_final_state=True,
                                                   use_qk_l2norm_in_kernel=True)
    T1 = 1000
    o_a, s_a = m.fast_chunk_gated_delta_rule(tq[:, :T1], tk[:, :T1], tv[:, :T1], tg[:, :T1], tb[:, :T1],
                                             initial_state=ts, output_final_state=True, use_qk_l2norm_in_kernel=True)
    o_b, s_b = m.fast_chunk_gated_delta_rule(tq[:, T1:], tk[:, T1:], tv[:, T1:], tg[:, T1:], tb[:, T1:],
                                             initial_state=s_a, output_final_state=True, use_qk_l2norm_in_kernel=True)
    assert_parity(torch.cat([o_a, o_b], 1).float().cpu().numpy(), o_full.float().cpu().numpy(), "bf16", "out")
    assert_parity(s_b.cpu().numpy(), s_full.cpu().numpy(), "bf16", "state")


def test_batch_independence_config3_sample():
    """Config 3 sample (B=64 at T=512): every sequence equals its own B=1 run."""
    m = ops()
    B, T, H = 64, 512, 16
    torch.manual_seed(1)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device="cuda"), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device="cuda"), dim=-1).bfloat16()
    v = torch.randn(B, T, H, 128, device="cuda").bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda"))
    beta = torch.randn(B, T, H, device="cuda").sigmoid()
    s0 = torch.randn(B, H, 128, 128, device="cuda") * 0.02
    o, s = m.fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                         use_qk_l2norm_in_kernel=True)
    for b in (0, 17, 63):
        ob, sb = m.fast_chunk_gated_delta_rule(q[b:b + 1], k[b:b + 1], v[b:b + 1], g[b:b + 1], beta[b:b + 1],
                                               initial_state=s0[b:b + 1], output_final_state=True,
                                               use_qk_l2norm_in_kernel=True)
        torch.testing.assert_close(ob, o[b:b + 1], rtol=0, atol=0)
        torch.testing.assert_close(sb, s[b:b + 1], rtol=0, atol=0)


@pytest.mark.parametrize("B,T,H,with_state,ofs", [
    (3, 777, 8, True, True),     # 24 (b, h) chains: the lean scan (more than one wave of 16-column slices); ragged
    (2, 65, 16, False, True),    # two chunks, the second of one token, zero start
    (4, 300, 6, True, False),    # no final state
])
def test_many_chains_ragged_vs_oracle(B, T, H, with_state, ofs):
    """More (b, h) chains than the 16-column scan fits in one wave (B*H > 18): the lean scan, held to the
    oracle on ragged lengths, with and without initial and final states; and each sequence equals its own
    B=1 call (16-column scan) bit for bit."""
    m = ops()
    q, k, v, g, beta, s0 = O.make_inputs(B, T, H, seed=40 + T, in_dtype="bf16", init_state_std=0.02,
                                         normalize_qk=False)
    s0 = s0 if with_state else None
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, ts = dev(g), dev(beta), dev(s0)
    o, s = m.fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=ts, output_final_state=ofs,
                                         use_qk_l2norm_in_kernel=True)
    assert_parity(o.float().cpu().numpy(), ro, "bf16", "out")
    if ofs:
        assert_parity(s.cpu().numpy(), rs, "bf16", "final_state")
    else:
        assert s is None
    for b in (0, B - 1):
        ob, sb = m.fast_chunk_gated_delta_rule(tq[b:b + 1], tk[b:b + 1], tv[b:b + 1], tg[b:b + 1], tb[b:b + 1],
                                               initial_state=None if ts is None else ts[b:b + 1],
                                               output_final_state=ofs, use_qk_l2norm_in_kernel=True)
        assert torch.equal(ob, o[b:b + 1])
        if ofs:
            assert torch.equal(sb, s[b:b + 1])


def test_config3_full_size_sequences_vs_oracle():
    """Config 3 at full size (B=64, T=4096, H=16, bf16, initial state ~ N(0, 0.02)): three sequences of the
    batched call against the oracle, each on its own."""
    m = ops()
    B, T, H = 64, 4096, 16
    gen = torch.Generator(device="cuda").manual_seed(5)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device="cuda", generator=gen), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device="cuda", generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, 128, device="cuda", generator=gen).bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=gen))
    beta = torch.randn(B, T, H, device="cuda", generator=gen).sigmoid()
    s0 = torch.randn(B, H, 128, 128, device="cuda", generator=gen) * 0.02
    o, s = m.fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                         use_qk_l2norm_in_kernel=True)
    for b in (0, 31, 63):
        host = [x[b:b + 1].float().cpu().numpy() for x in (q, k, v, g, beta, s0)]
        ro, rs = O.chunk_gated_delta_rule(*host[:5], initial_state=host[5], output_final_state=True,
                                          use_qk_l2norm_in_kernel=True, in_dtype="bf16")
        assert_parity(o[b:b + 1].float().cpu().numpy(), ro, "bf16", f"sequence {b} out")
        assert_parity(s[b:b + 1].cpu().numpy(), rs, "bf16", f"sequence {b} state")


@pytest.mark.parametrize("in_dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("T", [1, 2, 37])
def test_recurrent_vs_oracle(in_dtype, T):
    q, k, v, g, beta, s0 = O.make_inputs(3, T, 4, seed=200 + T, in_dtype=in_dtype, init_state_std=0.02,
                                         normalize_qk=False)
    o, s = run_rec(q, k, v, g, beta, s0, in_dtype)
    ro, rs = O.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, use_qk_l2norm_in_kernel=True,
                                          in_dtype=in_dtype)
    assert_parity(o, ro, in_dtype, "out")
    assert_parity(s, rs, in_dtype, "state")


@pytest.mark.parametrize("in_dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("B,H,std", [(10, 16, 0.02), (19, 16, 0.5), (32, 16, 0.5), (3, 64, 0.02)])
def test_recurrent_decode_batches_vs_oracle(in_dtype, B, H, std):
    """One decode token over decode-sized batches (160 to 512 heads, the config-4 batch of 32 among them),
    with small and large initial states."""
    q, k, v, g, beta, s0 = O.make_inputs(B, 1, H, seed=300 + B, in_dtype=in_dtype, init_state_std=std,
                                         normalize_qk=False)
    o, s = run_rec(q, k, v, g, beta, s0, in_dtype)
    ro, rs = O.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, use_qk_l2norm_in_kernel=True,
                                          in_dtype=in_dtype)
    assert_parity(o, ro, in_dtype, "out")
    assert_parity(s, rs, in_dtype, "state")


def test_recurrent_decode_batch_variants():
    """A decode batch without an initial state, without a final state and in place, each equal to the
    oracle; and the batch equals the same sequences decoded one call each."""
    m = ops()
    B, H = 20, 16
    q, k, v, g, beta, s0 = O.make_inputs(B, 1, H, seed=41, in_dtype="bf16", init_state_std=0.3, normalize_qk=False)
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, ts = dev(g), dev(beta), dev(s0)
    ro, rs = O.recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    zo, zs = O.recurrent_gated_delta_rule(q, k, v, g, beta, None, True, use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    o, s = m.fast_recurrent_gated_delta_rule(tq, tk, tv, tg, tb, None, True, use_qk_l2norm_in_kernel=True)
    assert_parity(o.float().cpu().numpy(), zo, "bf16", "zero initial state: out")
    assert_parity(s.cpu().numpy(), zs, "bf16", "zero initial state: state")
    o, s = m.fast_recurrent_gated_delta_rule(tq, tk, tv, tg, tb, ts, False, use_qk_l2norm_in_kernel=True)
    assert s is None
    assert_parity(o.float().cpu().numpy(), ro, "bf16", "no final state: out")
    groups = [m.fast_recurrent_gated_delta_rule(tq[b:b + 1], tk[b:b + 1], tv[b:b + 1], tg[b:b + 1], tb[b:b + 1],
                                                ts[b:b + 1], True, use_qk_l2norm_in_kernel=True) for b in range(B)]
    state = ts.clone()
    o, s = m.fast_recurrent_gated_delta_rule(tq, tk, tv, tg, tb, state, True, use_qk_l2norm_in_kernel=True,
                                             out_state=state)
    assert s.data_ptr() == state.data_ptr()
    assert_parity(o.float().cpu().numpy(), ro, "bf16", "in place: out")
    assert_parity(state.cpu().numpy(), rs, "bf16", "in place: state")
    torch.testing.assert_close(o, torch.cat([x[0] for x in groups]), rtol=1e-2, atol=1e-5)
    torch.testing.assert_close(state, torch.cat([x[1] for x in groups]), rtol=1e-5, atol=1e-6)
    from llms_from_scratch_b200.ops import check_device_errors
    check_device_errors(sync=True)  # raises if a bounded wait gave up


def test_recurrent_in_place_decode_matches_chunk_prefix():
    """Prefill via the chunk kernel, then 8 in-place single-token decode steps ==
    the chunk kernel over the whole sequence (the model's prefill->decode path)."""
    m = ops()
    q, k, v, g, beta, _ = O.make_inputs(2, 136, 16, seed=9, in_dtype="bf16", normalize_qk=False)
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb = dev(g), dev(beta)
    o_full, s_full = m.fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, output_final_state=True,
                                                   use_qk_l2norm_in_kernel=True)
    P = 128
    _, state = m.fast_chunk_gated_delta_rule(tq[:, :P], tk[:, :P], tv[:, :P], tg[:, :P], tb[:, :P],
                                             output_final_state=True, use_qk_l2norm_in_kernel=True)
    outs = []
    for t in range(P, 136):
        sl = slice(t, t + 1)
        o_t, s_t = m.fast_recurrent_gated_delta_rule(tq[:, sl], tk[:, sl], tv[:, sl], tg[:, sl], tb[:, sl], state,
                                                     True, use_qk_l2norm_in_kernel=True, out_state=state)
        assert s_t.data_ptr() == state.data_ptr()
        outs.append(o_t)
    assert_parity(torch.cat(outs, 1).float().cpu().numpy(), o_full[:, P:].float().cpu().numpy(), "bf16", "decode out")
    assert_parity(state.cpu().numpy(), s_full.cpu().numpy(), "bf16", "decode state")


def test_empty_sequence_returns_initial_state():
    m = ops()
    q = torch.zeros(2, 0, 3, 128, device="cuda", dtype=torch.bfloat16)
    g = torch.zeros(2, 0, 3, device="cuda")
    s0 = torch.randn(2, 3, 128, 128, device="cuda")
    o, s = m.fast_chunk_gated_delta_rule(q, q, q, g, g, initial_state=s0, output_final_state=True)
    assert o.shape == (2, 0, 3, 128)
    torch.testing.assert_close(s, s0, rtol=0, atol=0)
    o, s = m.fast_chunk_gated_delta_rule(q, q, q, g, g, output_final_state=True)
    assert float(s.abs().max()) == 0.0


def test_inputs_are_not_modified():
    m = ops()
    q, k, v, g, beta, s0 = O.make_inputs(1, 100, 2, seed=5, in_dtype="bf16", init_state_std=0.02)
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, ts = dev(g), dev(beta), dev(s0)
    before = [x.clone() for x in (tq, tk, tv, tg, tb, ts)]
    m.fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=ts, output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    for a, b in zip(before, (tq, tk, tv, tg, tb, ts)):
        assert torch.equal(a, b)


def test_launch_counter_and_phase_events():
    import ctypes

    from llms_from_scratch_b200 import _lib
    m = ops()
    lib = _lib.load()
    q, k, v, g, beta, _ = O.make_inputs(1, 256, 4, seed=1, in_dtype="bf16")
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb = dev(g), dev(beta)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for e in evs:
        e.record()  # torch creates the underlying cudaEvent_t on first record
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 3)(*[e.cuda_event for e in evs])
    n0 = lib.gdn_launch_count()
    lib.gdn_set_phase_events(arr, 3)
    try:
        m.fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, use_qk_l2norm_in_kernel=True)
    finally:
        lib.gdn_set_phase_events(None, 0)
    torch.cuda.synchronize()
    assert lib.gdn_launch_count() - n0 >= 2
    assert evs[0].elapsed_time(evs[1]) > 0 and evs[1].elapsed_time(evs[2]) > 0


def test_tensor_core_and_cuda_core_paths_agree():
    """bf16 inputs with 8-byte-aligned rows take the tcgen05 path; the same values
    behind a 2-byte offset take the CUDA-core path.  Both match the oracle."""
    m = ops()
    q, k, v, g, beta, s0 = O.make_inputs(2, 300, 4, seed=21, in_dtype="bf16", init_state_std=0.02,
                                         normalize_qk=False)
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")

    def shifted(x):
        buf = torch.zeros(x.size + 1, dtype=torch.bfloat16, device="cuda")
        view = buf[1:].view(x.shape)
        view.copy_(torch.from_numpy(x).to(torch.bfloat16))
        assert view.data_ptr() % 8 != 0
        return view

    outs = {}
    for name, mk in (("tc", lambda x: dev(x, torch.bfloat16)), ("simt", shifted)):
        o, s = m.fast_chunk_gated_delta_rule(mk(q), mk(k), mk(v), dev(g), dev(beta), initial_state=dev(s0),
                                             output_final_state=True, use_qk_l2norm_in_kernel=True)
        outs[name] = (o.float().cpu().numpy(), s.cpu().numpy())
        assert_parity(outs[name][0], ro, "bf16", f"{name} out")
        assert_parity(outs[name][1], rs, "bf16", f"{name} state")
    assert_parity(outs["tc"][0], outs["simt"][0], "bf16", "tc vs simt out")


@pytest.mark.parametrize("gscale", [0.05, 1.0, 4.0])
def test_decay_range_vs_oracle(gscale):
    """Weak (g*0.05) to strong (g*4) decay: the inter-chunk state matters most when decay is weak."""
    q, k, v, g, beta, s0 = O.make_inputs(1, 512, 4, seed=31, in_dtype="bf16", init_state_std=0.02,
                                         normalize_qk=False)
    g = (g * gscale).astype(np.float32)
    o, s = run_chunk(q, k, v, g, beta, s0, "bf16")
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    assert_parity(o, ro, "bf16", "out")
    assert_parity(s, rs, "bf16", "state")


def test_device_error_word_is_clear():
    from llms_from_scratch_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.load().gdn_device_error(1) == 0
