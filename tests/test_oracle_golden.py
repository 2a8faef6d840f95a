"""Pin the CPU oracle against vectors produced by the reference's own torch code.

The fixtures under tests/golden/ were made by tests/golden/make_golden.py,
which calls torch_chunk_gated_delta_rule / torch_recurrent_gated_delta_rule
(qwen3_5_transformers.py:110-229) on CPU.
"""
import glob
import os

import numpy as np
import pytest

from oracle import gdn_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(p for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
               if not os.path.basename(p).startswith(("config1", "layer_", "bwd_", "model_")))  # layer_*, bwd_*, model_*: their own tests


def _load(path):
    z = np.load(path)
    d = {k: z[k] for k in z.files}
    d["kind"] = str(d["kind"])
    d["in_dtype"] = str(d["in_dtype"])
    return d


def _run_oracle(d, acc=np.float32):
    fn = O.chunk_gated_delta_rule if d["kind"] == "chunk" else O.recurrent_gated_delta_rule
    kw = dict(initial_state=d.get("initial_state"), output_final_state=bool(d["output_final_state"]),
              use_qk_l2norm_in_kernel=bool(d["l2norm"]), in_dtype=d["in_dtype"], acc=acc)
    if d["kind"] == "chunk":
        kw["chunk_size"] = 64
    return fn(d["q"], d["k"], d["v"], d["g"], d["beta"], **kw)


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(p)[:-4] for p in CASES])
def test_oracle_matches_reference_fixture(path):
    d = _load(path)
    if "q_l2" in d:
        # 16-bit case: feed the reference's own normalised q/k (exact fp32 values of
        # bf16 numbers) so the chunk/recurrent arithmetic is pinned exactly.
        d2 = dict(d, q=d["q_l2"], k=d["k_l2"], l2norm=np.array(False))
        out, state = _run_oracle(d2)
    else:
        out, state = _run_oracle(d)
    ref_out = O.from_bf16_bits(d["out"]) if d["in_dtype"] == "bf16" else d["out"]
    assert out.shape == ref_out.shape
    if d["in_dtype"] == "bf16":
        # fp32 summation order may flip the final bf16 rounding by one ulp
        ulp = np.maximum(np.abs(ref_out), np.abs(out)) * 2.0 ** -7 + 1e-30
        assert np.all(np.abs(out - ref_out) <= ulp)
        assert np.mean(out != ref_out) < 0.01
    else:
        np.testing.assert_allclose(out, ref_out, rtol=1e-5, atol=2e-6)
    if "final_state" in d:
        assert state is not None
        np.testing.assert_allclose(state, d["final_state"], rtol=1e-5, atol=2e-6)
    else:
        assert state is None


@pytest.mark.parametrize("path", [p for p in CASES if "bf16" in p], ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_bf16_l2norm_and_end_to_end(path):
    """The oracle's bf16 l2norm uses a correctly rounded rsqrt; torch's CPU
    bf16 rsqrt is a hardware estimate, so at most a few rows differ by one
    ulp of the inverse norm.  End to end the oracle stays well inside the
    bf16 tolerance class (max-abs 2e-2, rel-L2 5e-3)."""
    d = _load(path)
    for n in ("q", "k"):
        mine = O.l2norm(d[n], "bf16")
        rows_off = np.any(mine != d[n + "_l2"], axis=-1)
        assert rows_off.mean() < 0.02
        np.testing.assert_allclose(mine, d[n + "_l2"], rtol=2 ** -6, atol=0)
    out, state = _run_oracle(d)
    ref_out = O.from_bf16_bits(d["out"])
    assert np.abs(out - ref_out).max() < 2e-2
    assert np.linalg.norm(out - ref_out) / np.linalg.norm(ref_out) < 5e-3
    if state is not None:
        # The final state is dominated by the last few tokens, so a one-ulp change in
        # the inverse norm of one recent key moves it by up to ~0.5% (rel-L2) when q/k
        # are far from unit norm.
        assert np.linalg.norm(state - d["final_state"]) / np.linalg.norm(d["final_state"]) < 1e-2


def test_oracle_config1_sample():
    z = np.load(os.path.join(GOLDEN, "config1_fp32_B1_T256_H16.npz"))
    B, T, H, seed = int(z["B"]), int(z["T"]), int(z["H"]), int(z["seed"])
    q, k, v, g, beta, _ = O.make_inputs(B, T, H, seed=seed)
    import hashlib
    h = hashlib.sha256()
    for a in (q, k, v, g, beta):
        h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    assert h.hexdigest() == str(z["digest"]), "input generator drifted from the fixture"
    out, state = O.chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, output_final_state=True,
                                          use_qk_l2norm_in_kernel=True)
    s = int(z["stride"])
    np.testing.assert_allclose(out.reshape(-1)[::s], z["out_sample"], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(state.reshape(-1)[::s], z["state_sample"], rtol=1e-5, atol=2e-6)
    assert abs(out.astype(np.float64).sum() - float(z["out_sum"])) < 1e-3
    assert abs(state.astype(np.float64).sum() - float(z["state_sum"])) < 1e-3


def test_chunk_and_recurrent_oracles_agree():
    """Cross-oracle identity: the chunked and token-recurrent forms are the same map."""
    q, k, v, g, beta, s0 = O.make_inputs(2, 150, 2, seed=11, init_state_std=0.02, normalize_qk=False)
    oc, sc = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, acc=np.float64)
    orr, sr = O.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                           use_qk_l2norm_in_kernel=True, acc=np.float64)
    np.testing.assert_allclose(oc, orr, rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(sc, sr, rtol=1e-9, atol=1e-11)


def test_bf16_rounding_helper():
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0, 1e-30], dtype=np.float32)
    r = O.round_bf16(x)
    # every result is representable in bf16 and within half an ulp
    assert np.all((r.view(np.uint32) & 0xFFFF) == 0)
    assert np.all(np.abs(r - x) <= np.abs(x) * 2 ** -8)
    assert r[1] == 1.0  # tie rounds to even
