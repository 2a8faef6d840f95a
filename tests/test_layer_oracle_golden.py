"""The layer oracle (oracle/gdn_layer_oracle.py) against fixtures made by the
reference's own torch code (tests/golden/make_golden_layer.py).

Every bf16 output of the reference is reproduced bit for bit; g (fp32) to 1e-6
relative (the fp32 exp/log1p of numpy and torch differ in the last bits).
"""
import glob
import os

import numpy as np
import pytest

from oracle import gdn_layer_oracle as L

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "layer_conv_T*.npz"))))
def test_prefill_conv_matches_reference_bitwise(path):
    z = np.load(path)
    y, s = L.causal_conv1d_silu(z["x"], z["weight"])
    np.testing.assert_array_equal(y, z["out"])
    np.testing.assert_array_equal(s, z["conv_state"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "layer_convupd_*.npz"))))
def test_decode_conv_update_matches_reference_bitwise(path):
    z = np.load(path)
    y, s = L.causal_conv1d_update(z["x"], z["conv_state"], z["weight"])
    np.testing.assert_array_equal(y, z["out"])
    np.testing.assert_array_equal(s, z["new_state"])


def test_gates_match_reference():
    z = _load("layer_gates.npz")
    g, beta = L.gates(z["a"], z["b"], z["A_log"], z["dt_bias"])
    np.testing.assert_array_equal(beta, z["beta"])
    np.testing.assert_allclose(g, z["g"], rtol=1e-6, atol=0)
    assert (z["a"] + z["dt_bias"][None, None, :] > 20).any()  # the softplus threshold branch is covered


def test_rms_norm_gated_matches_reference_bitwise():
    z = _load("layer_rmsnorm_gated.npz")
    out = L.rms_norm_gated(z["x"], z["gate"], z["weight"], float(z["eps"]))
    np.testing.assert_array_equal(out, z["out"])


def test_decode_updates_chain_into_the_prefill_conv():
    """Token-by-token decode from a zero state equals the prefill convolution (the cache contract)."""
    rng = np.random.default_rng(5)
    from oracle.gdn_oracle import round_bf16
    x = round_bf16(rng.standard_normal((2, 9, 24), dtype=np.float32))
    w = round_bf16(rng.standard_normal((24, 4), dtype=np.float32) * np.float32(0.5))
    y, state = L.causal_conv1d_silu(x, w)
    s = np.zeros((2, 24, 4), np.float32)
    outs = []
    for t in range(9):
        o, s = L.causal_conv1d_update(x[:, t:t + 1], s, w)
        outs.append(o)
    np.testing.assert_array_equal(np.concatenate(outs, axis=1), y)
    np.testing.assert_array_equal(s, state)
