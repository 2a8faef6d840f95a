"""The backward oracle reproduces the reference's own autograd gradients.

``tests/golden/bwd_*.npz`` hold the gradients autograd takes through the reference's
``torch_chunk_gated_delta_rule`` (made by ``make_golden_bwd.py``).  That function casts
its inputs to float32 (qwen3_5_transformers.py:122-127), so those gradients carry fp32
round-off (~1e-6 relative); the hand-written float64 chunk backward of
``oracle/gdn_bwd_oracle.py`` must match them to within 2e-5 of each gradient's largest
magnitude (a wrong term would be off by order one)."""
import glob
import os

import numpy as np
import pytest

from oracle.gdn_bwd_oracle import chunk_gated_delta_rule_bwd

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(glob.glob(os.path.join(GOLDEN, "bwd_*.npz")))


def load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def test_fixtures_present():
    assert len(CASES) >= 5


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(p)[:-4] for p in CASES])
def test_oracle_matches_reference_autograd(path):
    z = load(path)
    got = chunk_gated_delta_rule_bwd(z["q"], z["k"], z["v"], z["g"], z["beta"], z["d_out"],
                                     initial_state=z.get("h0"), d_final_state=z.get("d_final_state"),
                                     use_qk_l2norm_in_kernel=bool(z["l2norm"]))
    for name, ours in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), got):
        if name == "dh0" and "dh0" not in z:
            continue
        ref = z[name]
        err = np.abs(ours - ref).max() / max(np.abs(ref).max(), 1e-300)
        assert err < 2e-5, f"{name}: relative max error {err:.2e}"
