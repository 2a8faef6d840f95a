"""The allocation-free chunked forward (gdn_chunk_gated_delta_rule_noalloc).

It serves callers that cannot allocate device memory when they run the op
(runtimes that plan every buffer ahead of time, plugins whose framework owns
all allocations): they pass inputs and outputs only, and the workspace comes
from a fixed 64 MiB array inside the library.  These tests call it through
the C ABI and check it against the regular entry point, which takes a
caller-allocated workspace, on two calls in a row -- the second call runs on
scratch the first one left behind.  Collected last so that a stop-at-first-
failure run has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

BF16_MAX_ABS, BF16_REL_L2, FP32_MAX_ABS = 2e-2, 5e-3, 1e-4


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llms_from_scratch_b200 import _lib
    return _lib.load()


def _inputs(B, T, H, seed, dtype):
    in_dtype = {torch.bfloat16: "bf16", torch.float32: "fp32"}[dtype]
    q, k, v, g, beta, s0 = O.make_inputs(B, T, H, seed=seed, in_dtype=in_dtype, init_state_std=0.02,
                                         normalize_qk=False)
    t = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dt)  # noqa: E731
    return t(q, dtype), t(k, dtype), t(v, dtype), t(g), t(beta), t(s0)


def _noalloc(lib, q, k, v, g, beta, s0):
    from llms_from_scratch_b200 import _lib
    from llms_from_scratch_b200.ops import _desc
    B, T, H, D = q.shape
    out = torch.empty((B, T, H, D), dtype=q.dtype, device=q.device)
    st = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, g, beta, out))
    rc = lib.gdn_chunk_gated_delta_rule_noalloc(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg), ctypes.byref(db), 64,
        s0.data_ptr(), 1, 1, ctypes.byref(do), st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    return out, st


def _close(a, b, dtype):
    a = a.float().cpu().numpy()
    b = b.float().cpu().numpy()
    err = float(np.abs(a - b).max())
    if dtype == torch.float32:
        assert err <= FP32_MAX_ABS, err
    else:
        rel = float(np.linalg.norm(a - b) / np.linalg.norm(b))
        assert err <= BF16_MAX_ABS and rel <= BF16_REL_L2, (err, rel)


def test_noalloc_matches_workspace_entry_point_on_two_calls(lib):
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    # two calls in a row with different shapes and dtypes: the second reuses the
    # scratch the first one left behind
    for (B, T, H, seed, dtype) in [(1, 1000, 16, 1, torch.bfloat16), (2, 130, 3, 2, torch.float32)]:
        q, k, v, g, beta, s0 = _inputs(B, T, H, seed, dtype)
        out_n, st_n = _noalloc(lib, q, k, v, g, beta, s0)
        out_w, st_w = fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                                  use_qk_l2norm_in_kernel=True)
        torch.cuda.synchronize()
        _close(out_n, out_w, dtype)
        _close(st_n, st_w, dtype)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch(lib):
    from llms_from_scratch_b200 import _lib
    B, T, H = 1, 4096, 16
    need = lib.gdn_chunk_workspace_bytes(B, T, H, 128, 128, _lib.GDN_BF16)
    assert need > _lib.GDN_NOALLOC_SCRATCH_BYTES
    q, k, v, g, beta, s0 = _inputs(B, T, H, 3, torch.bfloat16)
    n0 = lib.gdn_launch_count()
    with pytest.raises(_lib.GDNError, match="too large for the fixed scratch"):
        _noalloc(lib, q, k, v, g, beta, s0)
    assert lib.gdn_launch_count() == n0
