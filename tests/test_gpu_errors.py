"""Device-side failures reach the caller as exceptions, and the context survives them.

Every wait inside the kernels is bounded: one that runs out sets a bit in the
library's device error word and the kernel returns.  The ops poll a page-locked
host mirror of that word before each launch, so the failure surfaces as a
``GDNError`` (``GDN_ERR_KERNEL``) at the next op on the device, with no
synchronisation on the hot path.  Here a wait is made to run out on purpose
(``gdn_selftest_bounded_wait``: a barrier nothing arms, with a 1 ms limit) and
packed-sequence offsets are made invalid; neither faults the GPU.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _small_call():
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    q, k, v, g, beta, s0 = O.make_inputs(1, 130, 2, seed=21, in_dtype="bf16", init_state_std=0.02)
    d = lambda x, dt=torch.float32: torch.from_numpy(x).cuda().to(dt)  # noqa: E731
    o, s = fast_chunk_gated_delta_rule(d(q, torch.bfloat16), d(k, torch.bfloat16), d(v, torch.bfloat16), d(g),
                                       d(beta), initial_state=d(s0), output_final_state=True,
                                       use_qk_l2norm_in_kernel=True)
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    return o.float().cpu().numpy(), s.cpu().numpy(), ro, rs


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_timed_out_wait_raises_at_the_next_call_and_the_context_survives():
    from llms_from_scratch_b200 import _lib
    from llms_from_scratch_b200.ops import check_device_errors
    lib = _lib.load()
    check_device_errors(sync=True)  # nothing pending
    assert lib.gdn_device_error_pending() == 0
    stream = torch.cuda.current_stream()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    _lib.check(lib.gdn_selftest_bounded_wait(1_000_000, ctypes.c_void_p(stream.cuda_stream)))
    t1.record(stream)
    torch.cuda.synchronize()  # the kernel returns on its own: no hang
    waited_ms = t0.elapsed_time(t1)
    assert 0.5 <= waited_ms < 1000.0, f"the bounded wait took {waited_ms:.3f} ms"
    # the mirror shows the bit without any device synchronisation
    assert lib.gdn_device_error_pending() & 16
    with pytest.raises(_lib.GDNError) as exc:
        _small_call()
    assert exc.value.status == _lib.GDN_ERR_KERNEL and "0x10" in str(exc.value)
    # raising cleared the word: the next call runs and matches the oracle
    assert lib.gdn_device_error_pending() == 0
    o, s, ro, rs = _small_call()
    assert np.abs(o - ro).max() < 2e-2 and _rel(o, ro) < 5e-3
    assert _rel(s, rs) < 5e-3
    torch.cuda.synchronize()
    assert lib.gdn_device_error(0) == 0


def test_invalid_offsets_raise_at_the_next_call():
    from llms_from_scratch_b200 import _lib, chunk_gated_delta_rule_varlen
    from llms_from_scratch_b200.ops import check_device_errors
    check_device_errors()
    torch.manual_seed(3)
    T, H = 100, 2
    q = torch.nn.functional.normalize(torch.randn(1, T, H, 128, device="cuda"), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(1, T, H, 128, device="cuda"), dim=-1).bfloat16()
    v = torch.randn(1, T, H, 128, device="cuda").bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(1, T, H, device="cuda"))
    beta = torch.rand(1, T, H, device="cuda")
    bad = torch.tensor([0, 90, 40], dtype=torch.int32, device="cuda")  # decreasing
    chunk_gated_delta_rule_varlen(q, k, v, g, beta, bad, output_final_state=True)
    torch.cuda.synchronize()
    with pytest.raises(_lib.GDNError) as exc:
        check_device_errors()
    assert exc.value.status == _lib.GDN_ERR_KERNEL and "cu_seqlens" in str(exc.value)
    good = torch.tensor([0, 60, 100], dtype=torch.int32, device="cuda")
    chunk_gated_delta_rule_varlen(q, k, v, g, beta, good, output_final_state=True)
    torch.cuda.synchronize()
    check_device_errors()


def test_self_test_rejects_out_of_range_limits_without_launching():
    from llms_from_scratch_b200 import _lib
    lib = _lib.load()
    n0 = lib.gdn_launch_count()
    for bad in (0, 999, 200_000_000):
        assert lib.gdn_selftest_bounded_wait(bad, None) == _lib.GDN_ERR_INVALID_ARGUMENT
    assert lib.gdn_launch_count() == n0


def test_workspace_on_the_wrong_device_is_rejected_before_any_launch():
    from llms_from_scratch_b200 import _lib, fast_chunk_gated_delta_rule
    lib = _lib.load()
    x = torch.randn(1, 70, 2, 128, device="cuda").bfloat16()
    g = torch.zeros(1, 70, 2, device="cuda")
    n0 = lib.gdn_launch_count()
    with pytest.raises(RuntimeError, match="workspace"):
        fast_chunk_gated_delta_rule(x, x, x, g, g, workspace=torch.empty(1 << 24, dtype=torch.uint8))
    assert lib.gdn_launch_count() == n0
