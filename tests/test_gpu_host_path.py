"""The host-buffer entry point (gdn_chunk_gated_delta_rule_host): CPU tensors in,
CPU tensors out, copies pipelined in time slices against the compute.

Its slices start on chunk boundaries and pass the state on in fp32, so it must
reproduce one device call on the whole sequence bit for bit; the device call
itself is held to the oracle by test_gpu_parity.py, and one case here checks the
host path against the oracle directly.
"""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _inputs(B, T, H, dtype, seed, pin=True, with_state=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, 128, generator=g).to(dtype)
    k = torch.randn(B, T, H, 128, generator=g).to(dtype)
    v = torch.randn(B, T, H, 128, generator=g).to(dtype)
    gg = -torch.nn.functional.softplus(torch.randn(B, T, H, generator=g))
    bb = torch.rand(B, T, H, generator=g)
    s0 = 0.05 * torch.randn(B, H, 128, 128, generator=g) if with_state else None
    xs = [q, k, v, gg, bb] + ([s0] if with_state else [])
    if pin:
        xs = [x.pin_memory() for x in xs]
    return xs if with_state else xs + [None]


def _device_call(q, k, v, g, b, s0):
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    d = [x.cuda() for x in (q, k, v, g, b)]
    o, s = fast_chunk_gated_delta_rule(*d, initial_state=None if s0 is None else s0.cuda(), output_final_state=True,
                                       use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    return o.cpu(), s.cpu()


@pytest.mark.parametrize("B,T,H,dtype,slice_tokens,pin,with_state", [
    (1, 4096, 16, torch.bfloat16, 0, True, True),      # the bench shape, default slices (4 x 1024)
    (2, 1000, 4, torch.bfloat16, 256, True, True),     # ragged last slice, batch stride
    (3, 130, 2, torch.bfloat16, 64, True, False),      # 3 slices, the last of 2 tokens, zero start state
    (1, 700, 3, torch.float32, 128, True, True),       # fp32 inputs: the CUDA-core kernels per slice
    (2, 333, 2, torch.bfloat16, 0, False, True),       # pageable host memory (copies serialise)
    (1, 64, 1, torch.bfloat16, 0, True, True),         # a single chunk
])
def test_host_path_equals_one_device_call(B, T, H, dtype, slice_tokens, pin, with_state):
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    q, k, v, g, b, s0 = _inputs(B, T, H, dtype, seed=B * 1000 + T, pin=pin, with_state=with_state)
    o, s = fast_chunk_gated_delta_rule(q, k, v, g, b, initial_state=s0, output_final_state=True,
                                       use_qk_l2norm_in_kernel=True, slice_tokens=slice_tokens)
    assert o.device.type == "cpu" and s.device.type == "cpu"
    assert o.dtype == dtype and s.dtype == torch.float32
    ref_o, ref_s = _device_call(q, k, v, g, b, s0)
    assert torch.equal(o, ref_o)
    assert torch.equal(s, ref_s)


def test_host_path_matches_the_oracle():
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    q, k, v, g, b, s0 = O.make_inputs(2, 200, 2, seed=21, in_dtype="bf16", init_state_std=0.02,
                                      normalize_qk=False)
    t = [torch.from_numpy(x).to(torch.bfloat16) for x in (q, k, v)]
    o, s = fast_chunk_gated_delta_rule(*t, torch.from_numpy(g), torch.from_numpy(b),
                                       initial_state=torch.from_numpy(s0), output_final_state=True,
                                       use_qk_l2norm_in_kernel=True, slice_tokens=64)
    ref_o, ref_s = O.chunk_gated_delta_rule(q, k, v, g, b, initial_state=s0, output_final_state=True,
                                            use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    for ours, ref in ((o.float().numpy(), ref_o), (s.numpy(), ref_s)):  # bf16 tolerance of the path
        ref = np.asarray(ref, np.float32)
        assert float(np.abs(ours - ref).max()) <= 2e-2
        assert np.linalg.norm(ours - ref) / np.linalg.norm(ref) <= 5e-3


def test_host_path_empty_sequence_and_no_state_output():
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    q, k, v, g, b, s0 = _inputs(1, 0, 2, torch.bfloat16, seed=3)
    o, s = fast_chunk_gated_delta_rule(q, k, v, g, b, initial_state=s0, output_final_state=True)
    assert o.shape == (1, 0, 2, 128)
    assert torch.equal(s, s0)
    q, k, v, g, b, s0 = _inputs(1, 100, 2, torch.bfloat16, seed=4)
    o, s = fast_chunk_gated_delta_rule(q, k, v, g, b, initial_state=s0, output_final_state=False,
                                       use_qk_l2norm_in_kernel=True)
    assert s is None
    ref_o, _ = _device_call(q, k, v, g, b, s0)
    assert torch.equal(o, ref_o)


def test_host_path_orders_against_the_callers_stream():
    """Work queued on the caller's stream before the call finishes before its copies read host memory."""
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    q, k, v, g, b, s0 = _inputs(1, 512, 4, torch.bfloat16, seed=5)
    ref_o, _ = _device_call(q, k, v, g, b, s0)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        big = torch.empty(64 << 20, device="cuda")
        for _ in range(20):  # keep the stream busy, then write q from the device
            big.mul_(1.0)
        q_dev = q.cuda(non_blocking=True)
        scratch = torch.zeros_like(q).pin_memory()
        scratch.copy_(q_dev, non_blocking=True)
        o, _ = fast_chunk_gated_delta_rule(scratch, k, v, g, b, initial_state=s0, output_final_state=True,
                                           use_qk_l2norm_in_kernel=True)
    assert torch.equal(o, ref_o)
