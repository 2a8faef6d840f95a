"""Packed variable-length sequences (``cu_seqlens``) on the tensor-core chunk path.

Sequence n of a packed batch owns tokens cu_seqlens[n] .. cu_seqlens[n+1] and
its own state; the chunk tables are built on the device.  Each sequence's
chunks run the same kernels, on the same chunk boundaries, with the same
arithmetic as a separate call, so a packed call must reproduce per-sequence
``fast_chunk_gated_delta_rule`` calls bit for bit; one case also holds it to the
oracle.  The vLLM 0.22 adapter is held to the oracle, and to vLLM's own FLA
kernels where vLLM imports.
"""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

BF16_MAX_ABS, BF16_REL_L2 = 2e-2, 5e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _packed(lengths, H, seed, state_std=0.05):
    T = int(sum(lengths))
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(1, T, H, 128, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(1, T, H, 128, device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn(1, T, H, 128, device="cuda", generator=gen).to(torch.bfloat16)
    g = -torch.nn.functional.softplus(torch.randn(1, T, H, device="cuda", generator=gen))
    beta = torch.sigmoid(torch.randn(1, T, H, device="cuda", generator=gen))
    s0 = state_std * torch.randn(len(lengths), H, 128, 128, device="cuda", generator=gen)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device="cuda")
    return q, k, v, g, beta, s0, cu


@pytest.mark.parametrize("lengths,H", [
    ([0, 1, 63, 64, 65, 300], 4),            # empty, one token, chunk edges, ragged tail
    ([4096], 16),                             # one sequence: the bench shape
    ([1000, 0, 0, 2500, 7], 16),              # empty sequences between others
    ([17] * 40, 2),                           # many short sequences, one partial chunk each
    ([4096, 1, 8000, 64, 4223], 16),          # 16K tokens of ragged lengths
])
def test_packed_call_equals_per_sequence_calls(lengths, H):
    from llms_from_scratch_b200 import chunk_gated_delta_rule_varlen, fast_chunk_gated_delta_rule
    q, k, v, g, beta, s0, cu = _packed(lengths, H, seed=len(lengths) * 100 + H)
    o, s = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, output_final_state=True,
                                         use_qk_l2norm_in_kernel=True)
    assert o.shape == (1, sum(lengths), H, 128) and s.shape == (len(lengths), H, 128, 128)
    edges = [0] + list(np.cumsum(lengths))
    for n, (a, b) in enumerate(zip(edges[:-1], edges[1:])):
        on, sn = fast_chunk_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                             initial_state=s0[n:n + 1], output_final_state=True,
                                             use_qk_l2norm_in_kernel=True)
        assert torch.equal(o[:, a:b], on), f"sequence {n} (tokens {a}..{b}): outputs differ"
        assert torch.equal(s[n:n + 1], sn), f"sequence {n}: final states differ"
    from llms_from_scratch_b200 import _lib
    assert _lib.load().gdn_device_error(0) == 0


def test_packed_call_matches_oracle():
    from llms_from_scratch_b200 import chunk_gated_delta_rule_varlen
    lengths, H = [5, 130, 0, 64], 2
    q, k, v, g, beta, s0, cu = _packed(lengths, H, seed=7)
    o, s = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, output_final_state=True,
                                         use_qk_l2norm_in_kernel=True)
    o, s = o.float().cpu().numpy(), s.cpu().numpy()
    host = [x.float().cpu().numpy() for x in (q, k, v, g, beta, s0)]
    edges = [0] + list(np.cumsum(lengths))
    for n, (a, b) in enumerate(zip(edges[:-1], edges[1:])):
        if a == b:
            np.testing.assert_array_equal(s[n], host[5][n])  # an empty sequence passes its state through
            continue
        ro, rs = O.chunk_gated_delta_rule(*(x[:, a:b] for x in host[:5]), initial_state=host[5][n:n + 1],
                                          output_final_state=True, use_qk_l2norm_in_kernel=True, in_dtype="bf16")
        for ours, ref in ((o[:, a:b], ro), (s[n:n + 1], rs)):
            err = float(np.abs(ours - ref).max())
            rel = float(np.linalg.norm(ours - ref) / np.linalg.norm(ref))
            assert err <= BF16_MAX_ABS and rel <= BF16_REL_L2, f"sequence {n}: max-abs {err:.3e}, rel-L2 {rel:.3e}"


def test_no_final_state_and_reused_workspace():
    from llms_from_scratch_b200 import chunk_gated_delta_rule_varlen, chunk_varlen_workspace_bytes
    lengths, H = [200, 77], 4
    q, k, v, g, beta, s0, cu = _packed(lengths, H, seed=3)
    ws = torch.empty(chunk_varlen_workspace_bytes(sum(lengths), len(lengths), H), dtype=torch.uint8, device="cuda")
    o1, s1 = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, workspace=ws,
                                           use_qk_l2norm_in_kernel=True)
    o2, s2 = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, output_final_state=True,
                                           workspace=ws, use_qk_l2norm_in_kernel=True)
    assert s1 is None and s2 is not None
    assert bool(torch.isfinite(o1).all()) and torch.equal(o1, o2)


@pytest.mark.parametrize("offsets", [
    [0, 50, 30, 100],   # decreasing
    [0, 40, 90],        # ends before T
    [3, 40, 100],       # does not start at 0
])
def test_invalid_offsets_set_the_device_error_bit(offsets):
    """Offsets are read on the device only; a bad set makes every sequence empty (no kernel reads
    past the packed tensors) and sets bit 8 of the device error word."""
    from llms_from_scratch_b200 import _lib, chunk_gated_delta_rule_varlen
    lib = _lib.load()
    assert lib.gdn_device_error(1) == 0
    q, k, v, g, beta, s0, _ = _packed([100], 2, seed=11)
    cu = torch.tensor(offsets, dtype=torch.int32, device="cuda")
    s0 = s0.expand(len(offsets) - 1, -1, -1, -1).contiguous()
    _, s = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, output_final_state=True)
    torch.cuda.synchronize()
    assert lib.gdn_device_error(1) == 8
    assert torch.equal(s, s0)
    assert lib.gdn_device_error(0) == 0
    # the context is intact: a valid call right after runs normally
    good = torch.tensor([0, 60, 100], dtype=torch.int32, device="cuda")
    chunk_gated_delta_rule_varlen(q, k, v, g, beta, good, initial_state=s0[:2], output_final_state=True)
    torch.cuda.synchronize()
    assert lib.gdn_device_error(0) == 0


def _vllm_layout_inputs(lengths, H, seed):
    q, k, v, g, beta, s0, cu = _packed(lengths, H, seed, state_std=0.1)
    return q, k, v, g, beta, s0.transpose(-1, -2).contiguous(), cu  # vLLM keeps the state as [N, H, V, K]


def test_vllm_adapter_contract_against_oracle():
    from llms_from_scratch_b200 import vllm_adapter
    lengths, H = [70, 0, 129], 2
    q, k, v, g, beta, s_vk, cu = _vllm_layout_inputs(lengths, H, seed=5)
    core = torch.full((sum(lengths), H, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    o, s = vllm_adapter.forward(None, q, k, v, g, beta.to(torch.bfloat16), s_vk, True, cu_seqlens=cu,
                                use_qk_l2norm_in_kernel=True, core_attn_out=core)
    assert s.shape == (len(lengths), H, 128, 128) and s.dtype == torch.float32
    assert torch.equal(core, o.squeeze(0))
    host = [x.float().cpu().numpy() for x in (q, k, v, g, beta.to(torch.bfloat16))]
    s_kv = s_vk.transpose(-1, -2).cpu().numpy()
    o, s = o.float().cpu().numpy(), s.transpose(-1, -2).cpu().numpy()
    edges = [0] + list(np.cumsum(lengths))
    for n, (a, b) in enumerate(zip(edges[:-1], edges[1:])):
        if a == b:
            np.testing.assert_array_equal(s[n], s_kv[n])
            continue
        ro, rs = O.chunk_gated_delta_rule(*(x[:, a:b] for x in host), initial_state=s_kv[n:n + 1],
                                          output_final_state=True, use_qk_l2norm_in_kernel=True, in_dtype="bf16")
        for ours, ref in ((o[:, a:b], ro), (s[n:n + 1], rs)):
            err = float(np.abs(ours - ref).max())
            rel = float(np.linalg.norm(ours - ref) / np.linalg.norm(ref))
            assert err <= BF16_MAX_ABS and rel <= BF16_REL_L2, f"sequence {n}: max-abs {err:.3e}, rel-L2 {rel:.3e}"
    # a single sequence without cu_seqlens and without a start state
    o1, s1 = vllm_adapter.forward(None, q[:, :70], k[:, :70], v[:, :70], g[:, :70], beta[:, :70], None, False)
    assert s1 is None and o1.shape == (1, 70, H, 128)


def test_vllm_adapter_agrees_with_vllm_fla():
    """The adapter against vLLM 0.22's own FLA prefill on the same packed batch: both approximate the
    same fp32 result from bf16 inputs, so they agree to twice the path tolerance; a state read in the
    wrong layout or a sequence boundary misplaced would differ by O(1)."""
    try:
        from vllm.model_executor.layers.fla.ops import chunk_gated_delta_rule as fla
    except Exception as e:  # vLLM absent or not importable on this box
        pytest.skip(f"vLLM FLA not importable: {e}")
    from llms_from_scratch_b200 import vllm_adapter
    lengths, H = [300, 5, 1024, 64], 16
    q, k, v, g, beta, s_vk, cu = _vllm_layout_inputs(lengths, H, seed=9)
    ro, rs = fla(q=q, k=k, v=v, g=g, beta=beta, initial_state=s_vk.clone(), output_final_state=True,
                 cu_seqlens=cu, use_qk_l2norm_in_kernel=True)
    o, s = vllm_adapter.forward(None, q, k, v, g, beta, s_vk, True, cu_seqlens=cu, use_qk_l2norm_in_kernel=True)
    for ours, ref, what in ((o.float(), ro.float(), "out"), (s, rs.float(), "state")):
        err = float((ours - ref).abs().max())
        rel = float((ours - ref).norm() / ref.norm())
        assert err <= 2 * BF16_MAX_ABS and rel <= 2 * BF16_REL_L2, f"{what}: max-abs {err:.3e}, rel-L2 {rel:.3e}"
