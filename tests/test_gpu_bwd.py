"""Backward of the chunked rule on the GPU (``chunk_gated_delta_rule_bwd`` through the C ABI).

The reference is inference-only; its torch forward is differentiable, and
``tests/golden/bwd_*.npz`` hold the gradients autograd takes through it (fp32
inputs).  The CUDA backward computes in fp32 and is held to those to 2e-4 of each
gradient's largest magnitude; with bf16 inputs (gradients returned in bf16) to the
oracle at the 16-bit path tolerance.  At the bench shape, where no CPU reference
finishes in seconds, the gradients must be finite and linear in (d_out, d_final_state).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle.gdn_bwd_oracle import chunk_gated_delta_rule_bwd as oracle_bwd

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = sorted(glob.glob(os.path.join(GOLDEN, "bwd_*.npz")))
NAMES = ("dq", "dk", "dv", "dg", "dbeta", "dh0")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda").to(dtype)


def rel_max(ours, ref):
    ours = np.asarray(ours, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(ours - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(p)[:-4] for p in CASES])
def test_bwd_matches_reference_autograd(path):
    from llms_from_scratch_b200 import chunk_gated_delta_rule_bwd
    z = {k: v for k, v in np.load(path).items()}
    grads = chunk_gated_delta_rule_bwd(dev(z["q"]), dev(z["k"]), dev(z["v"]), dev(z["g"]), dev(z["beta"]),
                                       dev(z["d_out"]), initial_state=dev(z.get("h0")),
                                       d_final_state=dev(z.get("d_final_state")),
                                       use_qk_l2norm_in_kernel=bool(z["l2norm"]))
    torch.cuda.synchronize()
    for name, g in zip(NAMES, grads):
        if name not in z:
            assert g is None
            continue
        err = rel_max(g.cpu().numpy(), z[name])
        assert err <= 2e-4, f"{name}: relative max error {err:.2e}"


def _inputs(B, T, H, seed, dtype=torch.bfloat16, state=True):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, H, 128, device="cuda", generator=gen).to(dtype)
    k = torch.randn(B, T, H, 128, device="cuda", generator=gen).to(dtype)
    v = torch.randn(B, T, H, 128, device="cuda", generator=gen).to(dtype)
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, H, device="cuda", generator=gen))
    h0 = 0.05 * torch.randn(B, H, 128, 128, device="cuda", generator=gen) if state else None
    do = torch.randn(B, T, H, 128, device="cuda", generator=gen).to(dtype)
    dhT = torch.randn(B, H, 128, 128, device="cuda", generator=gen)
    return q, k, v, g, beta, h0, do, dhT


@pytest.mark.parametrize("B,T,H", [(1, 300, 2), (2, 64, 1), (1, 65, 3)])
def test_bwd_bf16_matches_oracle(B, T, H):
    from llms_from_scratch_b200 import chunk_gated_delta_rule_bwd
    q, k, v, g, beta, h0, do, dhT = _inputs(B, T, H, seed=T + 7 * H)
    grads = chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=h0, d_final_state=dhT,
                                       use_qk_l2norm_in_kernel=True)
    assert grads[0].dtype == torch.bfloat16 and grads[3].dtype == torch.float32
    host = lambda x: x.float().cpu().numpy()  # noqa: E731
    ref = oracle_bwd(*(host(x) for x in (q, k, v, g, beta, do)), initial_state=host(h0), d_final_state=host(dhT),
                     use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    for name, ours, r in zip(NAMES, grads, ref):
        ours = ours.float().cpu().numpy()
        err = rel_max(ours, r)
        rl2 = float(np.linalg.norm(ours - r) / np.linalg.norm(r))
        assert err <= 1e-2 and rl2 <= 5e-3, f"{name}: relative max {err:.2e}, rel-L2 {rl2:.2e}"


@pytest.mark.parametrize("l2norm,with_state", [(True, False), (False, True)])
def test_bwd_bf16_without_state_or_l2norm_matches_oracle(l2norm, with_state):
    """The tensor-core path with no initial state and no final-state gradient, and with pre-normalised q/k
    (use_qk_l2norm_in_kernel=False)."""
    from llms_from_scratch_b200 import chunk_gated_delta_rule_bwd
    q, k, v, g, beta, h0, do, dhT = _inputs(1, 200, 2, seed=31 + int(l2norm), state=with_state)
    if not l2norm:
        q = torch.nn.functional.normalize(q.float(), dim=-1).to(torch.bfloat16)
        k = torch.nn.functional.normalize(k.float(), dim=-1).to(torch.bfloat16)
    dhT = dhT if with_state else None
    grads = chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=h0, d_final_state=dhT,
                                       use_qk_l2norm_in_kernel=l2norm)
    assert (grads[5] is None) == (not with_state)
    host = lambda x: None if x is None else x.float().cpu().numpy()  # noqa: E731
    ref = oracle_bwd(*(host(x) for x in (q, k, v, g, beta, do)), initial_state=host(h0), d_final_state=host(dhT),
                     use_qk_l2norm_in_kernel=l2norm, in_dtype="bf16")
    for name, ours, r in zip(NAMES[:5], grads[:5], ref[:5]):
        ours = ours.float().cpu().numpy()
        err = rel_max(ours, r)
        rl2 = float(np.linalg.norm(ours - r) / np.linalg.norm(r))
        assert err <= 1e-2 and rl2 <= 5e-3, f"{name}: relative max {err:.2e}, rel-L2 {rl2:.2e}"


def test_autograd_wrapper_equals_direct_call():
    from llms_from_scratch_b200 import chunk_gated_delta_rule, chunk_gated_delta_rule_bwd
    q, k, v, g, beta, h0, do, dhT = _inputs(1, 200, 2, seed=3, dtype=torch.float32)
    leaves = [x.clone().requires_grad_() for x in (q, k, v, g, beta, h0)]
    o, s = chunk_gated_delta_rule(*leaves[:5], initial_state=leaves[5], output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    ((o * do).sum() + (s * dhT).sum()).backward()
    direct = chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=h0, d_final_state=dhT,
                                        use_qk_l2norm_in_kernel=True)
    for name, leaf, d in zip(NAMES, leaves, direct):
        assert torch.equal(leaf.grad, d), name


def test_bwd_is_linear_at_bench_shape():
    """B=1, T=4096, H=16: grads(d1 + d2) = grads(d1) + grads(d2) (fp32 inputs, so every gradient is fp32)."""
    from llms_from_scratch_b200 import chunk_gated_delta_rule_bwd
    q, k, v, g, beta, h0, do1, dh1 = _inputs(1, 4096, 16, seed=11, dtype=torch.float32)
    _, _, _, _, _, _, do2, dh2 = _inputs(1, 4096, 16, seed=12, dtype=torch.float32)
    run = lambda do, dh: chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=h0, d_final_state=dh,  # noqa: E731
                                                    use_qk_l2norm_in_kernel=True)
    a, b, ab = run(do1, dh1), run(do2, dh2), run(do1 + do2, dh1 + dh2)
    for name, x, y, z in zip(NAMES, a, b, ab):
        assert bool(torch.isfinite(z).all()), name
        err = float((x + y - z).abs().max() / z.abs().max())
        assert err <= 1e-4, f"{name}: {err:.2e}"


def test_bwd_strided_views_and_empty():
    from llms_from_scratch_b200 import chunk_gated_delta_rule_bwd
    q, k, v, g, beta, h0, do, dhT = _inputs(1, 130, 2, seed=5)
    packed = torch.cat([q, k, v], dim=-1)  # q/k/v as channel views of one projection
    qv, kv, vv = packed[..., :128], packed[..., 128:256], packed[..., 256:]
    a = chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=h0, d_final_state=dhT,
                                   use_qk_l2norm_in_kernel=True)
    b = chunk_gated_delta_rule_bwd(qv, kv, vv, g, beta, do, initial_state=h0, d_final_state=dhT,
                                   use_qk_l2norm_in_kernel=True)
    for name, x, y in zip(NAMES, a, b):
        assert torch.equal(x, y), name
    e = chunk_gated_delta_rule_bwd(q[:, :0], k[:, :0], v[:, :0], g[:, :0], beta[:, :0], do[:, :0],
                                   initial_state=h0, d_final_state=dhT)
    assert torch.equal(e[5], dhT) and e[0].shape == (1, 0, 2, 128)

