"""Sequence parallelism through the CUDA kernels.

One GPU: a sequence cut into shards (boundaries off the 64-token chunk grid) is
summarised shard by shard, the start states are composed on the host and every
shard is finished from its start state -- the concatenation must match one call
over the whole sequence and the oracle.  Two or more GPUs: the same over NCCL
with one shard per rank (tests/sp_nccl_worker.py under torchrun).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def dev(x, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda().to(dt)


@pytest.mark.parametrize("T,H,cuts,gscale", [
    (700, 4, [0, 150, 469, 700], 1.0),
    (700, 4, [0, 150, 469, 700], 0.05),
    # config 5's layout (H=16, bf16, time shards) at a length the oracle finishes in seconds
    (8192, 16, [0, 2731, 5461, 8192], 1.0),
])
def test_shards_composed_on_one_gpu_match_the_full_sequence(T, H, cuts, gscale):
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    from llms_from_scratch_b200.parallel import chunk_shard_finish, chunk_shard_summary, compose_start_states
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    q, k, v, g, beta, s0 = O.make_inputs(1, T, H, seed=12, in_dtype="bf16", init_state_std=0.02, normalize_qk=False)
    g = (g * gscale).astype(np.float32)
    tq, tk, tv = (dev(x, torch.bfloat16) for x in (q, k, v))
    tg, tb, ts = dev(g), dev(beta), dev(s0)
    shards = [(cuts[i], cuts[i + 1]) for i in range(3)]
    summaries = [chunk_shard_summary(tq[:, lo:hi], tk[:, lo:hi], tv[:, lo:hi], tg[:, lo:hi], tb[:, lo:hi],
                                     use_qk_l2norm_in_kernel=True) for lo, hi in shards]
    starts = compose_start_states([m for m, _, _ in summaries], [b for _, b, _ in summaries], ts)
    outs = []
    for (lo, hi), (_, _, ws), st in zip(shards, summaries, starts):
        o, s = chunk_shard_finish(tq[:, lo:hi], tk[:, lo:hi], tv[:, lo:hi], tg[:, lo:hi], tb[:, lo:hi], st, True,
                                  True, ws)
        outs.append(o)
    o_sp = torch.cat(outs, 1).float().cpu().numpy()
    o_full, s_full = fast_chunk_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=ts, output_final_state=True,
                                                 use_qk_l2norm_in_kernel=True)
    ro, rs = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                      use_qk_l2norm_in_kernel=True, in_dtype="bf16")
    for name, a, b in (("sp vs full", o_sp, o_full.float().cpu().numpy()), ("sp vs oracle", o_sp, ro)):
        assert np.abs(a - b).max() < 2e-2 and rel(a, b) < 5e-3, name
    assert rel(s.cpu().numpy(), rs) < 5e-3
    assert rel(starts[-1].cpu().numpy(), rs) < 5e-3


def test_shard_summary_matches_the_oracle_affine_map():
    """Weak decay so the transition is far from zero: S_end = M S_start + b."""
    from llms_from_scratch_b200.parallel import chunk_shard_summary
    q, k, v, g, beta, _ = O.make_inputs(1, 200, 2, seed=13, in_dtype="bf16", normalize_qk=False)
    g = (g * 0.05).astype(np.float32)
    M, b, _ = chunk_shard_summary(*(dev(x, torch.bfloat16) for x in (q, k, v)), dev(g), dev(beta),
                                  use_qk_l2norm_in_kernel=True)
    _, rb = O.chunk_gated_delta_rule(q, k, v, g, beta, output_final_state=True, use_qk_l2norm_in_kernel=True,
                                     in_dtype="bf16", acc=np.float64)
    eye = np.broadcast_to(np.eye(128), (1, 2, 128, 128)).copy()
    _, re = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=eye, output_final_state=True,
                                     use_qk_l2norm_in_kernel=True, in_dtype="bf16", acc=np.float64)
    assert rel(b.cpu().numpy(), rb) < 5e-3
    assert rel(M.cpu().numpy(), re - rb) < 1e-2  # the transition's running product passes through bf16 operands


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_over_nccl():
    n = min(torch.cuda.device_count(), 8)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, "tests", "sp_nccl_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True, cwd=ROOT,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "SP-OK" in r.stdout
