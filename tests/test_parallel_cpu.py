"""Host logic of the multi-GPU paths, on CPU.

The shard summaries and finishes are replaced by CPU stand-ins built on the
oracle, so the exchange (gloo all_gather over two ranks), the start-state
composition and the failure path run without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import gdn_oracle as O

D = 128


def _oracle_run(q, k, v, g, beta, start, acc=np.float64):
    o, s = O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=start, output_final_state=True,
                                    use_qk_l2norm_in_kernel=True, acc=acc)
    return np.asarray(o, np.float64), np.asarray(s, np.float64)


def oracle_summary(q, k, v, g, beta, use_l2):
    """(transition, local_state, None) of a shard: S_end = M S_start + b, from two oracle runs."""
    qn, kn, vn, gn, bn = (x.numpy() for x in (q, k, v, g, beta))
    B, T, H, _ = qn.shape
    _, b = _oracle_run(qn, kn, vn, gn, bn, None)
    eye = np.broadcast_to(np.eye(D), (B, H, D, D)).copy()
    _, s_eye = _oracle_run(qn, kn, vn, gn, bn, eye)
    return torch.from_numpy(s_eye - b), torch.from_numpy(b), None


def oracle_finish(q, k, v, g, beta, start, ofs, use_l2, ws):
    qn, kn, vn, gn, bn = (x.numpy() for x in (q, k, v, g, beta))
    o, s = _oracle_run(qn, kn, vn, gn, bn, None if start is None else start.numpy())
    return torch.from_numpy(o), (torch.from_numpy(s) if ofs else None)


def _shards(T, P):
    cuts = [T * i // P for i in range(P + 1)]
    return [(cuts[i], cuts[i + 1]) for i in range(P)]


def test_compose_start_states_matches_prefix_states():
    """(The oracle rounds a start state to fp32, as the reference casts it to the value dtype.)"""
    from llms_from_scratch_b200.parallel import compose_start_states
    q, k, v, g, beta, s0 = O.make_inputs(1, 300, 2, seed=4, init_state_std=0.02, normalize_qk=False)
    t = [torch.from_numpy(x) for x in (q, k, v, g, beta)]
    Ms, bs = [], []
    shards = _shards(300, 3)
    for lo, hi in shards:
        M, b, _ = oracle_summary(*(x[:, lo:hi] for x in t), True)
        Ms.append(M)
        bs.append(b)
    starts = compose_start_states(Ms, bs, torch.from_numpy(s0).double())
    for r, (lo, hi) in enumerate(shards):
        if lo == 0:
            ref = s0
        else:
            _, ref = _oracle_run(q[:, :lo], k[:, :lo], v[:, :lo], g[:, :lo], beta[:, :lo], s0)
        np.testing.assert_allclose(starts[r].numpy(), ref, rtol=1e-6, atol=1e-9)
    _, full_state = _oracle_run(q, k, v, g, beta, s0)
    np.testing.assert_allclose(starts[-1].numpy(), full_state, rtol=1e-6, atol=1e-9)


def test_shard_batch_covers_every_sequence_once():
    from llms_from_scratch_b200.parallel import shard_batch
    x = torch.arange(10)
    parts = [shard_batch(x, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts), x)
    assert [len(p) for p in parts] == [2, 3, 2, 3]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _sp_worker(rank, world, port, inputs, s0, results):
    import torch.distributed as dist

    from llms_from_scratch_b200.parallel import sequence_parallel_chunk_gated_delta_rule
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        T = inputs[0].shape[1]
        lo, hi = _shards(T, world)[rank]
        shard = [x[:, lo:hi] for x in inputs]
        o, s = sequence_parallel_chunk_gated_delta_rule(*shard, initial_state=s0, output_final_state=True,
                                                        use_qk_l2norm_in_kernel=True, summary_fn=oracle_summary,
                                                        finish_fn=oracle_finish)
        results[rank] = (o.numpy(), s.numpy())
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_two_gloo_ranks_match_the_full_sequence():
    q, k, v, g, beta, s0 = O.make_inputs(1, 200, 2, seed=8, init_state_std=0.02, normalize_qk=False)
    inputs = [torch.from_numpy(x) for x in (q, k, v, g, beta)]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_sp_worker, args=(2, _free_port(), inputs, torch.from_numpy(s0).double(), results),
                           nprocs=2, join=True, start_method="spawn")
        res = dict(results)
    out = np.concatenate([res[0][0], res[1][0]], axis=1)
    ref_o, ref_s = _oracle_run(q, k, v, g, beta, s0)
    np.testing.assert_allclose(out, ref_o, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(res[1][1], ref_s, rtol=1e-6, atol=1e-9)


def _failing_worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results[1] = "left before the exchange"
        return  # this rank never joins the all_gather
    try:
        packed = torch.zeros(2, 4)
        dist.all_gather([torch.empty_like(packed) for _ in range(world)], packed)
        results[0] = "exchange completed"
    except Exception as e:  # the short process-group timeout ends the collective with an error
        results[0] = "error: " + type(e).__name__


@pytest.mark.timeout(120)
def test_a_rank_that_leaves_makes_the_exchange_fail_not_hang():
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, results)) for r in range(2)]
        for p_ in procs:
            p_.start()
        for p_ in procs:
            p_.join(timeout=90)
        alive = [p_.is_alive() for p_ in procs]
        for p_ in procs:
            if p_.is_alive():
                p_.kill()
        res = dict(results)
    assert not any(alive), "a rank hung past the process-group timeout"
    assert res.get(1) == "left before the exchange"
    assert str(res.get(0, "")).startswith("error"), res

