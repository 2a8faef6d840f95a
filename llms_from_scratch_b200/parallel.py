"""Multi-GPU execution of the chunked gated delta rule.

Two partitions, as the path allows:

* **Batch x head** (``shard_batch``): sequences are independent, so each rank
  runs its own slice of the batch with no collective.
* **Sequence parallel** (``sequence_parallel_chunk_gated_delta_rule``): one
  long sequence is cut into contiguous time shards, one per rank.  The state at
  the end of a shard is an affine map of the state at its start,
  ``S_end = M_p S_start + b_p``; each rank computes its ``(M_p, b_p)``
  (``gdn_chunk_sp_summary``), one ``all_gather`` over NCCL exchanges them, each
  rank composes its own start state from the shards before it, and finishes its
  shard from that state (``gdn_chunk_sp_finish``, reusing the chunk records the
  summary left in the workspace).  The reference runs the whole sequence on one
  device (qwen3_5_cutedsl_kernels.py:427-453).

The exchange moves ``2 x B x H x 128 x 128`` fp32 per rank (2 MiB at B=1, H=16)
into each rank's own memory before use.
"""

from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _DTYPES, _as_kernel_tensor, _desc, _raise_pending, _workspace

D = 128


def shard_batch(x: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """Contiguous slice ``rank`` of ``world`` along ``dim`` (batch x head sharding)."""
    n = x.shape[dim]
    lo, hi = n * rank // world, n * (rank + 1) // world
    return x.narrow(dim, lo, hi - lo)


def compose_start_states(transitions: Sequence[torch.Tensor], local_states: Sequence[torch.Tensor],
                         initial_state: Optional[torch.Tensor]) -> List[torch.Tensor]:
    """Start state of every shard: ``S_0 = initial``, ``S_{r+1} = M_r S_r + b_r`` (fp32)."""
    S = (torch.zeros_like(local_states[0]) if initial_state is None
         else initial_state.to(torch.float32).to(local_states[0].device))
    starts = []
    for M, b in zip(transitions, local_states):
        starts.append(S)
        S = torch.matmul(M.to(torch.float32), S) + b.to(torch.float32)
    starts.append(S)
    return starts


def _inputs(query, key, value, g, beta):
    q = _as_kernel_tensor(query, "query", 4)
    k = _as_kernel_tensor(key, "key", 4)
    v = _as_kernel_tensor(value, "value", 4)
    gg = _as_kernel_tensor(g, "g", 3)
    bb = _as_kernel_tensor(beta, "beta", 3)
    return q, k, v, gg, bb


def shard_workspace(query: torch.Tensor) -> torch.Tensor:
    B, T, H, Dk = query.shape
    n = _lib.load().gdn_chunk_workspace_bytes(B, T, H, Dk, D, _DTYPES.get(query.dtype, _lib.GDN_F32))
    return torch.empty((max(n, 1),), dtype=torch.uint8, device=query.device)


def chunk_shard_summary(query, key, value, g, beta, use_qk_l2norm_in_kernel: bool = False,
                        workspace: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(transition [B,H,Dk,Dk], local_state [B,H,Dk,Dv], workspace)`` of one time shard."""
    q, k, v, gg, bb = _inputs(query, key, value, g, beta)
    B, T, H, _ = q.shape
    lib = _lib.load()
    need = lib.gdn_chunk_workspace_bytes(B, T, H, D, D, _DTYPES.get(q.dtype, _lib.GDN_F32))
    workspace = _workspace(workspace, need, q.device)
    M = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    b = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device)
    with torch.cuda.device(q.device):
        _raise_pending(lib, q.device)
        dq, dk, dv, dg, db = (_desc(x) for x in (q, k, v, gg, bb))
        rc = lib.gdn_chunk_sp_summary(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg),
                                      ctypes.byref(db), 64, int(bool(use_qk_l2norm_in_kernel)), M.data_ptr(),
                                      b.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                      torch.cuda.current_stream(q.device).cuda_stream)
        _lib.check(rc)
    return M, b, workspace


def chunk_shard_finish(query, key, value, g, beta, initial_state: Optional[torch.Tensor],
                       output_final_state: bool, use_qk_l2norm_in_kernel: bool,
                       workspace: torch.Tensor) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Outputs and end state of a shard from its start state, reusing the summary's workspace."""
    q, k, v, gg, bb = _inputs(query, key, value, g, beta)
    B, T, H, _ = q.shape
    lib = _lib.load()
    out = torch.empty((B, T, H, D), dtype=q.dtype, device=q.device)
    final = torch.empty((B, H, D, D), dtype=torch.float32, device=q.device) if output_final_state else None
    h0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    if not isinstance(workspace, torch.Tensor) or workspace.device != q.device:
        raise RuntimeError(f"workspace must be the shard summary's CUDA workspace on {q.device}")
    with torch.cuda.device(q.device):
        _raise_pending(lib, q.device)
        dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, gg, bb, out))
        rc = lib.gdn_chunk_sp_finish(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg),
                                     ctypes.byref(db), 64, h0.data_ptr() if h0 is not None else None,
                                     int(bool(output_final_state)), int(bool(use_qk_l2norm_in_kernel)),
                                     ctypes.byref(do), final.data_ptr() if final is not None else None,
                                     workspace.data_ptr(), workspace.numel(),
                                     torch.cuda.current_stream(q.device).cuda_stream)
        _lib.check(rc)
    if out.dtype != query.dtype:
        out = out.to(query.dtype)
    return out, final


def sequence_parallel_chunk_gated_delta_rule(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    group=None,
    summary_fn: Callable = chunk_shard_summary,
    finish_fn: Callable = chunk_shard_finish,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Chunked gated delta rule over a sequence split in time across the ranks of ``group``.

    Rank ``r`` passes its contiguous shard ``[B, T_r, H, D]`` (shards in rank
    order) and the same ``initial_state`` as every other rank; it gets back the
    outputs of its shard and, with ``output_final_state``, the state at the end
    of its shard (on the last rank: the state at the end of the sequence).
    ``summary_fn`` / ``finish_fn`` default to the CUDA kernels; tests substitute
    CPU stand-ins to exercise the exchange on ``gloo``.
    """
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    M, b, ws = summary_fn(query, key, value, g, beta, use_qk_l2norm_in_kernel)
    packed = torch.stack([M, b]).contiguous()
    gathered = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(gathered, packed, group=group)
    if rank == 0:
        start = initial_state
    else:
        start = compose_start_states([x[0] for x in gathered[:rank]], [x[1] for x in gathered[:rank]],
                                     initial_state)[rank]
    return finish_fn(query, key, value, g, beta, start, output_final_state, use_qk_l2norm_in_kernel, ws)
