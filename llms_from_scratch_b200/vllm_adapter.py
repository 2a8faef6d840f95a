"""vLLM 0.22 adapter: run vLLM's GatedDeltaNet prefill on this package's kernels.

The reference patches vLLM 0.17's ``ChunkGatedDeltaRule.forward_native`` /
``forward_cuda`` with its op and falls back to FLA for packed batches
(vllm_inference.py:82-119).  In vLLM 0.22 the class lives in
``vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn``, picks
``self._forward_method`` in ``__init__``, its methods take extra keyword
arguments (``chunk_indices``, ``chunk_offsets``, ``core_attn_out``), and its
FLA kernels keep the recurrent state as ``[N, H, V, K]``
(fla/ops/chunk.py:168-181) where this package uses ``[N, H, K, V]``.

``forward`` below has that signature: packed batches (``cu_seqlens``) run
``chunk_gated_delta_rule_varlen`` (every sequence on the tensor-core path; no
FLA fallback), single sequences ``fast_chunk_gated_delta_rule``; the state is
transposed on the way in and out, and ``core_attn_out`` is filled as vLLM's own
methods fill it.  ``install()`` makes every ``ChunkGatedDeltaRule`` built after
it use ``forward``; call it before ``LLM(...)`` constructs the model.
"""

from __future__ import annotations

from typing import Optional

import torch

from .ops import chunk_gated_delta_rule_varlen, fast_chunk_gated_delta_rule

_ORIGINALS: dict = {}


def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
            initial_state: Optional[torch.Tensor], output_final_state: bool,
            cu_seqlens: Optional[torch.Tensor] = None, chunk_indices=None, chunk_offsets=None,
            use_qk_l2norm_in_kernel: bool = True, core_attn_out: Optional[torch.Tensor] = None):
    """``ChunkGatedDeltaRule.forward_*`` of vLLM 0.22 on the B200 kernels.

    q/k/v ``[1, T, H, 128]``, g/beta ``[1, T, H]``, ``initial_state`` ``[N, H, V, K]`` (vLLM's layout) or
    None; returns ``(o [1, T, H, V], final_state [N, H, V, K] fp32 or None)``.  ``chunk_indices`` and
    ``chunk_offsets`` (FLA's precomputed chunk tables) are not needed: the chunk tables are built on
    the device from ``cu_seqlens``."""
    h0 = None if initial_state is None else initial_state.transpose(-1, -2).to(torch.float32)
    if cu_seqlens is not None:
        o, final_state = chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu_seqlens, initial_state=h0,
                                                       output_final_state=output_final_state,
                                                       use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    else:
        o, final_state = fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=h0,
                                                     output_final_state=output_final_state,
                                                     use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    if final_state is not None:
        final_state = final_state.transpose(-1, -2).contiguous()
    if core_attn_out is not None:
        o_flat = o.squeeze(0).reshape(-1)
        core_attn_out.reshape(-1)[: o_flat.numel()].copy_(o_flat)
    return o, final_state


def install():
    """Route vLLM's ``ChunkGatedDeltaRule`` (0.22) to ``forward``; returns the patched class."""
    from vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn import ChunkGatedDeltaRule

    if _ORIGINALS:
        return ChunkGatedDeltaRule
    _ORIGINALS.update(__init__=ChunkGatedDeltaRule.__init__, forward_native=ChunkGatedDeltaRule.forward_native,
                      forward_cuda=ChunkGatedDeltaRule.forward_cuda)
    original_init = _ORIGINALS["__init__"]

    def __init__(self, *args, **kw):
        original_init(self, *args, **kw)
        self._forward_method = forward.__get__(self)

    ChunkGatedDeltaRule.__init__ = __init__
    ChunkGatedDeltaRule.forward_native = forward
    ChunkGatedDeltaRule.forward_cuda = forward
    return ChunkGatedDeltaRule


def uninstall():
    """Undo ``install()`` (instances built while it was active keep ``forward``)."""
    if not _ORIGINALS:
        return
    from vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn import ChunkGatedDeltaRule

    for name, fn in _ORIGINALS.items():
        setattr(ChunkGatedDeltaRule, name, fn)
    _ORIGINALS.clear()
