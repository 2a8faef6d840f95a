"""B200 (sm_100a) GatedDeltaNet kernels behind the reference's call signatures.

    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule

The CUDA library ``libgdn_b200.so`` is built in-tree by
``python -m llms_from_scratch_b200.build``; its C ABI is ``include/gdn_b200.h``.
"""

from .ops import (  # noqa: F401
    chunk_bwd_workspace_bytes,
    chunk_gated_delta_rule,
    chunk_gated_delta_rule_bwd,
    chunk_gated_delta_rule_varlen,
    chunk_host_workspace_bytes,
    chunk_varlen_workspace_bytes,
    chunk_workspace_bytes,
    fast_chunk_gated_delta_rule,
    fast_recurrent_gated_delta_rule,
    get_backend,
    l2norm,
)

__all__ = ["fast_chunk_gated_delta_rule", "fast_recurrent_gated_delta_rule", "chunk_workspace_bytes",
           "chunk_host_workspace_bytes", "chunk_gated_delta_rule_varlen", "chunk_varlen_workspace_bytes",
           "chunk_gated_delta_rule", "chunk_gated_delta_rule_bwd", "chunk_bwd_workspace_bytes",
           "get_backend", "l2norm"]
