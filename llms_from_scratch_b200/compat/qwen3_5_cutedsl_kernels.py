"""Drop-in replacement for the reference module ``qwen3_5_cutedsl_kernels``.

Put ``llms_from_scratch_b200/compat`` first on ``sys.path`` (or install this
file under that name) and the reference's callers pick up the B200 kernels
unchanged:

* ``qwen3_5_transformers.py:25-30`` imports ``fast_chunk_gated_delta_rule``
  at load time and binds it per layer (:285);
* ``benchmark.py:136-149, 261, 345, 448`` read ``fast_chunk_gated_delta_rule``,
  ``get_backend``, ``_TRITON_OK`` and ``_CUTE_OK``;
* ``vllm_inference.py:75`` imports ``fast_chunk_gated_delta_rule``.

Every backend name the reference accepts other than ``"torch"`` ("auto",
"triton", "cute") runs this package's sm_100a CUDA kernels, so the two
availability flags report that those names are served here.
"""

from llms_from_scratch_b200.ops import (  # noqa: F401
    fast_chunk_gated_delta_rule,
    fast_recurrent_gated_delta_rule,
    get_backend,
    l2norm,
)

_TRITON_OK = True
_CUTE_OK = True

__all__ = ["fast_chunk_gated_delta_rule", "fast_recurrent_gated_delta_rule", "get_backend", "l2norm",
           "_TRITON_OK", "_CUTE_OK"]
