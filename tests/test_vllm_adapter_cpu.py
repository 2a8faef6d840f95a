"""The vLLM 0.22 adapter patches and restores ``ChunkGatedDeltaRule`` (no GPU needed)."""
import pytest


def test_install_routes_chunk_gated_delta_rule_and_uninstall_restores():
    try:
        from vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn import ChunkGatedDeltaRule
    except Exception as e:  # vLLM absent or not importable here
        pytest.skip(f"vLLM not importable: {e}")
    from llms_from_scratch_b200 import vllm_adapter
    before = {n: getattr(ChunkGatedDeltaRule, n) for n in ("__init__", "forward_native", "forward_cuda")}
    cls = vllm_adapter.install()
    try:
        assert cls is ChunkGatedDeltaRule
        assert ChunkGatedDeltaRule.forward_native is vllm_adapter.forward
        assert ChunkGatedDeltaRule.forward_cuda is vllm_adapter.forward
        assert ChunkGatedDeltaRule.__init__ is not before["__init__"]
        assert vllm_adapter.install() is cls  # idempotent
    finally:
        vllm_adapter.uninstall()
    for n, fn in before.items():
        assert getattr(ChunkGatedDeltaRule, n) is fn
