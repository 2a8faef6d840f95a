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


def test_ttft_harness_model_is_the_benchmark_shape():
    """The TTFT harness's random-init model has config 4's shape (Qwen3.5-0.8B's text stack) and is registered
    under the text class name that its checkpoint declares."""
    from llms_from_scratch_b200.model import QWEN3_5_0_8B
    from llms_from_scratch_b200.vllm_ttft import ARCH, text_config
    cfg = text_config()
    assert cfg.architectures == [ARCH] and cfg.model_type == "qwen3_5_text"
    c = QWEN3_5_0_8B
    assert (cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers) == \
        (c["vocab_size"], c["emb_dim"], c["hidden_dim"], c["n_layers"])
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim) == (c["n_heads"], c["n_kv_groups"], c["head_dim"])
    assert (cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim) == \
        (c["linear_num_key_heads"], c["linear_num_value_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"])
    assert list(cfg.layer_types) == list(c["layer_types"])
