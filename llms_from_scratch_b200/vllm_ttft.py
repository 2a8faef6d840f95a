"""Time to first token of vLLM 0.22 serving a Qwen3.5-0.8B-shaped model: vLLM's own GatedDeltaNet prefill
kernels against this package's (``vllm_adapter.install()``) -- the reference's TTFT harness
(vllm_inference.py:1-33, :128-164) on this box.

    python -m llms_from_scratch_b200.vllm_ttft --lengths 256 1024 4096            # both backends
    python -m llms_from_scratch_b200.vllm_ttft --backend ours --lengths 1024       # one backend, in-process

What differs from the reference's harness, and why:

* The model is random-init (weights ~ N(0, 0.02), the transformers initialisation) with Qwen3.5-0.8B's text
  shape (hidden 1024, 24 layers: 18 GatedDeltaNet + 6 gated attention, FFN 3584, vocab 151,936), built
  with transformers and saved once to a local directory: no trained checkpoint is available offline.  vLLM
  registers Qwen3.5 only as its vision-language wrapper, so its text-only ``Qwen3_5ForCausalLM`` class is
  registered here (with the wrapper's hybrid-state hooks) and the checkpoint's weights carry its names.
* Prompts are seeded random token ids of the given lengths (the reference's English prompts need the
  checkpoint's tokenizer); vLLM runs without a tokenizer.
* vLLM runs in-process (``VLLM_ENABLE_V1_MULTIPROCESSING=0``) so that the patched ``ChunkGatedDeltaRule``
  is the one the model uses, and each backend runs in its own subprocess (the patch is process-wide); the
  ``ours`` run reports how many of this package's kernels it launched, which shows the patch took effect.
* Each prompt fits one scheduler step (``max_num_batched_tokens`` = the longest prompt), so one prefill pass
  is timed, as the reference's single-request TTFT is.

TTFT is the reference's proxy: the wall time of ``llm.generate(prompt, max_tokens=1)`` after warm-up, the
median of ``--repeats`` runs.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

# Qwen3.5-0.8B's text stack (the benchmark's config 4 shape; model.QWEN3_5_0_8B) in transformers' names
TEXT_CONFIG = dict(vocab_size=151_936, hidden_size=1_024, intermediate_size=3_584, num_hidden_layers=24,
                   num_attention_heads=8, num_key_value_heads=2, head_dim=256, linear_num_key_heads=16,
                   linear_num_value_heads=16, linear_key_head_dim=128, linear_value_head_dim=128,
                   linear_conv_kernel_dim=4, layer_types=(["linear_attention"] * 3 + ["full_attention"]) * 6,
                   rope_parameters={"rope_type": "default", "rope_theta": 10_000_000.0, "partial_rotary_factor": 0.25},
                   rms_norm_eps=1e-6, tie_word_embeddings=False, max_position_embeddings=262_144)
ARCH = "Qwen3_5ForCausalLM"


def text_config():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    cfg = Qwen3_5TextConfig(**TEXT_CONFIG)
    cfg.architectures = [ARCH]
    return cfg


def make_checkpoint(path: str, seed: int = 0) -> str:
    """Save a random-init model of ``TEXT_CONFIG`` to ``path`` (config.json + model.safetensors, bf16) unless
    one is there; weights named as vLLM's ``Qwen3_5ForCausalLM`` loads them (``model.layers...``)."""
    if os.path.exists(os.path.join(path, "config.json")) and os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    import torch
    from safetensors.torch import save_file
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    os.makedirs(path, exist_ok=True)
    cfg = text_config()
    torch.manual_seed(seed)
    dev = "cuda" if torch.cuda.is_available() else "cpu"  # the initialisation is ~10x faster on the GPU
    with torch.device(dev):
        model = Qwen3_5ForCausalLM(cfg).to(torch.bfloat16)
    state = {k.replace("model.language_model.", "model."): v.detach().to("cpu").contiguous()
             for k, v in model.state_dict().items()}
    del model
    save_file(state, os.path.join(path, "model.safetensors"), metadata={"format": "pt"})
    cfg.save_pretrained(path)
    if dev == "cuda":
        torch.cuda.empty_cache()
    return path


def _text_model_class():
    """vLLM's text-only Qwen3.5 model marked as the hybrid (attention + GatedDeltaNet state) model it is, with
    the state-shape hooks of vLLM's Qwen3.5 wrapper, so the engine sizes its recurrent-state cache."""
    from vllm.model_executor.models.interfaces import IsHybrid
    from vllm.model_executor.models.qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5ForConditionalGeneration as W

    class Qwen3_5TextForCausalLM(Qwen3_5ForCausalLM, IsHybrid):
        get_mamba_state_dtype_from_config = classmethod(W.get_mamba_state_dtype_from_config.__func__)
        get_mamba_state_shape_from_config = classmethod(W.get_mamba_state_shape_from_config.__func__)
        get_mamba_state_copy_func = classmethod(W.get_mamba_state_copy_func.__func__)

    return Qwen3_5TextForCausalLM


def run_backend(backend: str, ckpt: str, lengths, repeats: int, warmup: int, seed: int) -> dict:
    """TTFT per prompt length with one backend, in this process."""
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ.setdefault("HF_HUB_OFFLINE", "1")
    os.environ.setdefault("TRANSFORMERS_OFFLINE", "1")
    import torch
    if backend == "ours":
        from . import _lib
        from .vllm_adapter import install
        install()
        lib = _lib.load()
    from vllm import LLM, ModelRegistry, SamplingParams
    from vllm.inputs import TokensPrompt

    ModelRegistry.register_model(ARCH, _text_model_class())
    top = max(lengths)
    llm = LLM(model=ckpt, skip_tokenizer_init=True, dtype="bfloat16", enforce_eager=True,
              max_model_len=top + 16, max_num_batched_tokens=top + 16, gpu_memory_utilization=0.5, seed=seed)
    sp = SamplingParams(temperature=0.0, max_tokens=1, detokenize=False)
    gen = torch.Generator().manual_seed(seed)
    out = {"backend": backend, "ttft_ms": {}}
    for L in lengths:
        ids = torch.randint(0, TEXT_CONFIG["vocab_size"], (L,), generator=gen).tolist()
        prompt = TokensPrompt(prompt_token_ids=ids)
        for _ in range(warmup):
            llm.generate([prompt], sp, use_tqdm=False)
        n0 = lib.gdn_launch_count() if backend == "ours" else 0
        times = []
        for _ in range(repeats):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            llm.generate([prompt], sp, use_tqdm=False)
            torch.cuda.synchronize()
            times.append((time.perf_counter() - t0) * 1e3)
        out["ttft_ms"][str(L)] = statistics.median(times)
        if backend == "ours":
            out.setdefault("package_launches_per_prefill", {})[str(L)] = (lib.gdn_launch_count() - n0) / repeats
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--backend", choices=["default", "ours", "both"], default="both")
    ap.add_argument("--lengths", type=int, nargs="+", default=[256, 1024, 4096])
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--checkpoint", default=os.path.join(tempfile.gettempdir(), "gdn_b200_q35_0p8b_random"),
                    help="directory of the random-init checkpoint (made if absent)")
    a = ap.parse_args(argv)
    make_checkpoint(a.checkpoint, a.seed)
    if a.backend != "both":
        print(json.dumps(run_backend(a.backend, a.checkpoint, a.lengths, a.repeats, a.warmup, a.seed)), flush=True)
        return 0
    results = {}
    for backend in ("default", "ours"):
        cmd = [sys.executable, "-m", "llms_from_scratch_b200.vllm_ttft", "--backend", backend, "--checkpoint",
               a.checkpoint, "--repeats", str(a.repeats), "--warmup", str(a.warmup), "--seed", str(a.seed),
               "--lengths", *map(str, a.lengths)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode != 0 or not lines:
            sys.stderr.write(r.stdout[-4000:] + r.stderr[-8000:])
            results[backend] = {"error": f"exit {r.returncode}"}
            continue
        results[backend] = json.loads(lines[-1])
    line = {"workload": "vLLM 0.22 TTFT (generate, max_tokens=1), random-init Qwen3.5-0.8B-shaped model, bf16, "
                        "seeded token-id prompts, enforce_eager", "results": results}
    d, o = results.get("default", {}).get("ttft_ms"), results.get("ours", {}).get("ttft_ms")
    if d and o:
        line["speedup"] = {L: d[L] / o[L] for L in d if L in o}
    print(json.dumps(line), flush=True)
    return 0 if all("error" not in v for v in results.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
