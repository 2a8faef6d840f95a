"""The drop-in through the reference's own callers, on the GPU.

With this package's ``compat/`` directory first on ``sys.path``, the reference's
modules (its unmodified install in ``baseline/_ref``) import the module name
``qwen3_5_cutedsl_kernels`` and get this package's kernels:

* ``qwen3_5_transformers.py:25-30`` binds ``fast_chunk_gated_delta_rule`` as the
  module global ``chunk_gated_delta_rule`` at import, and every
  ``Qwen3_5GatedDeltaNet`` takes it at construction (:285);
* ``benchmark.build_gated_delta_net`` (benchmark.py:107-124) builds the layer and
  ``benchmark.patch_model_backend`` (benchmark.py:254-280) re-binds the global per
  backend.

The layer's output on this package's kernels is held to the same layer on the
reference's ``torch_chunk_gated_delta_rule`` (max-abs 2e-2, rel-L2 5e-3), for a
prefill and for a prefill-then-decode run through the layer's cache contract
(qwen3_5_transformers.py:312-326, :337-348, :396-402) with this package's decode
hooks.  Skipped when the reference install is absent.
"""
import collections
import importlib.util
import os
import sys
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
COMPAT = os.path.join(ROOT, "llms_from_scratch_b200", "compat")
_NAMES = ("qwen3_5_cutedsl_kernels", "qwen3_5_transformers", "benchmark")


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(os.path.join(REF, "qwen3_5_transformers.py")):
        pytest.skip("the reference install (baseline/_ref) is absent")
    saved = {k: sys.modules.pop(k) for k in _NAMES if k in sys.modules}
    sys.path[:0] = [COMPAT, REF]
    try:
        mods = {}
        for name in ("qwen3_5_transformers", "benchmark"):
            spec = importlib.util.spec_from_file_location(name, os.path.join(REF, name + ".py"))
            m = importlib.util.module_from_spec(spec)
            sys.modules[name] = m
            spec.loader.exec_module(m)
            mods[name] = m
        yield SimpleNamespace(t=mods["qwen3_5_transformers"], bench=mods["benchmark"],
                              shim=sys.modules["qwen3_5_cutedsl_kernels"])
    finally:
        del sys.path[:2]
        for k in _NAMES:
            sys.modules.pop(k, None)
        sys.modules.update(saved)


def _close(a, b, what):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    rel = ((a - b).norm() / b.norm()).item()
    assert err <= 2e-2 and rel <= 5e-3, f"{what}: max-abs {err:.3e}, rel-L2 {rel:.3e}"


def _layer(ref, seed):
    torch.manual_seed(seed)
    cfg = dict(ref.bench.QWEN3_5_CONFIG, dtype=torch.bfloat16)
    return ref.bench.build_gated_delta_net(cfg, torch.device("cuda"))


def test_reference_module_binds_this_package(ref):
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    assert ref.shim.__file__.startswith(COMPAT)
    assert ref.t.chunk_gated_delta_rule is fast_chunk_gated_delta_rule
    assert ref.t.is_fast_path_available
    layer = _layer(ref, 0)
    assert layer.chunk_gated_delta_rule is fast_chunk_gated_delta_rule


def test_layer_prefill_matches_the_torch_rule(ref):
    from llms_from_scratch_b200 import _lib
    layer = _layer(ref, 1)
    x = torch.randn(2, 300, layer.hidden_size, device="cuda").to(torch.bfloat16)
    lib = _lib.load()
    with torch.no_grad():
        n0 = lib.gdn_launch_count()
        ours = layer(x)
        assert lib.gdn_launch_count() > n0  # the kernels ran
        layer.chunk_gated_delta_rule = ref.t.torch_chunk_gated_delta_rule
        want = layer(x)
    _close(ours, want, "layer prefill")


class _Cache:
    """The cache object the layer reads and writes (qwen3_5_transformers.py:312-326, :343-348, :401-402); it
    reads both entries before the prefill writes them, so they start as None."""

    def __init__(self):
        self.conv_states = collections.defaultdict(lambda: None)
        self.recurrent_states = collections.defaultdict(lambda: None)
        self.has_previous_state = False


def test_layer_prefill_then_decode_through_the_cache_contract(ref):
    """Prefill 37 tokens with a cache, then 3 single-token steps (has_previous_state): on this package's
    chunk rule, decode conv and recurrent rule vs the reference's torch ones."""
    from llms_from_scratch_b200 import fast_recurrent_gated_delta_rule, layer as L
    layer = _layer(ref, 2)
    xs = torch.randn(1, 40, layer.hidden_size, device="cuda").to(torch.bfloat16)
    outs = {}
    for impl in ("ours", "torch"):
        if impl == "ours":
            layer.chunk_gated_delta_rule = ref.shim.fast_chunk_gated_delta_rule
            layer.recurrent_gated_delta_rule = fast_recurrent_gated_delta_rule
            layer.causal_conv1d_update = L.causal_conv1d_update
        else:
            layer.chunk_gated_delta_rule = ref.t.torch_chunk_gated_delta_rule
            layer.recurrent_gated_delta_rule = ref.t.torch_recurrent_gated_delta_rule
            layer.causal_conv1d_update = ref.t.torch_causal_conv1d_update
        cache = _Cache()
        with torch.no_grad():
            steps = [layer(xs[:, :37], cache_params=cache)]
            cache.has_previous_state = True
            for t in range(37, 40):
                steps.append(layer(xs[:, t:t + 1], cache_params=cache, cache_position=torch.tensor([t])))
        outs[impl] = (steps, cache)
    for i, (a, b) in enumerate(zip(outs["ours"][0], outs["torch"][0])):
        _close(a, b, f"step {i}")
    _close(outs["ours"][1].recurrent_states[0], outs["torch"][1].recurrent_states[0], "recurrent state")


def test_benchmark_backend_patch_routes_to_this_package(ref):
    """benchmark.patch_model_backend("triton") re-binds the module global to fast_chunk_gated_delta_rule(...,
    backend="triton") from the shim: this package's kernels serve it; "torch" restores the torch rule."""
    from llms_from_scratch_b200 import _lib
    lib = _lib.load()
    saved = ref.t.chunk_gated_delta_rule
    try:
        ref.bench.patch_model_backend("triton")
        layer = _layer(ref, 3)
        x = torch.randn(1, 70, layer.hidden_size, device="cuda").to(torch.bfloat16)
        with torch.no_grad():
            n0 = lib.gdn_launch_count()
            ours = layer(x)
            assert lib.gdn_launch_count() > n0
            ref.bench.patch_model_backend("torch")
            layer_t = _layer(ref, 3)
            assert layer_t.chunk_gated_delta_rule is ref.t.torch_chunk_gated_delta_rule
            n1 = lib.gdn_launch_count()
            want = layer_t(x)
            assert lib.gdn_launch_count() == n1
        _close(ours, want, "patched backend")
    finally:
        ref.t.chunk_gated_delta_rule = saved
