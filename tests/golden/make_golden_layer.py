"""Generate golden vectors for the GatedDeltaNet layer steps around the gated delta rule.

Run where the reference checkout is available:

    python tests/golden/make_golden_layer.py --reference /path/to/llms_from_scratch

From the reference's qwen3_5_transformers.py it calls ``torch_causal_conv1d_update``
(:85-101) and ``Qwen3_5RMSNormGated`` (:56-71) directly, and runs the layer's prefill
convolution and gates with the same torch ops as ``Qwen3_5GatedDeltaNet`` (the
depthwise ``nn.Conv1d`` of :253-260 followed by ``F.silu(conv(x)[:, :, :seq_len])``
at :356 and the cache pad at :346-348; ``b.sigmoid()`` and
``-A_log.float().exp() * F.softplus(a.float() + dt_bias)`` at :377-379), all on CPU
in bf16 as the model runs them.  (The layer itself cannot be built on a CPU-only
host: it asks FLA's fused norm for a CUDA device.)  Inputs are seeded numpy draws
rounded to bf16; every array is stored as float32.  Output: ``layer_*.npz`` beside
this script; the tests never read the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.gdn_oracle import round_bf16  # noqa: E402


def _bf16(rng, shape, scale=1.0):
    return round_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    import torch.nn.functional as F
    from torch import nn

    import qwen3_5_transformers as ref

    bf = torch.bfloat16
    K = 4

    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x)).to(bf)

    # ---- prefill convolution (+ the cache's conv state)
    for name, B, T, C, seed in [("layer_conv_T70", 2, 70, 96, 11), ("layer_conv_T3", 2, 3, 64, 12),
                                ("layer_conv_T1", 1, 1, 32, 13)]:
        rng = np.random.default_rng(seed)
        x = _bf16(rng, (B, T, C))
        w = _bf16(rng, (C, K), 0.5)
        conv = nn.Conv1d(C, C, K, groups=C, padding=K - 1, bias=False).to(bf)
        with torch.no_grad():
            conv.weight.copy_(t(w)[:, None, :])
            xb = t(x).transpose(1, 2)                       # [B, C, T], as the layer transposes (:334)
            y = F.silu(conv(xb)[:, :, :T])                  # :356
            state = F.pad(xb, (K - xb.shape[-1], 0))        # :346-348
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, weight=w,
                            out=y.transpose(1, 2).float().numpy(), conv_state=state.float().numpy())
        print(name, tuple(y.shape))

    # ---- decode convolution against the cached state
    for name, B, T, C, seed in [("layer_convupd_T1", 3, 1, 64, 21), ("layer_convupd_T2", 2, 2, 32, 22)]:
        rng = np.random.default_rng(seed)
        x = _bf16(rng, (B, T, C))
        s = _bf16(rng, (B, C, K))
        w = _bf16(rng, (C, K), 0.5)
        state = t(s)
        with torch.no_grad():
            y = ref.torch_causal_conv1d_update(t(x).transpose(1, 2), state, t(w), None, "silu")
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, conv_state=s, weight=w,
                            out=y.transpose(1, 2).float().numpy(), new_state=state.float().numpy())
        print(name, tuple(y.shape))

    # ---- gates
    rng = np.random.default_rng(31)
    B, T, H = 2, 9, 4
    a = round_bf16(rng.standard_normal((B, T, H), dtype=np.float32) * np.float32(8.0))
    a[0, 0, :] = [25.0, 21.5, -25.0, 19.75]  # both sides of softplus' threshold (x > 20 returns x)
    b = _bf16(rng, (B, T, H), 3.0)
    A_log = round_bf16(np.log(rng.uniform(0.5, 16.0, H).astype(np.float32)))
    dt_bias = _bf16(rng, (H,))
    with torch.no_grad():
        beta = t(b).sigmoid()
        g = -t(A_log).float().exp() * F.softplus(t(a).float() + t(dt_bias))
    np.savez_compressed(os.path.join(HERE, "layer_gates.npz"), a=a, b=b, A_log=A_log, dt_bias=dt_bias,
                        g=g.float().numpy(), beta=beta.float().numpy())
    print("layer_gates", tuple(g.shape))

    # ---- gated RMS norm
    rng = np.random.default_rng(41)
    N, D = 37, 128
    x = _bf16(rng, (N, D), 2.0)
    z = _bf16(rng, (N, D), 2.0)
    w = round_bf16(np.float32(1.0) + rng.standard_normal(D, dtype=np.float32) * np.float32(0.2))
    norm = ref.Qwen3_5RMSNormGated(D, eps=1e-6).to(bf)
    with torch.no_grad():
        norm.weight.copy_(t(w))
        o = norm(t(x), t(z))
    np.savez_compressed(os.path.join(HERE, "layer_rmsnorm_gated.npz"), x=x, gate=z, weight=w, eps=np.float32(1e-6),
                        out=o.float().numpy())
    print("layer_rmsnorm_gated", tuple(o.shape))


if __name__ == "__main__":
    main()
