"""Golden gradients of the chunked gated delta rule, from the reference's own torch code.

The reference is inference-only (no backward kernel), but its pure-PyTorch forward
``torch_chunk_gated_delta_rule`` (qwen3_5_transformers.py:110-187) is differentiable.
This script runs it on CPU (float64 leaves; the function itself computes in float32,
qwen3_5_transformers.py:122-127) on float32-exact inputs, takes autograd's
gradients of ``sum(out * d_out) + sum(final_state * d_final_state)`` with respect to
q, k, v, g, beta and the initial state, and stores inputs and gradients as
``bwd_*.npz`` beside this script:

    python tests/golden/make_golden_bwd.py --reference /path/to/llms_from_scratch

The tests never read the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, T, H, l2norm_in_kernel, initial_state, d_final_state, decay_scale, seed)
CASES = [
    ("bwd_T150_l2_state", 1, 150, 2, True, True, True, 1.0, 11),
    ("bwd_B2_T64_prenorm", 2, 64, 1, False, False, True, 1.0, 12),
    ("bwd_T1_l2", 1, 1, 2, True, True, False, 1.0, 13),
    ("bwd_T130_strong_decay", 1, 130, 1, True, True, True, 4.0, 14),
    ("bwd_T63_weak_decay", 1, 63, 2, True, False, False, 0.05, 15),
]


def make(ref_mod, B, T, H, l2, with_s0, with_ds, decay_scale, seed):
    import torch

    rng = np.random.default_rng(seed)
    D = 128
    f32 = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    q, k, v = f32(B, T, H, D), f32(B, T, H, D), f32(B, T, H, D)
    if not l2:
        q = (q / np.sqrt((q * q).sum(-1, keepdims=True))).astype(np.float32)
        k = (k / np.sqrt((k * k).sum(-1, keepdims=True))).astype(np.float32)
    g = (-np.logaddexp(0.0, f32(B, T, H)) * decay_scale).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-f32(B, T, H)))).astype(np.float32)
    s0 = (0.05 * f32(B, H, D, D)).astype(np.float32) if with_s0 else None
    d_out = f32(B, T, H, D)
    d_fs = f32(B, H, D, D) if with_ds else None
    xs = [torch.from_numpy(x).double().requires_grad_() for x in (q, k, v, g, beta)]
    h0 = torch.from_numpy(s0).double().requires_grad_() if with_s0 else None
    o, s = ref_mod.torch_chunk_gated_delta_rule(*xs, chunk_size=64, initial_state=h0, output_final_state=True,
                                                use_qk_l2norm_in_kernel=l2)
    loss = (o * torch.from_numpy(d_out).double()).sum()
    if with_ds:
        loss = loss + (s * torch.from_numpy(d_fs).double()).sum()
    loss.backward()
    out = dict(q=q, k=k, v=v, g=g, beta=beta, d_out=d_out, l2norm=np.array(l2),
               dq=xs[0].grad.numpy(), dk=xs[1].grad.numpy(), dv=xs[2].grad.numpy(), dg=xs[3].grad.numpy(),
               dbeta=xs[4].grad.numpy())
    if with_s0:
        out["h0"] = s0
        out["dh0"] = h0.grad.numpy()
    if with_ds:
        out["d_final_state"] = d_fs
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of pbanavara/llms_from_scratch")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import qwen3_5_transformers as ref_mod

    for name, B, T, H, l2, s0, ds, dsc, seed in CASES:
        arrs = make(ref_mod, B, T, H, l2, s0, ds, dsc, seed)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)
        print(name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
