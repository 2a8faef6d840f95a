"""Generate golden input/output vectors from the reference's own torch code.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/llms_from_scratch

It imports ``qwen3_5_transformers`` from the reference and calls
``torch_chunk_gated_delta_rule`` (qwen3_5_transformers.py:110-187) and
``torch_recurrent_gated_delta_rule`` (qwen3_5_transformers.py:190-229)
directly on CPU.  (Going through ``qwen3_5_cutedsl_kernels`` would pick the
Triton backend whenever Triton is importable, qwen3_5_cutedsl_kernels.py:104-109,
which cannot run on CPU tensors.)

Inputs come from ``oracle.gdn_oracle.make_inputs`` (numpy PCG64, seeded), so
the large config-1 case stores only a digest of its inputs plus a strided
sample of its outputs; small cases store everything.  Output files are the
``*.npz`` beside this script; the tests never read the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.gdn_oracle import bf16_bits, make_inputs  # noqa: E402

# (name, kind, B, T, H, in_dtype, init_std, l2norm_in_kernel, normalize_inputs, output_final_state, seed)
CASES = [
    ("chunk_fp32_T65_raw_l2", "chunk", 1, 65, 2, "fp32", 0.0, True, False, True, 1),
    ("chunk_fp32_T63_init", "chunk", 2, 63, 2, "fp32", 0.02, False, True, True, 2),
    ("chunk_fp32_T1", "chunk", 1, 1, 3, "fp32", 0.02, True, True, True, 3),
    ("chunk_fp32_T64_nostate", "chunk", 1, 64, 2, "fp32", 0.0, True, True, False, 4),
    ("chunk_fp32_T200_init", "chunk", 1, 200, 1, "fp32", 0.02, True, True, True, 5),
    ("chunk_bf16_T130_init", "chunk", 1, 130, 2, "bf16", 0.02, True, False, True, 6),
    ("chunk_bf16_T128_init", "chunk", 2, 128, 1, "bf16", 0.02, True, True, True, 7),
    ("rec_fp32_T5_init", "recurrent", 2, 5, 2, "fp32", 0.02, True, False, True, 8),
    ("rec_bf16_T1_init", "recurrent", 2, 1, 2, "bf16", 0.02, True, True, True, 9),
    ("rec_fp32_T3_nostate", "recurrent", 1, 3, 2, "fp32", 0.0, True, True, True, 10),
]

# Config 1 of the benchmark: B=1, T=256, H=16, d=128, fp32, zero initial state, seed 0.
CONFIG1 = dict(B=1, T=256, H=16, seed=0)
SAMPLE_STRIDE = 61


def input_digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()


def _torch_inputs(torch, q, k, v, g, beta, state, in_dtype):
    tdt = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[in_dtype]
    tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x)).to(tdt) for x in (q, k, v))
    tg = torch.from_numpy(np.ascontiguousarray(g))
    tb = torch.from_numpy(np.ascontiguousarray(beta))
    ts = None if state is None else torch.from_numpy(np.ascontiguousarray(state))
    return tq, tk, tv, tg, tb, ts


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    import qwen3_5_transformers as ref

    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    for (name, kind, B, T, H, in_dtype, init_std, l2, norm_in, ofs, seed) in CASES:
        q, k, v, g, beta, state = make_inputs(B, T, H, seed=seed, in_dtype=in_dtype,
                                              init_state_std=init_std, normalize_qk=norm_in)
        tq, tk, tv, tg, tb, ts = _torch_inputs(torch, q, k, v, g, beta, state, in_dtype)
        if kind == "chunk":
            o, s = ref.torch_chunk_gated_delta_rule(tq, tk, tv, tg, tb, chunk_size=64, initial_state=ts,
                                                    output_final_state=ofs, use_qk_l2norm_in_kernel=l2)
        else:
            o, s = ref.torch_recurrent_gated_delta_rule(tq, tk, tv, tg, tb, initial_state=ts,
                                                        output_final_state=ofs, use_qk_l2norm_in_kernel=l2)
        o32 = o.float().numpy()
        rec = dict(kind=kind, in_dtype=in_dtype, l2norm=l2, output_final_state=ofs,
                   q=q, k=k, v=v, g=g, beta=beta)
        if in_dtype != "fp32" and l2:
            # torch's CPU rsqrt for 16-bit tensors is a hardware estimate that can land
            # one ulp away from the correctly rounded value; keep the reference's own
            # normalised q/k so the rest of the arithmetic can be pinned exactly.
            rec["q_l2"] = ref.l2norm(tq).float().numpy()
            rec["k_l2"] = ref.l2norm(tk).float().numpy()
        if state is not None:
            rec["initial_state"] = state
        rec["out"] = bf16_bits(o32) if in_dtype == "bf16" else o32
        if s is not None:
            rec["final_state"] = s.float().numpy()
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print(name, o.shape, None if s is None else tuple(s.shape))

    c = CONFIG1
    q, k, v, g, beta, state = make_inputs(c["B"], c["T"], c["H"], seed=c["seed"])
    tq, tk, tv, tg, tb, ts = _torch_inputs(torch, q, k, v, g, beta, state, "fp32")
    o, s = ref.torch_chunk_gated_delta_rule(tq, tk, tv, tg, tb, chunk_size=64, initial_state=None,
                                            output_final_state=True, use_qk_l2norm_in_kernel=True)
    o, s = o.numpy(), s.numpy()
    np.savez_compressed(
        os.path.join(HERE, "config1_fp32_B1_T256_H16.npz"),
        digest=np.array(input_digest(q, k, v, g, beta)), B=c["B"], T=c["T"], H=c["H"], seed=c["seed"],
        out_sample=o.reshape(-1)[::SAMPLE_STRIDE], state_sample=s.reshape(-1)[::SAMPLE_STRIDE],
        out_sum=np.float64(o.astype(np.float64).sum()), out_abs_sum=np.float64(np.abs(o).astype(np.float64).sum()),
        state_sum=np.float64(s.astype(np.float64).sum()), stride=SAMPLE_STRIDE,
    )
    print("config1", o.shape, s.shape)


if __name__ == "__main__":
    main()
