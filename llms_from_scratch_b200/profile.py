"""Small, fixed workloads for running a profiler (ncu) on this package's kernels.

    python -m llms_from_scratch_b200.profile chunk     # chunked forward, B=1, T=4096, H=16 (bench shape), 4 calls
    python -m llms_from_scratch_b200.profile batched   # chunked forward, B=8, T=4096, H=16 (the lean scan), 3 calls
    python -m llms_from_scratch_b200.profile rec       # recurrent decode step, B=32, H=16, 4 calls
    python -m llms_from_scratch_b200.profile decode    # decoder: prefill 26 tokens + 8 decode steps, batch 32

Each holds a few hundred MB on the device at most and launches few kernels, so a capture such as

    ncu --set full --clock-control none -k regex:gdn_prep_tc -s 2 -c 1 -o prep \\
        python -m llms_from_scratch_b200.profile chunk

ends in about a minute.  Inputs are seeded synthetic tensors with the benchmark's distributions.
"""

from __future__ import annotations

import sys

import torch


def _inputs(B, T, H, gen, dev="cuda"):
    q = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device=dev, generator=gen), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, 128, device=dev, generator=gen), dim=-1).bfloat16()
    v = torch.randn(B, T, H, 128, device=dev, generator=gen).bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device=dev, generator=gen))
    beta = torch.randn(B, T, H, device=dev, generator=gen).sigmoid()
    s0 = torch.randn(B, H, 128, 128, device=dev, generator=gen) * 0.02
    return q, k, v, g, beta, s0


def main(argv=None) -> int:
    from . import fast_chunk_gated_delta_rule, fast_recurrent_gated_delta_rule
    what = (argv or sys.argv[1:] or ["chunk"])[0]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    if what == "chunk":
        q, k, v, g, beta, s0 = _inputs(1, 4096, 16, gen)
        for _ in range(4):
            fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                        use_qk_l2norm_in_kernel=True)
    elif what == "batched":  # 128 (b, h) chains: gdn_scan_lean_tc; 1.2 GB of records
        q, k, v, g, beta, s0 = _inputs(8, 4096, 16, gen)
        for _ in range(3):
            fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                        use_qk_l2norm_in_kernel=True)
    elif what == "rec":
        q, k, v, g, beta, s0 = _inputs(32, 1, 16, gen)
        for _ in range(4):
            fast_recurrent_gated_delta_rule(q, k, v, g, beta, s0, True, use_qk_l2norm_in_kernel=True, out_state=s0)
    elif what == "decode":
        from .model import QWEN3_5_0_8B, Qwen35Decoder, random_weights
        dec = Qwen35Decoder(QWEN3_5_0_8B, random_weights(QWEN3_5_0_8B, device="cuda"), device="cuda", max_len=64)
        prompt = torch.randint(0, QWEN3_5_0_8B["vocab_size"], (32, 26), device="cuda", generator=gen)
        dec.generate(prompt, 8, use_graph=False)
    else:
        print(f"unknown workload {what!r}: chunk | batched | rec | decode", file=sys.stderr)
        return 2
    torch.cuda.synchronize()
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
