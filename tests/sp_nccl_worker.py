"""torchrun worker for tests/test_gpu_parallel.py: one time shard per rank over NCCL.

Every rank builds the same seeded sequence, runs its shard through
sequence_parallel_chunk_gated_delta_rule, and rank 0 compares the gathered
outputs and the last rank's end state with one single-GPU call."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from llms_from_scratch_b200 import fast_chunk_gated_delta_rule  # noqa: E402
from llms_from_scratch_b200.parallel import sequence_parallel_chunk_gated_delta_rule  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    B, T, H, D = 1, 1000 * world + 37, 8, 128
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    q = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16()
    k = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16()
    v = torch.randn(B, T, H, D, device=dev, generator=gen).bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device=dev, generator=gen)) * 0.1
    beta = torch.randn(B, T, H, device=dev, generator=gen).sigmoid()
    s0 = torch.randn(B, H, D, D, device=dev, generator=gen) * 0.02
    lo, hi = T * rank // world, T * (rank + 1) // world
    o, s = sequence_parallel_chunk_gated_delta_rule(q[:, lo:hi], k[:, lo:hi], v[:, lo:hi], g[:, lo:hi],
                                                    beta[:, lo:hi], initial_state=s0, output_final_state=True,
                                                    use_qk_l2norm_in_kernel=True)
    sizes = [T * (r + 1) // world - T * r // world for r in range(world)]
    outs = [torch.empty(B, n, H, D, device=dev, dtype=o.dtype) for n in sizes]
    dist.all_gather(outs, o.contiguous())
    last = s.clone()
    dist.broadcast(last, src=world - 1)
    if rank == 0:
        ref_o, ref_s = fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                                   use_qk_l2norm_in_kernel=True)
        o_all = torch.cat(outs, 1).float()
        err = (o_all - ref_o.float()).abs().max().item()
        r_o = ((o_all - ref_o.float()).norm() / ref_o.float().norm()).item()
        r_s = ((last - ref_s).norm() / ref_s.norm()).item()
        print(f"world={world} max-abs={err:.3e} rel-L2 out={r_o:.3e} state={r_s:.3e}", flush=True)
        if err < 2e-2 and r_o < 5e-3 and r_s < 5e-3:
            print("SP-OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
