#!/usr/bin/env python
"""GatedDeltaNet chunked forward benchmark (B200, one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per rank: B=1, T=4096, H=16, Dk=Dv=128, chunk 64, bf16 q/k/v
(q,k ~ N(0,1) then L2-normalised, v ~ N(0,1)), fp32 g = -softplus(N(0,1)),
beta = sigmoid(N(0,1)), initial state ~ N(0, 0.02), l2norm in the kernel,
final state returned.  With N GPUs every rank runs its own shard of a global
batch of N sequences (batch x head sharding, no collective): weak scaling.

A step is one call of ``fast_chunk_gated_delta_rule`` over that batch.  Device
time per step comes from CUDA events on the launching stream; a 256 MiB buffer
(2x L2) is written between timed steps so every step starts with a cold L2.
``e2e`` times the same op called with page-locked host tensors (inputs copied
in and outputs copied out inside the timed region, which the op pipelines in
time slices against its kernels).  rank 0 prints one JSON line.

``--impl reference`` times the reference's own CPU path, its
``torch_chunk_gated_delta_rule`` (qwen3_5_transformers.py:110-187) imported
unmodified from the reference install in ``baseline/_ref``, on rank 0 with all
host threads, on the same seeded inputs at the same B, T, H; without that
install it falls back to the numpy port of the same algorithm
(``oracle/gdn_oracle.py``, kind "port").
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GDN chunk-fwd tok/s @B=1,T=4096 (1/2/4/8 GPU) + % roofline; 0.8B decode tok/s"
UNIT = "tok/s"
D = 128
CHUNK = 64
# algorithmic bytes (fused I/O, intermediates excluded) per token per head:
# q, k, v, o in bf16 (4 x 128 x 2) + g, beta in fp32
BYTES_PER_TOKEN_HEAD = 4 * D * 2 + 8
STATE_BYTES = D * D * 4


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--B", type=int, default=1, help="sequences per rank")
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline budget (rank 0, N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs35", action="store_true", help="skip the config 3 (B=64) and config 5 (--sp-T "
                                                                    "time-sharded) legs")
    ap.add_argument("--no-decode-model", action="store_true", help="skip the config 4 decoder leg")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's Triton path (baseline/_ref) beside this package's")
    ap.add_argument("--soak-seconds", type=float, default=1.0, help="untimed load before timing (clock sampling)")
    ap.add_argument("--sp", action="store_true",
                    help="config 5: one sequence of --sp-T tokens (B=1) split in time across the ranks")
    ap.add_argument("--sp-T", type=int, default=131072)
    ap.add_argument("--decode-batch", type=int, default=32, help="sequences of the decode-kernel leg")
    ap.add_argument("--fla", action="store_true",
                    help="also time vLLM's FLA prefill (its default GatedDeltaNet kernels) on the headline and packed "
                         "workloads, for comparison")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f)
        return t.get(workload, {}).get(kernel)
    except Exception:
        return None


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 50 ms."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples = []
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than guess
            self.err = str(e)
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.05)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [n for b, n in self.REASONS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


# --------------------------------------------------------------------------- inputs

L2_NOTE = "cold L2: a 256 MiB buffer written, then another 256 MiB buffer read, between timed steps"


class L2Flush:
    """Cold, clean L2 between timed steps: write one 256 MiB buffer (2x the 126 MB L2), then read another, so
    no line of the previous step survives and the flush's own dirty lines are written back before the next
    step starts instead of inside it."""

    def __init__(self, torch, device):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.r = torch.zeros(256 << 20, dtype=torch.uint8, device=device)
        self.acc = torch.int32

    def __call__(self, i: int):
        self.w.fill_(i & 0xFF)
        self.r.sum(dtype=self.acc)


def time_layer_kernels(torch, lib, flush, device, T, H, Bd, peak, reps=20):
    """Device time and GB/s of the layer steps around the rule (Qwen3.5 GatedDeltaNet, C = 3 H 128
    channels): prefill conv1d+SiLU and gated RMS norm at B=1, T tokens; gates; decode conv update at Bd."""
    from llms_from_scratch_b200 import layer
    C, D = 3 * H * 128, 128
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    bf = torch.bfloat16
    mixed = torch.randn(1, T, C, device=device, generator=gen).to(bf)
    w = (0.5 * torch.randn(C, 4, device=device, generator=gen)).to(bf)
    st = torch.empty(1, C, 4, dtype=bf, device=device)
    a = torch.randn(1, T, H, device=device, generator=gen).to(bf)
    b = torch.randn(1, T, H, device=device, generator=gen).to(bf)
    A_log = torch.log(torch.rand(H, device=device, generator=gen) * 15 + 0.5).to(bf)
    dt = torch.randn(H, device=device, generator=gen).to(bf)
    o = torch.randn(T * H, D, device=device, generator=gen).to(bf)
    z = torch.randn(T * H, D, device=device, generator=gen).to(bf)
    nw = torch.ones(D, dtype=bf, device=device)
    xd = torch.randn(Bd, C, 1, device=device, generator=gen).to(bf)
    sd = torch.randn(Bd, C, 4, device=device, generator=gen).to(bf)
    legs = {
        "conv1d_silu": (lambda: layer.causal_conv1d_silu(mixed, w, conv_state=st), 2 * 2 * T * C + 2 * C * 4 * 2,
                        f"B=1 T={T} C={C}"),
        "gates": (lambda: layer.gates(a, b, A_log, dt), T * H * (2 + 2 + 4 + 2), f"B=1 T={T} H={H}"),
        "rms_norm_gated": (lambda: layer.rms_norm_gated(o, z, nw, 1e-6), 3 * T * H * D * 2, f"rows={T * H} D={D}"),
        "conv1d_update": (lambda: layer.causal_conv1d_update(xd, sd, w, None, "silu"),
                          Bd * C * (2 + 2 + 2 * 4 * 2) + C * 4 * 2, f"B={Bd} T=1 C={C}"),
    }
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 2)(*[e.cuda_event for e in ev])
    res = {}
    for name, (fn, nbytes, shape) in legs.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for i in range(reps):
            flush(i)
            lib.gdn_set_phase_events(arr, 2)
            fn()
            lib.gdn_set_phase_events(None, 0)
            torch.cuda.synchronize()
            ts.append(ev[0].elapsed_time(ev[1]))
        ms = statistics.median(ts)
        res[name] = {"shape": shape, "ms": ms, "bytes": nbytes, "achieved_gbs": nbytes / (ms / 1e3) / 1e9,
                     "frac_hbm": nbytes / (ms / 1e3) / 1e9 / peak}
    return res


PACKED_LENGTHS = (4096, 37, 2000, 5000, 64, 129, 5058)  # 16,384 tokens in 7 ragged sequences


def _cold_median(torch, fn, flush, reps):
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for i in range(reps):
        flush(i)
        ev[0].record()
        fn()
        ev[1].record()
        torch.cuda.synchronize()
        ts.append(ev[0].elapsed_time(ev[1]))
    return statistics.median(ts)


def time_packed(torch, flush, device, H, peak, fla=None, reps=20):
    """Packed variable-length prefill (cu_seqlens, the vLLM serving layout): one call over PACKED_LENGTHS,
    against the same sequences as separate calls; with ``fla`` also vLLM's FLA on the same packed batch."""
    from llms_from_scratch_b200 import chunk_gated_delta_rule_varlen, chunk_varlen_workspace_bytes
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    T, N = sum(PACKED_LENGTHS), len(PACKED_LENGTHS)
    q, k, v, g, beta, _ = make_inputs(torch, 1, T, H, seed=17, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(18)
    s0 = torch.randn(N, H, D, D, device=device, generator=gen) * 0.02
    edges = [0]
    for n in PACKED_LENGTHS:
        edges.append(edges[-1] + n)
    cu = torch.tensor(edges, dtype=torch.int32, device=device)
    ws = torch.empty(chunk_varlen_workspace_bytes(T, N, H), dtype=torch.uint8, device=device)

    def packed():
        return chunk_gated_delta_rule_varlen(q, k, v, g, beta, cu, initial_state=s0, output_final_state=True,
                                             use_qk_l2norm_in_kernel=True, workspace=ws)

    def separate():
        for n in range(N):
            a, b = edges[n], edges[n + 1]
            fast_chunk_gated_delta_rule(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b],
                                        initial_state=s0[n:n + 1], output_final_state=True,
                                        use_qk_l2norm_in_kernel=True)

    nbytes = T * H * BYTES_PER_TOKEN_HEAD + 2 * N * H * STATE_BYTES
    res = {"workload": f"packed prefill, {N} sequences {list(PACKED_LENGTHS)} = {T} tokens, H={H}, bf16, "
                       "l2norm in kernel, start and final states",
           "tokens": T, "algorithmic_bytes": nbytes}
    for name, fn in (("packed_call", packed), ("separate_calls", separate)):
        ms = _cold_median(torch, fn, flush, reps)
        res[name] = {"ms": ms, "tok_s": T / (ms / 1e3), "frac_hbm": nbytes / (ms / 1e3) / 1e9 / peak}
    if fla is not None:
        s_vk = s0.transpose(-1, -2).contiguous()
        ms = _cold_median(torch, lambda: fla(q=q, k=k, v=v, g=g, beta=beta, initial_state=s_vk,
                                             output_final_state=True, cu_seqlens=cu,
                                             use_qk_l2norm_in_kernel=True), flush, reps)
        res["vllm_fla"] = {"ms": ms, "tok_s": T / (ms / 1e3), "frac_hbm": nbytes / (ms / 1e3) / 1e9 / peak}
    return res


def time_backward(torch, lib, flush, device, T, H, reps=10):
    """Backward of the chunked rule at B=1, T, H (bf16 q/k/v, fp32 g/beta/states, l2norm in kernel, gradients
    of the outputs and of the final state): device time of the whole call and of each of its launches."""
    from llms_from_scratch_b200 import chunk_bwd_workspace_bytes, chunk_gated_delta_rule_bwd
    q, k, v, g, beta, s0 = make_inputs(torch, 1, T, H, seed=31, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(32)
    do = torch.randn(1, T, H, D, device=device, generator=gen).bfloat16()
    dhT = torch.randn(1, H, D, D, device=device, generator=gen)
    ws = torch.empty(chunk_bwd_workspace_bytes(1, T, H), dtype=torch.uint8, device=device)

    def fn():
        return chunk_gated_delta_rule_bwd(q, k, v, g, beta, do, initial_state=s0, d_final_state=dhT,
                                          use_qk_l2norm_in_kernel=True, workspace=ws)

    names = ["fwd_prep", "fwd_scan_states", "bwd_scan", "bwd_states", "bwd_wy", "bwd_grads"]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * 7)(*[e.cuda_event for e in ev])
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    parts = {n: [] for n in names}
    total = []
    for i in range(reps):
        flush(i)
        lib.gdn_set_phase_events(arr, 7)
        fn()
        lib.gdn_set_phase_events(None, 0)
        torch.cuda.synchronize()
        for j, n in enumerate(names):
            parts[n].append(ev[j].elapsed_time(ev[j + 1]))
        total.append(ev[0].elapsed_time(ev[6]))
    ms = _cold_median(torch, fn, flush, reps)  # the call without the phase events between its kernels
    return {"workload": f"chunk backward B=1 T={T} H={H}, bf16 q/k/v and d_out, fp32 g/beta/states, l2norm in "
                        "kernel, d_final_state given; every kernel on the tensor cores (bf16 mode)",
            "ms": ms, "tok_s": T / (ms / 1e3), "ms_instrumented": statistics.median(total),
            "kernels_ms": {n: statistics.median(parts[n]) for n in names}}


def load_fla():
    """vLLM 0.22's FLA chunk_gated_delta_rule, or None with the reason."""
    try:
        from vllm.model_executor.layers.fla.ops import chunk_gated_delta_rule
        return chunk_gated_delta_rule, None
    except Exception as e:  # vLLM absent or not importable
        return None, f"{type(e).__name__}: {e}"[:200]


def make_inputs(torch, B, T, H, seed, device, on_host=False):
    """Config-2 inputs; ``on_host`` draws them with the host generator and copies them to ``device``, so the
    reference arm (which draws them on the host) times the very same tensors."""
    if on_host and str(device) != "cpu":
        return tuple(x.to(device) for x in make_inputs(torch, B, T, H, seed, "cpu"))
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    q = torch.randn(B, T, H, D, device=device, generator=gen)
    k = torch.randn(B, T, H, D, device=device, generator=gen)
    q = (q / q.norm(dim=-1, keepdim=True)).bfloat16()
    k = (k / k.norm(dim=-1, keepdim=True)).bfloat16()
    v = torch.randn(B, T, H, D, device=device, generator=gen).bfloat16()
    beta = torch.randn(B, T, H, device=device, generator=gen).sigmoid()
    g = -torch.nn.functional.softplus(torch.randn(B, T, H, device=device, generator=gen))
    s0 = torch.randn(B, H, D, D, device=device, generator=gen) * 0.02
    return q, k, v, g, beta, s0


# --------------------------------------------------------------------------- CPU (oracle port)

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference_module(name: str):
    """A module of the reference as installed (unmodified) in baseline/_ref, loaded by file path under a
    private name (this package's drop-in shim is also called qwen3_5_cutedsl_kernels), or None when the
    install is absent."""
    import importlib.util
    path = os.path.join(REF_DIR, name + ".py")
    if not os.path.exists(path):
        return None
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)  # its modules import each other by plain name
    key = "_reference_" + name
    if key in sys.modules:
        return sys.modules[key]
    spec = importlib.util.spec_from_file_location(key, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[key] = mod
    spec.loader.exec_module(mod)
    return mod


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def time_reference_torch(T, H, steps=None, warmup=1, seconds=None):
    """Time the reference's own torch_chunk_gated_delta_rule (qwen3_5_transformers.py:110-187) on the host
    cores at B=1, T, H on the headline's inputs (same seed, generated on the host); returns (times, cores) or
    None without the reference install."""
    ref = load_reference_module("qwen3_5_transformers")
    if ref is None:
        return None
    import torch
    cores = host_threads()
    torch.set_num_threads(cores)  # torchrun sets OMP_NUM_THREADS=1; use every core this process may run on
    q, k, v, g, beta, s0 = make_inputs(torch, 1, T, H, seed=1234, device="cpu")

    def one():
        ref.torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=CHUNK, initial_state=s0,
                                         output_final_state=True, use_qk_l2norm_in_kernel=True)

    with torch.no_grad():
        for _ in range(warmup):
            one()
        times = []
        t_start = time.perf_counter()
        while True:
            t = time.perf_counter()
            one()
            times.append(time.perf_counter() - t)
            if steps is not None and len(times) >= steps:
                break
            if seconds is not None and time.perf_counter() - t_start >= seconds and len(times) >= 3:
                break
    return times, cores


def time_reference_triton(torch, flush, device, H, Ts, reps=10):
    """The reference's GPU path, fast_chunk_gated_delta_rule(backend="triton") (qwen3_5_cutedsl_kernels.py:
    462-567: its Triton intra-chunk kernel plus the Python inter-chunk loop), at the correct [B,T,H,D] layout,
    beside this package's call on the same tensors, cold L2, at each T of config 2."""
    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule
    try:
        kern = load_reference_module("qwen3_5_cutedsl_kernels")
    except Exception as e:  # the reference module failed to import here
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    if kern is None:
        return {"unavailable": "baseline/_ref (the reference install) is absent"}
    if not getattr(kern, "_TRITON_OK", False):
        return {"unavailable": "triton is not importable"}
    res = {"workload": f"B=1, T in {list(Ts)}, H={H}, bf16 q/k/v, fp32 g/beta/state, l2norm in kernel, initial "
                       "and final state; cold L2; median of device times"}
    for T in Ts:
        q, k, v, g, beta, s0 = make_inputs(torch, 1, T, H, seed=1234, device=device)
        args = dict(chunk_size=CHUNK, initial_state=s0, output_final_state=True, use_qk_l2norm_in_kernel=True)

        def ref_fn():
            return kern.fast_chunk_gated_delta_rule(q, k, v, g, beta, backend="triton", **args)

        def our_fn():
            return fast_chunk_gated_delta_rule(q, k, v, g, beta, **args)

        r_ms = _cold_median(torch, ref_fn, flush, reps)
        o_ms = _cold_median(torch, our_fn, flush, reps)
        ro, rs = ref_fn()
        oo, os_ = our_fn()
        rel = float((oo.float() - ro.float()).norm() / ro.float().norm())
        res[str(T)] = {"reference_triton_ms": r_ms, "ours_ms": o_ms, "speedup": r_ms / o_ms,
                       "out_rel_l2_ours_vs_reference": rel}
    return res


def cpu_threads():
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        return max((i.get("num_threads", 1) for i in info), default=1)
    except Exception:
        return 1


def time_oracle(T_sample, H, seconds=None, steps=None, warmup=0):
    """Time the oracle port of torch_chunk_gated_delta_rule on a B=1, T_sample, H sample."""
    import numpy as np

    from oracle import gdn_oracle as O
    q, k, v, g, beta, s0 = O.make_inputs(1, T_sample, H, seed=0, in_dtype="bf16", init_state_std=0.02)

    def one():
        O.chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                 use_qk_l2norm_in_kernel=True, in_dtype="bf16")

    for _ in range(warmup):
        one()
    times = []
    t_start = time.perf_counter()
    while True:
        t = time.perf_counter()
        one()
        times.append(time.perf_counter() - t)
        if steps is not None and len(times) >= steps:
            break
        if seconds is not None and time.perf_counter() - t_start >= seconds and len(times) >= 2:
            break
    return times


def run_reference(args, rank, world):
    if rank != 0:
        return
    timed = time_reference_torch(args.T, args.H, steps=max(1, args.steps), warmup=max(0, args.warmup))
    if timed is not None:
        times, cores = timed
        T_run, kind = args.T, "reference"
        sample = (f"B=1, T={args.T}, H={args.H}, bf16 q/k/v, fp32 g/beta/state (the GPU arm's rank-0 inputs, "
                  f"seed 1234), l2norm in kernel, initial and final state; torch_chunk_gated_delta_rule from "
                  f"the unmodified reference install, torch on {cores} host threads")
        note = "the reference's own CPU path (qwen3_5_transformers.py:110-187) at the full configuration"
    else:  # no reference install on this box: the numpy port of the same algorithm on a sample
        T_run = min(1024, args.T)
        times = time_oracle(T_run, args.H, steps=max(1, args.steps), warmup=max(0, args.warmup))
        cores, kind = cpu_threads(), "port"
        sample = f"B=1, first {T_run} of T={args.T} tokens, H={args.H}, bf16 inputs (numpy oracle port)"
        note = "baseline/_ref absent: the numpy port in oracle/gdn_oracle.py (pinned to the reference's outputs)"
    mean_s = statistics.mean(times)
    value = args.B * T_run / mean_s
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": mean_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"gdn_chunk_fwd B={args.B} T={args.T} H={args.H} Dk=Dv=128 chunk=64 bf16 q/k/v, "
                               "fp32 g/beta/state, l2norm in kernel, final state out",
                   "global_batch": args.B, "seq_len": args.T, "heads": args.H, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm

def sequence_parallel_leg(torch, dist, rank, world, device, flush, T, H, steps, warmup):
    """Config 5: B=1, one sequence of T tokens, contiguous time shards, one per rank (strong scaling).  A step =
    shard summary + all_gather of (transition, local state) + start-state composition + shard finish; device
    time per step (CUDA events), max over ranks."""
    from llms_from_scratch_b200 import _lib
    from llms_from_scratch_b200.parallel import chunk_shard_finish, chunk_shard_summary, compose_start_states
    lo, hi = T * rank // world, T * (rank + 1) // world
    q, k, v, g, beta, s0 = make_inputs(torch, 1, hi - lo, H, seed=77 + rank, device=device)
    ws = torch.empty(_lib.load().gdn_chunk_workspace_bytes(1, hi - lo, H, D, D, _lib.GDN_BF16), dtype=torch.uint8,
                     device=device)

    def step():
        M, b, _ = chunk_shard_summary(q, k, v, g, beta, True, ws)
        packed = torch.stack([M, b])
        if world > 1:
            gathered = [torch.empty_like(packed) for _ in range(world)]
            dist.all_gather(gathered, packed)
        else:
            gathered = [packed]
        start = s0 if rank == 0 else compose_start_states([x[0] for x in gathered[:rank]],
                                                           [x[1] for x in gathered[:rank]], s0)[rank]
        return chunk_shard_finish(q, k, v, g, beta, start, True, True, ws)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush(i)
        evs[i][0].record()
        step()
        evs[i][1].record()
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b_) for a, b_ in evs)
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del q, k, v, g, beta, ws
    return {"workload": f"config 5: B=1 T={T} H={H} bf16, time-sharded x{world} (summary + all_gather + compose + "
                        "finish), strong scaling", "ms": ms, "tok_s": T / (ms / 1e3), "n_gpus": world}


def batched_leg(torch, dist, rank, world, device, flush, B_global, T, H, steps, warmup):
    """Config 3: a global batch of B_global sequences of T tokens sharded by batch over the ranks (no
    collective); whole-job tok/s from the max over ranks of the per-step device time."""
    from llms_from_scratch_b200 import _lib, fast_chunk_gated_delta_rule
    Bl = B_global // world
    q, k, v, g, beta, s0 = make_inputs(torch, Bl, T, H, seed=4321 + rank, device=device)
    ws = torch.empty(_lib.load().gdn_chunk_workspace_bytes(Bl, T, H, D, D, _lib.GDN_BF16), dtype=torch.uint8,
                     device=device)

    def step():
        return fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=s0, output_final_state=True,
                                           use_qk_l2norm_in_kernel=True, workspace=ws)

    ms = _timed_steps(torch, dist, world, device, step, flush, steps, warmup)
    del q, k, v, g, beta, ws
    return {"workload": f"config 3: global B={B_global} T={T} H={H} bf16, {Bl} sequences per rank (batch x head "
                        f"shards, no collective)", "ms": ms, "tok_s": B_global * T / (ms / 1e3), "n_gpus": world}


def _timed_steps(torch, dist, world, device, step, flush, steps, warmup):
    """Mean device time per step (CUDA events, cold L2), max over ranks."""
    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush(i)
        evs[i][0].record()
        step()
        evs[i][1].record()
    torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b_) for a, b_ in evs)
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def decode_model_leg(torch, device, peak, batches=(1, 32), steps=200, prompt_len=26):
    """Config 4: the Qwen3.5-0.8B-shaped decoder with random N(0, 0.02) weights (drawn on the device), a
    prompt of 26 uniform-random ids per sequence, then `steps` greedy decode steps (each a CUDA-graph replay
    of the whole step: 18 linear-attention layers through the recurrent kernel, 6 attention layers over the
    KV cache, the LM head and the argmax), at batch 1 and 32.  Device time by CUDA events; decode tok/s =
    B * steps / decode time.  A profiled eager pass of a few steps gives each kernel family's share of the
    step and the recurrent kernel's achieved GB/s."""
    from llms_from_scratch_b200.model import QWEN3_5_0_8B, Qwen35Decoder, count_parameters, random_weights
    cfg = QWEN3_5_0_8B
    w = random_weights(cfg, seed=0, device=device)
    dec = Qwen35Decoder(cfg, w, device=device, max_len=prompt_len + steps + 2)
    del w
    res = {"workload": f"random-init Qwen3.5-0.8B-shaped decoder ({count_parameters(cfg) / 1e6:.0f} M parameters, "
                       f"hidden 1024, 24 layers: 18 GatedDeltaNet + 6 full attention, vocab {cfg['vocab_size']}, "
                       f"bf16, weights ~ N(0, 0.02)); prefill of {prompt_len} uniform-random ids, then {steps} greedy "
                       "decode steps (one CUDA-graph replay each)", "steps": steps}
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    n_gdn = sum(1 for t in cfg["layer_types"] if t == "linear_attention")
    for B in batches:
        prompt = torch.randint(0, cfg["vocab_size"], (B, prompt_len), device=device, generator=gen)
        cache = dec.new_cache(B)
        dec.generate(prompt, steps, cache=cache)  # warm-up; captures the decode graph for this cache
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        runs = []
        for _ in range(3):
            ev[0].record()
            logits = dec.prefill(prompt, cache)
            ev[1].record()
            dec.step_tokens.copy_(logits.argmax(-1))
            for _ in range(steps):
                dec._graph.replay()
            ev[2].record()
            torch.cuda.synchronize()
            runs.append((ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])))
        prefill_ms = statistics.median(r[0] for r in runs)
        decode_ms = statistics.median(r[1] for r in runs)
        ms_tok = decode_ms / steps
        # kernel shares from a profiled eager pass of 8 decode steps (the same kernels the graph replays)
        share, rec_us = _decode_kernel_shares(torch, dec, cache, prompt, 8)
        # per (sequence, head): the fp32 state in and out; its 3 x 128 conv channels (4 bf16 taps in and out,
        # 4 weights, the new input); z and the output row; g/beta inputs
        Hh = cfg["linear_num_value_heads"]
        rec_bytes = B * Hh * (2 * STATE_BYTES + 384 * (8 + 8 + 8 + 2) + 2 * D * 2 + 4)
        res[f"batch{B}"] = {
            "tok_s": B * steps / (decode_ms / 1e3), "ms_per_token": ms_tok, "prefill_ms": prefill_ms,
            "kernel_share": share,
            "recurrent_kernel": {"kernel": "gdn_model_gdn_decode_kernel (conv update + gates + recurrent rule + "
                                           "gated norm, one token)", "us_per_layer": rec_us,
                                 "bytes_per_layer": rec_bytes,
                                 "achieved_gbs": rec_bytes / (rec_us / 1e6) / 1e9 if rec_us else None,
                                 "frac_hbm": rec_bytes / (rec_us / 1e6) / 1e9 / peak if rec_us else None,
                                 "layers_per_step": n_gdn},
        }
        del cache
        dec._graph = None
        torch.cuda.empty_cache()
    res["batch1_tok_s"] = res["batch1"]["tok_s"] if "batch1" in res else None
    res["batch32_tok_s"] = res["batch32"]["tok_s"] if "batch32" in res else None
    return res


def reference_decode_leg(torch, device, batches=(1, 32), steps=200, prompt_len=26):
    """The reference's own decode on the GPU, for comparison with ``decode_model``: its ``Qwen3_5Model``
    (unmodified install in baseline/_ref) at the same shape and random N(0, 0.02) weights, bf16, its
    GatedDeltaNet layers on its Triton path (``benchmark.patch_model_backend("triton")``,
    benchmark.py:254-280), greedy generation by its ``generate_text_basic_stream`` (qwen3_5.py:483-495:
    the whole prefix re-run for every token, no cache).  Device time by CUDA events around the
    generation of ``steps`` tokens after the same 26-token prompt."""
    if not os.path.exists(os.path.join(REF_DIR, "qwen3_5.py")):
        return {"unavailable": "baseline/_ref (the reference install) is absent"}
    names = ("qwen3_5_cutedsl_kernels", "qwen3_5_transformers", "qwen3_5", "benchmark")
    saved = {k: sys.modules.pop(k) for k in names if k in sys.modules}
    sys.path.insert(0, REF_DIR)
    try:
        import benchmark as ref_bench
        import qwen3_5 as ref_model
        from llms_from_scratch_b200.model import QWEN3_5_0_8B, random_weights
        ref_bench.patch_model_backend("triton")
        cfg = dict(ref_model.QWEN3_5_CONFIG)
        cfg.update({k: v for k, v in QWEN3_5_0_8B.items() if k in cfg})
        cfg.update(layer_types=list(QWEN3_5_0_8B["layer_types"]), context_length=prompt_len + steps + 8,
                   dtype=torch.bfloat16)
        with torch.device(device):
            model = ref_model.Qwen3_5Model(cfg)
        model.load_state_dict(random_weights(QWEN3_5_0_8B, seed=0, device=device), strict=True)
        model.eval()
        res = {"workload": f"the reference's Qwen3_5Model, same shape and weights as decode_model, bf16, GatedDeltaNet "
                           f"layers on its Triton backend; prompt of {prompt_len} ids, {steps} greedy tokens by its "
                           "generate_text_basic_stream (no cache: the whole prefix re-run per token)", "steps": steps}
        gen = torch.Generator(device=device)
        gen.manual_seed(11)
        for B in batches:
            prompt = torch.randint(0, cfg["vocab_size"], (B, prompt_len), device=device, generator=gen)
            for _ in ref_model.generate_text_basic_stream(model, prompt, 2):  # warm-up (Triton compile)
                pass
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            n = 0
            for _ in ref_model.generate_text_basic_stream(model, prompt, steps):
                n += 1
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b)
            res[f"batch{B}"] = {"tok_s": B * n / (ms / 1e3), "ms_per_token": ms / n}
        del model
        torch.cuda.empty_cache()
        return res
    except Exception as e:  # the reference's GPU path failed to run here: report, do not fail the bench
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    finally:
        sys.path.remove(REF_DIR)
        for k in names:
            sys.modules.pop(k, None)
        sys.modules.update(saved)


def _decode_kernel_shares(torch, dec, cache, prompt, n):
    """Device-time share of each kernel family over n eager decode steps (torch profiler), and the mean
    duration of the recurrent kernel in microseconds."""
    try:
        return _decode_kernel_shares_inner(torch, dec, cache, prompt, n)
    except Exception as e:  # a profiler that cannot trace here leaves the shares unreported, not the leg
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}, None


def _decode_kernel_shares_inner(torch, dec, cache, prompt, n):
    from torch.profiler import ProfilerActivity, profile
    logits = dec.prefill(prompt, cache)
    tok = logits.argmax(-1)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            tok = dec.decode_step(tok, cache).argmax(-1)
        torch.cuda.synchronize()
    fam = {"GatedDeltaNet decode (gdn_model_gdn_decode: conv update, gates, recurrent rule, gated norm)":
               ("gdn_model_gdn_decode", "gdn_recurrent", "conv_update", "gates_kernel", "rms_norm_gated"),
           "projections (gdn_model_gemm_kernel; cuBLAS for the prefill)": ("gemm", "gemv", "nvjet", "cutlass", "sm100",
                                                                           "xmma"),
           "attention (gdn_model_attention + attn_prep)": ("gdn_model_attention", "gdn_model_attn_prep"),
           "residual add + RMSNorm (gdn_model_add_rms_norm)": ("add_rms_norm",), "silu_mul": ("silu_mul",)}
    tot, by, rec = 0.0, {k: 0.0 for k in fam}, []
    by["other (embedding, argmax, copies)"] = 0.0
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        t = e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total
        tot += t
        name = e.name.lower()
        for k, keys in fam.items():
            if any(x in name for x in keys):
                by[k] += t
                break
        else:
            by["other (embedding, argmax, copies)"] += t
        if "gdn_model_gdn_decode" in name or "gdn_recurrent" in name:
            rec.append(t)
    share = {k: v / tot for k, v in by.items()} if tot else {}
    return share, (statistics.mean(rec) if rec else None)


def run_sequence_parallel(args, rank, world, local):
    """``--sp``: config 5 alone, printed as its own JSON line."""
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    flush = L2Flush(torch, device)
    r = sequence_parallel_leg(torch, dist, rank, world, device, flush, args.sp_T, args.H, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps({
            "metric": "GDN chunk-fwd tok/s, sequence parallel @B=1,T=%d" % args.sp_T, "value": r["tok_s"],
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": r["workload"], "global_batch": 1, "seq_len": args.sp_T,
                       "parallelism": f"sequence-parallel x{world}", "l2": L2_NOTE},
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.sp:
        run_sequence_parallel(args, rank, world, local)
        return

    import torch
    import torch.distributed as dist

    from llms_from_scratch_b200 import (_lib, chunk_host_workspace_bytes, fast_chunk_gated_delta_rule,
                                        fast_recurrent_gated_delta_rule)

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = _lib.load()
    B, T, H = args.B, args.T, args.H
    q, k, v, g, beta, s0 = make_inputs(torch, B, T, H, seed=1234 + rank, device=device, on_host=True)
    ws = torch.empty(lib.gdn_chunk_workspace_bytes(B, T, H, D, D, _lib.GDN_BF16), dtype=torch.uint8, device=device)
    flush = L2Flush(torch, device)

    def step():
        return fast_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=CHUNK, initial_state=s0,
                                           output_final_state=True, use_qk_l2norm_in_kernel=True, workspace=ws)

    clocks = ClockSampler(local)
    clocks.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_seconds:
        for _ in range(10):
            step()
        torch.cuda.synchronize()

    # ---- timed region: K steps, cold L2 before each
    K = args.steps
    n_phase = 3
    outer = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    phase = [[torch.cuda.Event(enable_timing=True) for _ in range(n_phase)] for _ in range(K)]
    for evs in phase:
        for e in evs:
            e.record()
    for a, b in outer:
        a.record()
        b.record()
    torch.cuda.synchronize()
    phase_arrays = [(ctypes.c_void_p * n_phase)(*[e.cuda_event for e in evs]) for evs in phase]

    barrier()
    torch.cuda.synchronize()
    launches0 = lib.gdn_launch_count()
    t_timed0 = time.perf_counter()
    host_s = []
    for i in range(K):  # the production call: no instrumentation between its kernels
        flush(i)
        outer[i][0].record()
        th = time.perf_counter()
        step()
        host_s.append(time.perf_counter() - th)
        outer[i][1].record()
    torch.cuda.synchronize()
    barrier()
    t_timed1 = time.perf_counter()
    launches = lib.gdn_launch_count() - launches0
    step_ms = [a.elapsed_time(b) for a, b in outer]
    # The same K steps again with the library's phase events between its kernels (the event between prep and
    # scan costs the launch pipelining, ~10 us a step): the per-kernel durations of the roofline.
    for i in range(K):
        flush(i)
        lib.gdn_set_phase_events(phase_arrays[i], n_phase)
        step()
    lib.gdn_set_phase_events(None, 0)
    torch.cuda.synchronize()
    barrier()
    prep_ms = [evs[0].elapsed_time(evs[1]) for evs in phase]
    scan_ms = [evs[1].elapsed_time(evs[2]) for evs in phase]
    ms_local = statistics.mean(step_ms)
    ms = max_over_ranks(ms_local)
    host_us_local = statistics.mean(host_s) * 1e6
    per_rank = [[ms_local, host_us_local]]
    if world > 1:
        mine = torch.tensor([ms_local, host_us_local], device=device, dtype=torch.float64)
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [x.tolist() for x in allr]
    tokens_job = world * B * T
    value = tokens_job / (ms / 1e3)

    # ---- end to end through the public API with host buffers
    hq, hk, hv, hg, hb, hs = (x.cpu().pin_memory() for x in (q, k, v, g, beta, s0))
    ho = torch.empty((B, T, H, D), dtype=torch.bfloat16).pin_memory()
    hst = torch.empty((B, H, D, D), dtype=torch.float32).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hg, hb, hs))
    d2h = ho.numel() * ho.element_size() + hst.numel() * hst.element_size()

    hws = torch.empty((chunk_host_workspace_bytes(B, T, H, D, D, torch.bfloat16),), dtype=torch.uint8, device=device)

    def e2e_step():
        # host tensors in, host tensors out: the op pipelines the PCIe copies against the compute
        o, st = fast_chunk_gated_delta_rule(hq, hk, hv, hg, hb, chunk_size=CHUNK, initial_state=hs,
                                            output_final_state=True, use_qk_l2norm_in_kernel=True, workspace=hws)
        assert o.shape == ho.shape and st.shape == hst.shape

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        flush(i)
        e2e_ev[i][0].record()
        e2e_step()
        e2e_ev[i][1].record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in e2e_ev))
    t_end = time.perf_counter()
    clocks.stop()

    # ---- decode step kernel (config 4 shape, one GatedDeltaNet layer at batch 32)
    Bd = args.decode_batch
    dq_, dk_, dv_, dg_, db_, dst = make_inputs(torch, Bd, 1, H, seed=99 + rank, device=device)
    dstate = dst.clone()
    for _ in range(5):
        fast_recurrent_gated_delta_rule(dq_, dk_, dv_, dg_, db_, dstate, True, use_qk_l2norm_in_kernel=True,
                                        out_state=dstate)
    dec_ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for e in dec_ev:
        e.record()
    torch.cuda.synchronize()
    dec_arr = (ctypes.c_void_p * 2)(*[e.cuda_event for e in dec_ev])
    dec_times = []
    for i in range(20):
        flush(i)
        lib.gdn_set_phase_events(dec_arr, 2)
        fast_recurrent_gated_delta_rule(dq_, dk_, dv_, dg_, db_, dstate, True, use_qk_l2norm_in_kernel=True,
                                        out_state=dstate)
        lib.gdn_set_phase_events(None, 0)
        torch.cuda.synchronize()
        dec_times.append(dec_ev[0].elapsed_time(dec_ev[1]))
    dec_ms = statistics.median(dec_times)
    dec_bytes = Bd * H * (2 * STATE_BYTES + 4 * D * 2 + 8)
    # the same step back to back, as a decode graph runs it: ten launches captured in one CUDA graph, each on
    # its own state (ten states: larger than L2), L2 flushed before every replay
    gstates = [dstate.clone() for _ in range(10)]
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for s_ in gstates:  # warm-up outside the capture
            fast_recurrent_gated_delta_rule(dq_, dk_, dv_, dg_, db_, s_, True, use_qk_l2norm_in_kernel=True, out_state=s_)
    torch.cuda.current_stream(device).wait_stream(side)
    dgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dgraph, stream=side):
        for s_ in gstates:
            fast_recurrent_gated_delta_rule(dq_, dk_, dv_, dg_, db_, s_, True, use_qk_l2norm_in_kernel=True, out_state=s_)
    torch.cuda.synchronize()
    graph_ms = []
    for i in range(10):
        flush(i)
        dec_ev[0].record()
        dgraph.replay()
        dec_ev[1].record()
        torch.cuda.synchronize()
        graph_ms.append(dec_ev[0].elapsed_time(dec_ev[1]) / len(gstates))
    dec_graph_ms = statistics.median(graph_ms)
    del dgraph, gstates
    peak_l, _ = load_peaks()
    layer_kernels = time_layer_kernels(torch, lib, flush, device, T, H, Bd, peak_l)
    backward = time_backward(torch, lib, flush, device, T, H)
    # ---- configs 3 and 5 over the same ranks (extra keys; the headline stays config 2 per rank)
    batched = sp = None
    if not args.no_configs35:
        batched = batched_leg(torch, dist, rank, world, device, flush, 64, 4096, H, steps=5, warmup=3)
        sp = sequence_parallel_leg(torch, dist, rank, world, device, flush, args.sp_T, H, steps=5, warmup=3)
        torch.cuda.empty_cache()
    decode_model = None
    if not args.no_decode_model:
        decode_model = decode_model_leg(torch, device, peak_l)
        torch.cuda.empty_cache()
        if world > 1:  # config 4 runs as replicas: every GPU decodes its own batch, no exchange
            mine = torch.tensor([decode_model["batch1_tok_s"] or 0.0, decode_model["batch32_tok_s"] or 0.0],
                                dtype=torch.float64, device=device)
            allr = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allr, mine)
            per = [x.tolist() for x in allr]
            decode_model["replicas"] = {"n": world, "scaling": "replicas (each GPU decodes its own batch; no exchange)",
                                        "batch1_tok_s_total": sum(x[0] for x in per),
                                        "batch32_tok_s_total": sum(x[1] for x in per),
                                        "per_rank": [{"rank": r, "batch1_tok_s": x[0], "batch32_tok_s": x[1]}
                                                     for r, x in enumerate(per)]}
        if rank == 0 and not args.no_reference_triton:
            decode_model["reference_decode"] = reference_decode_leg(torch, device)
    ref_triton = None
    if rank == 0 and not args.no_reference_triton:
        ref_triton = time_reference_triton(torch, flush, device, H, (256, 512, 1024, 2048, 4096))
    fla, fla_err = load_fla() if args.fla else (None, None)
    packed = time_packed(torch, flush, device, H, peak_l, fla=fla)
    fla_headline = None
    if args.fla:
        if fla is None:
            fla_headline = {"unavailable": fla_err}
        else:
            s_vk = s0.transpose(-1, -2).contiguous()
            fla_ms = _cold_median(torch, lambda: fla(q=q, k=k, v=v, g=g, beta=beta, initial_state=s_vk,
                                                     output_final_state=True, use_qk_l2norm_in_kernel=True),
                                  flush, 20)
            fla_headline = {"workload": f"B={B} T={T} H={H} (the headline workload)", "ms": fla_ms,
                            "tok_s": B * T / (fla_ms / 1e3)}

    # ---- roofline of the dominant kernel
    peak, peak_kind = load_peaks()
    prep_avg, scan_avg = statistics.mean(prep_ms), statistics.mean(scan_ms)
    kernels = {
        "gdn_prep": (prep_avg, B * H * T * (3 * D * 2 + 8)),                    # reads q, k, v, g, beta
        "gdn_scan": (scan_avg, B * H * T * D * 2 + 2 * B * H * STATE_BYTES),  # writes o; state in + out
    }
    dom = max(kernels, key=lambda n: kernels[n][0])
    dom_ms, dom_bytes = kernels[dom]
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    workload = f"B{B}_T{T}_H{H}_bf16"
    traffic = load_traffic(dom, workload)
    step_bytes = B * H * T * BYTES_PER_TOKEN_HEAD + 2 * B * H * STATE_BYTES

    cpu = cpu_port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        timed = time_reference_torch(T, H, warmup=1, seconds=args.cpu_seconds)
        if timed is not None:
            times, cores = timed
            cpu = {"value": B * T / statistics.mean(times), "unit": UNIT, "cores": cores, "kind": "reference",
                   "sample": f"B=1, T={T}, H={H}: the headline's rank-0 inputs, {len(times)} runs of the reference's "
                             f"own torch_chunk_gated_delta_rule (unmodified install) on {cores} host threads"}
        T_sample = min(1024, T)
        times = time_oracle(T_sample, H, seconds=min(3.0, args.cpu_seconds), warmup=1)
        cpu_port = {"value": T_sample / statistics.mean(times), "unit": UNIT, "cores": cpu_threads(),
                    "kind": "port", "sample": f"B=1, first {T_sample} of T={T} tokens, H={H}, bf16 inputs, "
                                              f"{len(times)} runs (numpy oracle port)"}
        if cpu is None:
            cpu = cpu_port

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"gdn_chunk_fwd B={B} T={T} H={H} Dk=Dv=128 chunk=64 bf16 q/k/v, fp32 g/beta/"
                                   "state, l2norm in kernel, final state out",
                       "global_batch": world * B, "seq_len": T, "heads": H,
                       "parallelism": f"batch-shard x{world} (no collective)",
                       "l2": L2_NOTE},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": dom_bytes, "ms_per_launch": dom_ms,
                         "kernel_timing": "library phase events (CUDA events on the launching stream) around each "
                                          "kernel, in a second pass of the same K steps after the timed one"},
            "step_roofline": {"algorithmic_bytes": step_bytes, "achieved_gbs": step_bytes / (ms / 1e3) / 1e9,
                              "frac": step_bytes / (ms / 1e3) / 1e9 / peak},
            "kernels_ms": {"gdn_prep": prep_avg, "gdn_scan": scan_avg},
            "e2e": {"value": tokens_job / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": launches,
            "per_rank": [{"rank": r, "step_ms": v[0], "host_enqueue_us": v[1]} for r, v in enumerate(per_rank)],
            "decode_model": decode_model,
            "batched_b64": batched,
            "sp": sp,
            "clocks": clocks.summary(t_soak, t_end),
            "layer_kernels": layer_kernels,
            "packed_prefill": packed,
            "backward": backward,
            "decode_step": {"workload": f"recurrent step B={Bd} H={H} (one GatedDeltaNet layer)",
                            "ms": dec_ms, "achieved_gbs": dec_bytes / (dec_ms / 1e3) / 1e9,
                            "frac_hbm": dec_bytes / (dec_ms / 1e3) / 1e9 / peak,
                            "timing": "ms: one launch between CUDA events, cold L2; ms_back_to_back: ten launches "
                                      "on ten states in one CUDA graph, cold L2, per launch",
                            "ms_back_to_back": dec_graph_ms,
                            "frac_hbm_back_to_back": dec_bytes / (dec_graph_ms / 1e3) / 1e9 / peak},
            "cpu_baseline": cpu,
            "cpu_port": cpu_port,
            "reference_triton": ref_triton,
        }
        if fla_headline is not None:
            line["vllm_fla"] = fla_headline
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
