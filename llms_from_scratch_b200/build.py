"""Build the sm_100a shared library ``libgdn_b200.so`` in-tree with nvcc.

    python -m llms_from_scratch_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel), then
one link produces ``llms_from_scratch_b200/libgdn_b200.so``.  Objects are
rebuilt when a source or header is newer.  nvcc cross-compiles, so no GPU is
needed to build.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libgdn_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + INCLUDE, "-I" + CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, obj: str, verbose: bool, extra=()):
    cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdr_time = _newest(_headers())
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if force or ptxas_info or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_time):
            jobs.append((s, o))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if ptxas_info and msg:
                    print(f"== {os.path.basename(futs[f])}\n{msg}")
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


TORCH_OPS_SRC = os.path.join(CSRC, "gdn_torch_ops.cpp")
TORCH_OPS_LIB = os.path.join(PKG, "libgdn_torch_ops.so")


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile the PyTorch operator library (torch.ops.gdn.*, ``csrc/gdn_torch_ops.cpp``) against the
    installed torch and link it to ``libgdn_b200.so`` (found next to it at run time)."""
    import torch
    from torch.utils import cpp_extension as ce
    deps = [TORCH_OPS_SRC, LIB, os.path.join(INCLUDE, "gdn_b200.h")]
    if not force and os.path.exists(TORCH_OPS_LIB) and os.path.getmtime(TORCH_OPS_LIB) >= _newest(deps):
        return TORCH_OPS_LIB
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    cmd += [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + ["-I" + INCLUDE, TORCH_OPS_SRC,
                                                                        "-o", TORCH_OPS_LIB]
    cmd += [f"-L{p}" for p in ce.library_paths(device_type="cuda")] + ["-L" + PKG, "-lgdn_b200", "-lc10", "-lc10_cuda",
                                                                       "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
                                                                       "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch operator library build failed:\n{r.stdout}\n{r.stderr}")
    return TORCH_OPS_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
    print(build_torch_ops(force=a.force, verbose=a.verbose))
    sys.exit(0)
