"""Drop-in GatedDeltaNet ops backed by the sm_100a CUDA library.

``fast_chunk_gated_delta_rule`` keeps the reference's exact signature
(qwen3_5_cutedsl_kernels.py:462-473) and return convention
(``(out [B,T,H,Dv] in query.dtype, final_state [B,H,Dk,Dv] fp32 or None)``).
``fast_recurrent_gated_delta_rule`` keeps the signature of
``torch_recurrent_gated_delta_rule`` (qwen3_5_transformers.py:190-192).

Both allocate their outputs (the caller owns them), never modify inputs, run
asynchronously on the current CUDA stream, and raise ``RuntimeError`` (a
``GDNError``) on bad arguments, as the reference's torch ops do.

``fast_chunk_gated_delta_rule`` given CPU tensors computes them on the current
CUDA device through ``gdn_chunk_gated_delta_rule_host``: the library streams
time slices in and out over PCIe while earlier slices compute, and the call
returns page-locked CPU outputs once they have landed.  There is no CPU compute
path: without a CUDA device, CPU tensors raise.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GDN_F32, torch.bfloat16: _lib.GDN_BF16, torch.float16: _lib.GDN_F16}

# backend names accepted for drop-in compatibility; all run this package's CUDA kernels
_CUDA_BACKENDS = ("auto", "cuda", "b200", "triton", "cute")


def l2norm(x: torch.Tensor, dim: int = -1, eps: float = 1e-6) -> torch.Tensor:
    """Same as the reference helper (qwen3_5_cutedsl_kernels.py:100-101)."""
    return x * torch.rsqrt((x * x).sum(dim=dim, keepdim=True) + eps)


def get_backend() -> str:
    """The backend ``backend="auto"`` resolves to (qwen3_5_cutedsl_kernels.py:104-109)."""
    return "cuda"


def _as_kernel_tensor(x: torch.Tensor, name: str, ndim: int) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if x.dim() != ndim:
        raise RuntimeError(f"{name} must have {ndim} dims, got shape {tuple(x.shape)}")
    if x.device.type != "cuda":
        raise RuntimeError(f"{name} is on {x.device}; the GatedDeltaNet kernels need CUDA tensors (no CPU path)")
    if x.dtype not in _DTYPES:
        x = x.float()
    if ndim == 4 and x.shape[-1] > 1 and x.stride(-1) != 1:
        x = x.contiguous()
    return x


def _desc(x: torch.Tensor) -> _lib.GdnTensor:
    d = _lib.GdnTensor()
    d.data = x.data_ptr() if x.numel() > 0 else 0
    d.dtype = _DTYPES[x.dtype]
    d.ndim = x.dim()
    for i in range(4):
        d.shape[i] = x.shape[i] if i < x.dim() else 1
        d.stride[i] = x.stride(i) if i < x.dim() else 1
    return d


def _state_in(initial_state: Optional[torch.Tensor], B, H, Dk, Dv, device) -> Optional[torch.Tensor]:
    if initial_state is None:
        return None
    if tuple(initial_state.shape) != (B, H, Dk, Dv):
        raise RuntimeError(f"initial_state must have shape {(B, H, Dk, Dv)}, got {tuple(initial_state.shape)}")
    if initial_state.device != device:
        raise RuntimeError(f"initial_state is on {initial_state.device}, expected {device}")
    return initial_state.to(torch.float32).contiguous()


_ERROR_BITS = {1: "a chunk prep wait timed out", 2: "a chunk scan wait timed out",
               8: "packed-sequence offsets were not a valid cu_seqlens", 16: "bounded-wait self-test"}


def _raise_pending(lib, dev: torch.device) -> None:
    """With ``dev`` current: raise GDNError (GDN_ERR_KERNEL) if the library's host mirror of the device error
    word shows a failure (one host read, no synchronisation), clearing the word."""
    bits = lib.gdn_device_error_pending()
    if bits:
        bits = lib.gdn_device_error(1) or bits
        what = "; ".join(v for b, v in _ERROR_BITS.items() if bits & b) or "unknown"
        raise _lib.GDNError(_lib.GDN_ERR_KERNEL, "GDN_ERR_KERNEL",
                            f"a kernel on {dev} reported device error bits 0x{bits:x} ({what}); the outputs of "
                            "the call that launched it are not valid")


def check_device_errors(device: Optional[torch.device] = None, sync: bool = False) -> None:
    """Raise ``GDNError`` (``GDN_ERR_KERNEL``) if a kernel on ``device`` (default: the current one) reported a
    failure in the library's device error word, and clear the word.

    Every op runs this check before it launches: it reads the page-locked host mirror the kernels write their
    error bits into, so it costs no synchronisation, and a failure surfaces at the next op on the device.
    ``sync=True`` first waits for the device, so the latest call's kernels are covered too."""
    dev = torch.device(device) if device is not None else None
    if dev is None or dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    with torch.cuda.device(dev):
        if sync:
            torch.cuda.synchronize(dev)
        _raise_pending(lib, dev)


def _workspace(workspace: Optional[torch.Tensor], need: int, dev: torch.device) -> torch.Tensor:
    """The caller's workspace if it is a large enough CUDA buffer on ``dev``, else a new one.  A workspace on
    another device or on the host is an error, not a silent reallocation: the kernels would write into it."""
    if workspace is not None:
        if not isinstance(workspace, torch.Tensor) or workspace.device != dev:
            where = workspace.device if isinstance(workspace, torch.Tensor) else type(workspace).__name__
            raise RuntimeError(f"workspace is on {where}; it must be a CUDA tensor on {dev}")
        if workspace.numel() * workspace.element_size() >= need and workspace.is_contiguous():
            return workspace
    return torch.empty((max(need, 1),), dtype=torch.uint8, device=dev)


TORCH_OPS_PATH = os.path.join(os.path.dirname(_lib.LIB_PATH), "libgdn_torch_ops.so")
_torch_ops_loaded: Optional[bool] = None


def _torch_ops() -> bool:
    """Load (once) the PyTorch operator library (torch.ops.gdn.chunk_fwd / decode_step, built beside
    libgdn_b200.so by ``build``); False if it was not built, in which case the ops call the C ABI through
    ctypes.  Both routes run the same kernels through the same C entry points."""
    global _torch_ops_loaded
    if _torch_ops_loaded is None:
        _lib.load()  # the operator library links libgdn_b200.so: the same loaded instance serves both
        _torch_ops_loaded = os.path.exists(TORCH_OPS_PATH)
        if _torch_ops_loaded:
            torch.ops.load_library(TORCH_OPS_PATH)
    return _torch_ops_loaded


_STATUS = {"GDN_ERR_INVALID_ARGUMENT": _lib.GDN_ERR_INVALID_ARGUMENT, "GDN_ERR_UNSUPPORTED": _lib.GDN_ERR_UNSUPPORTED,
           "GDN_ERR_WORKSPACE": _lib.GDN_ERR_WORKSPACE, "GDN_ERR_CUDA": _lib.GDN_ERR_CUDA,
           "GDN_ERR_DEVICE": _lib.GDN_ERR_DEVICE, "GDN_ERR_KERNEL": _lib.GDN_ERR_KERNEL}


def _op_error(e: RuntimeError) -> RuntimeError:
    """A torch.ops.gdn error as the GDNError the C ABI status names (argument errors stay RuntimeError)."""
    msg = str(e).split("\nException raised from")[0].strip()
    name, _, rest = msg.partition(": ")
    if name in _STATUS:
        return _lib.GDNError(_STATUS[name], name, rest)
    return RuntimeError(msg)


def _check_backend(backend: str) -> None:
    if backend == "torch":
        raise RuntimeError("backend 'torch' is the reference's pure-PyTorch path; this package runs only its "
                           "CUDA kernels (use backend='auto')")
    if backend not in _CUDA_BACKENDS:
        raise RuntimeError(f"Requested backend '{backend}' is not available.")


def fast_chunk_gated_delta_rule(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    chunk_size: int = 64,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    backend: str = "auto",
    workspace: Optional[torch.Tensor] = None,
    slice_tokens: int = 0,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Chunked gated delta rule forward on the GPU.

    Drop-in for the reference's ``fast_chunk_gated_delta_rule``: same
    arguments, layouts (``[B,T,H,D]``) and outputs.  ``workspace`` optionally
    supplies a reusable uint8 CUDA buffer of at least
    ``chunk_workspace_bytes(...)`` bytes (allocated per call otherwise).

    CPU inputs take the host-buffer path (module docstring): outputs come back
    as page-locked CPU tensors after the call has finished on the device;
    ``workspace`` is then a CUDA buffer of ``chunk_host_workspace_bytes(...)``
    bytes and ``slice_tokens`` the time slice the copies are pipelined in
    (0 = the library's choice).
    """
    _check_backend(backend)
    if isinstance(query, torch.Tensor) and query.device.type == "cpu":
        return _chunk_from_host(query, key, value, g, beta, chunk_size, initial_state, output_final_state,
                                use_qk_l2norm_in_kernel, workspace, slice_tokens)
    if isinstance(query, torch.Tensor) and query.is_cuda and _torch_ops():
        try:
            out, final = torch.ops.gdn.chunk_fwd(query, key, value, g, beta, int(chunk_size), initial_state,
                                                 bool(output_final_state), bool(use_qk_l2norm_in_kernel), workspace)
        except RuntimeError as e:
            raise _op_error(e) from None
        return out, (final if output_final_state else None)
    q = _as_kernel_tensor(query, "query", 4)
    k = _as_kernel_tensor(key, "key", 4)
    v = _as_kernel_tensor(value, "value", 4)
    gg = _as_kernel_tensor(g, "g", 3)
    bb = _as_kernel_tensor(beta, "beta", 3)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    dev = q.device
    for name, x in (("key", k), ("value", v), ("g", gg), ("beta", bb)):
        if x.device != dev:
            raise RuntimeError(f"{name} is on {x.device}, query on {dev}")
    h0 = _state_in(initial_state, B, H, Dk, Dv, dev)
    out_dtype = query.dtype
    out = torch.empty((B, T, H, Dv), dtype=q.dtype, device=dev)
    final = torch.empty((B, H, Dk, Dv), dtype=torch.float32, device=dev) if output_final_state else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        _raise_pending(lib, dev)
        ws_bytes = lib.gdn_chunk_workspace_bytes(B, T, H, Dk, Dv, _DTYPES[q.dtype])
        workspace = _workspace(workspace, ws_bytes, dev)
        dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, gg, bb, out))
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.gdn_chunk_gated_delta_rule(
            ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg), ctypes.byref(db),
            int(chunk_size), h0.data_ptr() if h0 is not None else None, int(bool(output_final_state)),
            int(bool(use_qk_l2norm_in_kernel)), ctypes.byref(do),
            final.data_ptr() if final is not None else None, workspace.data_ptr(), workspace.numel(), stream)
        _lib.check(rc)
    if out.dtype != out_dtype:
        out = out.to(out_dtype)
    return out, final


def chunk_workspace_bytes(B: int, T: int, H: int, Dk: int = 128, Dv: int = 128,
                          dtype: torch.dtype = torch.bfloat16) -> int:
    return int(_lib.load().gdn_chunk_workspace_bytes(B, T, H, Dk, Dv, _DTYPES.get(dtype, _lib.GDN_F32)))


def chunk_host_workspace_bytes(B: int, T: int, H: int, Dk: int = 128, Dv: int = 128,
                               dtype: torch.dtype = torch.bfloat16, slice_tokens: int = 0) -> int:
    """Device bytes the host-buffer path needs (``gdn_chunk_host_workspace_bytes``)."""
    return int(_lib.load().gdn_chunk_host_workspace_bytes(B, T, H, Dk, Dv, _DTYPES.get(dtype, _lib.GDN_F32),
                                                          int(slice_tokens)))


def _host_tensor(x, name: str, ndim: int) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if x.dim() != ndim:
        raise RuntimeError(f"{name} must have {ndim} dims, got shape {tuple(x.shape)}")
    if x.device.type != "cpu":
        raise RuntimeError(f"{name} is on {x.device}, query on cpu")
    if x.dtype not in _DTYPES:
        x = x.float()
    return x.contiguous()


def _chunk_from_host(query, key, value, g, beta, chunk_size, initial_state, output_final_state,
                     use_qk_l2norm_in_kernel, workspace, slice_tokens):
    if not torch.cuda.is_available():
        raise RuntimeError("query is on cpu: the GatedDeltaNet kernels compute host tensors on a CUDA device, "
                           "and none is available (no CPU path)")
    q = _host_tensor(query, "query", 4)
    k = _host_tensor(key, "key", 4)
    v = _host_tensor(value, "value", 4)
    gg = _host_tensor(g, "g", 3)
    bb = _host_tensor(beta, "beta", 3)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    h0 = None
    if initial_state is not None:
        if tuple(initial_state.shape) != (B, H, Dk, Dv):
            raise RuntimeError(f"initial_state must have shape {(B, H, Dk, Dv)}, got {tuple(initial_state.shape)}")
        if initial_state.device.type != "cpu":
            raise RuntimeError(f"initial_state is on {initial_state.device}, query on cpu")
        h0 = initial_state.to(torch.float32).contiguous()
    out = torch.empty((B, T, H, Dv), dtype=q.dtype, pin_memory=True)
    final = torch.empty((B, H, Dk, Dv), dtype=torch.float32, pin_memory=True) if output_final_state else None
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    with torch.cuda.device(dev):
        _raise_pending(lib, dev)
        need = lib.gdn_chunk_host_workspace_bytes(B, T, H, Dk, Dv, _DTYPES[q.dtype], int(slice_tokens))
        workspace = _workspace(workspace, need, dev)
        dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, gg, bb, out))
        stream = torch.cuda.current_stream(dev)
        rc = lib.gdn_chunk_gated_delta_rule_host(
            ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg), ctypes.byref(db),
            int(chunk_size), h0.data_ptr() if h0 is not None else None, int(bool(output_final_state)),
            int(bool(use_qk_l2norm_in_kernel)), ctypes.byref(do), final.data_ptr() if final is not None else None,
            int(slice_tokens), workspace.data_ptr(), workspace.numel(), stream.cuda_stream)
        _lib.check(rc)
        stream.synchronize()  # the outputs are host memory: hand them over complete
    if out.dtype != query.dtype:
        out = out.to(query.dtype)
    return out, final


def fast_recurrent_gated_delta_rule(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    initial_state: Optional[torch.Tensor],
    output_final_state: bool,
    use_qk_l2norm_in_kernel: bool = False,
    out_state: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Token-recurrent gated delta rule (the decode step) on the GPU.

    Same contract as ``torch_recurrent_gated_delta_rule``.  ``out_state``
    optionally names an fp32 ``[B,H,Dk,Dv]`` tensor to receive the final state;
    it may be ``initial_state`` itself for an in-place decode update.
    """
    if isinstance(query, torch.Tensor) and query.is_cuda and _torch_ops():
        try:
            out, final = torch.ops.gdn.decode_step(query, key, value, g, beta, initial_state, bool(output_final_state),
                                                   bool(use_qk_l2norm_in_kernel), out_state)
        except RuntimeError as e:
            raise _op_error(e) from None
        return out, (final if output_final_state else None)
    q = _as_kernel_tensor(query, "query", 4)
    k = _as_kernel_tensor(key, "key", 4)
    v = _as_kernel_tensor(value, "value", 4)
    gg = _as_kernel_tensor(g, "g", 3)
    bb = _as_kernel_tensor(beta, "beta", 3)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    dev = q.device
    h0 = _state_in(initial_state, B, H, Dk, Dv, dev)
    out_dtype = query.dtype
    out = torch.empty((B, T, H, Dv), dtype=q.dtype, device=dev)
    final = None
    if output_final_state:
        if out_state is not None:
            if (out_state.dtype != torch.float32 or tuple(out_state.shape) != (B, H, Dk, Dv)
                    or not out_state.is_contiguous() or out_state.device != dev):
                raise RuntimeError("out_state must be a contiguous fp32 [B,H,Dk,Dv] tensor on the query's device")
            final = out_state
        else:
            final = torch.empty((B, H, Dk, Dv), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _raise_pending(lib, dev)
        dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, gg, bb, out))
        stream = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.gdn_recurrent_gated_delta_rule(
            ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg), ctypes.byref(db),
            h0.data_ptr() if h0 is not None else None, int(bool(output_final_state)),
            int(bool(use_qk_l2norm_in_kernel)), ctypes.byref(do),
            final.data_ptr() if final is not None else None, stream)
        _lib.check(rc)
    if out.dtype != out_dtype:
        out = out.to(out_dtype)
    return out, final


def chunk_varlen_workspace_bytes(T: int, num_seqs: int, H: int, Dk: int = 128, Dv: int = 128,
                                 dtype: torch.dtype = torch.bfloat16) -> int:
    """Device bytes ``chunk_gated_delta_rule_varlen`` needs (``gdn_chunk_varlen_workspace_bytes``)."""
    return int(_lib.load().gdn_chunk_varlen_workspace_bytes(T, num_seqs, H, Dk, Dv, _DTYPES.get(dtype, _lib.GDN_F32)))


def chunk_gated_delta_rule_varlen(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    cu_seqlens: torch.Tensor,
    initial_state: Optional[torch.Tensor] = None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    workspace: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Chunked rule over packed sequences: ``query [1, T, H, Dk]`` holds sequence n at tokens
    ``cu_seqlens[n] .. cu_seqlens[n+1]`` (``cu_seqlens`` int32 on the device, read there only).  Each
    sequence has its own chunks and state (``initial_state`` / ``final_state`` ``[N, H, Dk, Dv]`` fp32)
    and gets exactly the results of a separate ``fast_chunk_gated_delta_rule`` call.  bf16 q/k/v."""
    q = _as_kernel_tensor(query, "query", 4)
    k = _as_kernel_tensor(key, "key", 4)
    v = _as_kernel_tensor(value, "value", 4)
    gg = _as_kernel_tensor(g, "g", 3)
    bb = _as_kernel_tensor(beta, "beta", 3)
    if not isinstance(cu_seqlens, torch.Tensor) or cu_seqlens.device != q.device or cu_seqlens.dim() != 1:
        raise RuntimeError("cu_seqlens must be a 1-D tensor on the inputs' device")
    for name, x in (("key", k), ("value", v), ("g", gg), ("beta", bb)):
        if x.device != q.device:
            raise RuntimeError(f"{name} is on {x.device}, query on {q.device}")
    cu = cu_seqlens.to(torch.int32).contiguous()
    N = cu.numel() - 1
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    h0 = _state_in(initial_state, N, H, Dk, Dv, q.device)
    out = torch.empty((B, T, H, Dv), dtype=q.dtype, device=q.device)
    final = torch.empty((N, H, Dk, Dv), dtype=torch.float32, device=q.device) if output_final_state else None
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _raise_pending(lib, q.device)
        need = lib.gdn_chunk_varlen_workspace_bytes(T, max(N, 1), H, Dk, Dv, _DTYPES[q.dtype])
        workspace = _workspace(workspace, need, q.device)
        dq, dk, dv, dg, db, do = (_desc(x) for x in (q, k, v, gg, bb, out))
        rc = lib.gdn_chunk_gated_delta_rule_varlen(
            ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(dg), ctypes.byref(db),
            cu.data_ptr(), N, 64, h0.data_ptr() if h0 is not None else None, int(bool(output_final_state)),
            int(bool(use_qk_l2norm_in_kernel)), ctypes.byref(do), final.data_ptr() if final is not None else None,
            workspace.data_ptr(), workspace.numel(), torch.cuda.current_stream(q.device).cuda_stream)
        _lib.check(rc)
    if out.dtype != query.dtype:
        out = out.to(query.dtype)
    return out, final


def chunk_bwd_workspace_bytes(B: int, T: int, H: int, Dk: int = 128, Dv: int = 128,
                              dtype: torch.dtype = torch.bfloat16) -> int:
    """Device bytes ``chunk_gated_delta_rule_bwd`` needs (``gdn_chunk_bwd_workspace_bytes``)."""
    return int(_lib.load().gdn_chunk_bwd_workspace_bytes(B, T, H, Dk, Dv, _DTYPES.get(dtype, _lib.GDN_F32)))


def chunk_gated_delta_rule_bwd(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    d_out: torch.Tensor,
    initial_state: Optional[torch.Tensor] = None,
    d_final_state: Optional[torch.Tensor] = None,
    use_qk_l2norm_in_kernel: bool = False,
    chunk_size: int = 64,
    workspace: Optional[torch.Tensor] = None,
):
    """Gradients of ``fast_chunk_gated_delta_rule``: returns ``(dq, dk, dv, dg, dbeta, dh0)`` for outputs
    receiving ``d_out`` and the final state receiving ``d_final_state`` (None = not used), each gradient in
    its input's dtype (``dh0`` fp32, None without ``initial_state``).  The reference has no backward; these
    are the gradients autograd takes through its torch forward (qwen3_5_transformers.py:110-187)."""
    q = _as_kernel_tensor(query, "query", 4)
    k = _as_kernel_tensor(key, "key", 4)
    v = _as_kernel_tensor(value, "value", 4)
    gg = _as_kernel_tensor(g, "g", 3)
    bb = _as_kernel_tensor(beta, "beta", 3)
    do = _as_kernel_tensor(d_out, "d_out", 4)
    B, T, H, Dk = q.shape
    Dv = v.shape[-1]
    dev = q.device
    for name, x in (("key", k), ("value", v), ("g", gg), ("beta", bb), ("d_out", do)):
        if x.device != dev:
            raise RuntimeError(f"{name} is on {x.device}, query on {dev}")
    h0 = _state_in(initial_state, B, H, Dk, Dv, dev)
    dhT = _state_in(d_final_state, B, H, Dk, Dv, dev)
    dq = torch.empty(q.shape, dtype=q.dtype, device=dev)
    dk = torch.empty(k.shape, dtype=k.dtype, device=dev)
    dv = torch.empty(v.shape, dtype=v.dtype, device=dev)
    dg = torch.empty(gg.shape, dtype=gg.dtype, device=dev)
    db = torch.empty(bb.shape, dtype=bb.dtype, device=dev)
    dh0 = torch.empty((B, H, Dk, Dv), dtype=torch.float32, device=dev) if initial_state is not None else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        _raise_pending(lib, dev)
        need = lib.gdn_chunk_bwd_workspace_bytes(B, T, H, Dk, Dv, _DTYPES[q.dtype])
        workspace = _workspace(workspace, need, dev)
        descs = [_desc(x) for x in (q, k, v, gg, bb, do, dq, dk, dv, dg, db)]
        rc = lib.gdn_chunk_gated_delta_rule_bwd(
            *[ctypes.byref(d) for d in descs[:6]], int(chunk_size), h0.data_ptr() if h0 is not None else None,
            dhT.data_ptr() if dhT is not None else None, int(bool(use_qk_l2norm_in_kernel)),
            *[ctypes.byref(d) for d in descs[6:]], dh0.data_ptr() if dh0 is not None else None,
            workspace.data_ptr(), workspace.numel(), torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(rc)
    cast = lambda x, ref: x if x.dtype == ref.dtype else x.to(ref.dtype)  # noqa: E731
    return (cast(dq, query), cast(dk, key), cast(dv, value), cast(dg, g), cast(db, beta), dh0)


class _ChunkRule(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, initial_state, output_final_state, use_qk_l2norm_in_kernel):
        o, s = fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=initial_state,
                                           output_final_state=output_final_state,
                                           use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
        ctx.save_for_backward(q, k, v, g, beta, initial_state)
        ctx.l2 = use_qk_l2norm_in_kernel
        ctx.has_state = initial_state is not None
        return o, s

    @staticmethod
    def backward(ctx, d_out, d_state):
        q, k, v, g, beta, h0 = ctx.saved_tensors
        grads = chunk_gated_delta_rule_bwd(q, k, v, g, beta, d_out.contiguous(),
                                           initial_state=h0 if ctx.has_state else None,
                                           d_final_state=d_state, use_qk_l2norm_in_kernel=ctx.l2)
        dh0 = grads[5]
        if ctx.has_state and dh0 is not None and dh0.dtype != h0.dtype:
            dh0 = dh0.to(h0.dtype)
        return grads[0], grads[1], grads[2], grads[3], grads[4], dh0, None, None


def chunk_gated_delta_rule(query, key, value, g, beta, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False):
    """Differentiable form of ``fast_chunk_gated_delta_rule`` (same arguments and outputs): its backward runs
    ``chunk_gated_delta_rule_bwd``.  For training; the drop-in itself, like the reference's, has no backward."""
    return _ChunkRule.apply(query, key, value, g, beta, initial_state, output_final_state, use_qk_l2norm_in_kernel)
