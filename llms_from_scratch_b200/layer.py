"""GatedDeltaNet layer steps around the gated delta rule, on the sm_100a library.

Drop-ins for the hooks ``Qwen3_5GatedDeltaNet`` calls on either side of the rule
(qwen3_5_transformers.py:304-419):

* ``causal_conv1d_fn(x, weight, bias=None, activation=None, seq_idx=None)`` —
  the prefill convolution the layer takes from the causal-conv1d package when it
  is installed (:349-355) and otherwise computes as
  ``F.silu(self.conv1d(mixed_qkv)[:, :, :seq_len])`` (:356).  ``x`` is
  ``[B, C, T]`` as the layer passes it.
* ``causal_conv1d_update(hidden_states, conv_state, weight, bias=None,
  activation=None)`` — ``torch_causal_conv1d_update`` (:85-101).
* ``gates(a, b, A_log, dt_bias)`` — ``beta = b.sigmoid()`` and
  ``g = -A_log.float().exp() * softplus(a.float() + dt_bias)`` (:377-379).
* ``rms_norm_gated(x, gate, weight, eps)`` / ``RMSNormGated`` —
  ``Qwen3_5RMSNormGated`` (:56-71).
* ``causal_conv1d_silu(mixed_qkv, weight, conv_state=None)`` — the native,
  token-major form of the prefill convolution: takes the ``in_proj_qkv`` output
  ``[B, T, C]`` and returns ``[B, T, C]`` whose channel ranges are q, k, v as
  strided views, with no transposes.

All run asynchronously on the current CUDA stream and raise ``RuntimeError``
(``GDNError``) on bad arguments; there is no CPU path.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from .ops import _DTYPES, _desc

_SILU = (None, "silu", "swish")


def _cuda(x: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if x.device.type != "cuda":
        raise RuntimeError(f"{name} is on {x.device}; the GatedDeltaNet kernels need CUDA tensors (no CPU path)")
    if x.dtype not in _DTYPES:
        raise RuntimeError(f"{name} has unsupported dtype {x.dtype}")
    return x if x.stride(-1) == 1 else x.contiguous()


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def causal_conv1d_silu(mixed_qkv: torch.Tensor, weight: torch.Tensor,
                       conv_state: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SiLU(depthwise causal conv1d, kernel 4) over ``mixed_qkv [B, T, C]``; writes the last four raw
    inputs of each sequence into ``conv_state [B, C, 4]`` when given (the cache, :346-348)."""
    x = _cuda(mixed_qkv, "mixed_qkv")
    w = _cuda(weight, "weight")
    if x.dim() != 3:
        raise RuntimeError(f"mixed_qkv must be [B, T, C], got shape {tuple(x.shape)}")
    if w.dim() == 3:  # conv1d.weight [C, 1, K]
        w = w.squeeze(1)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        dx, dw, do = _desc(x), _desc(w), _desc(out)
        ds = _desc(conv_state) if conv_state is not None else None
        rc = lib.gdn_causal_conv1d_silu(ctypes.byref(dx), ctypes.byref(dw), ctypes.byref(do),
                                        ctypes.byref(ds) if ds is not None else None, _stream(x.device))
        _lib.check(rc)
    return out


def causal_conv1d_fn(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                     activation: Optional[str] = None, seq_idx=None) -> torch.Tensor:
    """The causal-conv1d hook of the layer (:349-355): ``x [B, C, T]`` -> ``[B, C, T]``."""
    if bias is not None:
        raise RuntimeError("the Qwen3.5 conv has no bias (qwen3_5_transformers.py:256); bias must be None")
    if activation not in ("silu", "swish"):
        raise RuntimeError(f"activation {activation!r} is not supported; the layer uses 'silu'")
    if seq_idx is not None:
        raise RuntimeError("seq_idx (packed varlen sequences) is not supported")
    return causal_conv1d_silu(x.transpose(1, 2), weight).transpose(1, 2)


def causal_conv1d_update(hidden_states: torch.Tensor, conv_state: torch.Tensor, weight: torch.Tensor,
                         bias: Optional[torch.Tensor] = None, activation: Optional[str] = None) -> torch.Tensor:
    """``torch_causal_conv1d_update`` (:85-101): ``hidden_states [B, C, T]``, ``conv_state [B, C, 4]``
    updated in place; returns ``[B, C, T]``."""
    if bias is not None:
        raise RuntimeError("bias must be None (the Qwen3.5 conv has none)")
    if activation not in _SILU:
        raise RuntimeError(f"activation {activation!r} is not supported; the layer uses 'silu'")
    x = _cuda(hidden_states.transpose(1, 2), "hidden_states")
    w = _cuda(weight, "weight")
    if not isinstance(conv_state, torch.Tensor) or conv_state.device != x.device:
        raise RuntimeError("conv_state must be a CUDA tensor [B, C, 4] on the input's device")
    # The layer's prefill keeps F.pad(mixed_qkv, ...) as the state (:346-348), which can be a strided view; the
    # kernel updates a contiguous state, so such a view is updated through a copy (still in place for the caller).
    state = conv_state if conv_state.stride(-1) == 1 else conv_state.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        dx, ds, dw, do = _desc(x), _desc(state), _desc(w), _desc(out)
        rc = lib.gdn_causal_conv1d_update(ctypes.byref(dx), ctypes.byref(ds), ctypes.byref(dw), ctypes.byref(do),
                                          _stream(x.device))
        _lib.check(rc)
    if state is not conv_state:
        conv_state.copy_(state)
    return out.transpose(1, 2)


def gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor,
          dt_bias: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(g fp32, beta in b.dtype)`` from ``a, b [B, T, H]`` and ``A_log, dt_bias [H]`` (:377-379)."""
    ta, tb = _cuda(a, "a"), _cuda(b, "b")
    A, dt = _cuda(A_log, "A_log"), _cuda(dt_bias, "dt_bias")
    if dt.dtype != A.dtype:
        dt = dt.to(A.dtype)
    g = torch.empty(ta.shape, dtype=torch.float32, device=ta.device)
    beta = torch.empty(tb.shape, dtype=tb.dtype, device=tb.device)
    lib = _lib.load()
    with torch.cuda.device(ta.device):
        d = [_desc(x) for x in (ta, tb, A, dt, g, beta)]
        rc = lib.gdn_gates(*(ctypes.byref(x) for x in d), _stream(ta.device))
        _lib.check(rc)
    return g, beta


def rms_norm_gated(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``Qwen3_5RMSNormGated.forward(x, gate)`` (:62-71) over the last dim (128) of ``x``."""
    tx, tg, tw = _cuda(x, "x"), _cuda(gate, "gate"), _cuda(weight, "weight")
    shape = tx.shape
    x2 = tx.reshape(-1, shape[-1])
    g2 = tg.reshape(-1, tg.shape[-1])
    out = torch.empty(x2.shape, dtype=tx.dtype, device=tx.device)
    lib = _lib.load()
    with torch.cuda.device(tx.device):
        d = [_desc(t) for t in (x2, g2, tw)]
        do = _desc(out)
        rc = lib.gdn_rms_norm_gated(ctypes.byref(d[0]), ctypes.byref(d[1]), ctypes.byref(d[2]), float(eps),
                                    ctypes.byref(do), _stream(tx.device))
        _lib.check(rc)
    return out.reshape(shape)


class RMSNormGated(torch.nn.Module):
    """Module form of ``Qwen3_5RMSNormGated`` (:56-71): ``forward(hidden_states, gate)``."""

    def __init__(self, hidden_size: int, eps: float = 1e-6, **kwargs):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        return rms_norm_gated(hidden_states, gate, self.weight.to(hidden_states.dtype), self.variance_epsilon)
