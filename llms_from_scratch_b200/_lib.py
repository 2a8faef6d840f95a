"""ctypes binding of ``libgdn_b200.so`` (the C ABI declared in include/gdn_b200.h).

The library is built in-tree by ``python -m llms_from_scratch_b200.build``.
Loading fails loudly when it is missing: there is no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn_b200.so")

GDN_OK = 0
GDN_ERR_INVALID_ARGUMENT = 1
GDN_ERR_UNSUPPORTED = 2
GDN_ERR_WORKSPACE = 3
GDN_ERR_CUDA = 4
GDN_ERR_DEVICE = 5
GDN_ERR_KERNEL = 6

GDN_F32, GDN_BF16, GDN_F16 = 0, 1, 2
GDN_NOALLOC_SCRATCH_BYTES = 64 << 20  # include/gdn_b200.h

# Every symbol include/gdn_b200.h declares, with its ctypes signature.
c_void_p, c_int, c_int64, c_size_t, c_char_p = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                                 ctypes.c_size_t, ctypes.c_char_p)


class GdnTensor(ctypes.Structure):
    _fields_ = [
        ("data", c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", c_int64 * 4),
        ("stride", c_int64 * 4),
    ]


_P = ctypes.POINTER(GdnTensor)

SIGNATURES = {
    "gdn_chunk_gated_delta_rule": (c_int, [_P, _P, _P, _P, _P, c_int, c_void_p, c_int, c_int, _P, c_void_p,
                                           c_void_p, c_size_t, c_void_p]),
    "gdn_chunk_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int]),
    "gdn_chunk_gated_delta_rule_noalloc": (c_int, [_P, _P, _P, _P, _P, c_int, c_void_p, c_int, c_int, _P,
                                                   c_void_p, c_void_p]),
    "gdn_chunk_gated_delta_rule_host": (c_int, [_P, _P, _P, _P, _P, c_int, c_void_p, c_int, c_int, _P, c_void_p,
                                                c_int64, c_void_p, c_size_t, c_void_p]),
    "gdn_chunk_host_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int64]),
    "gdn_chunk_gated_delta_rule_varlen": (c_int, [_P, _P, _P, _P, _P, c_void_p, c_int64, c_int, c_void_p, c_int, c_int,
                                                  _P, c_void_p, c_void_p, c_size_t, c_void_p]),
    "gdn_chunk_varlen_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int]),
    "gdn_chunk_gated_delta_rule_bwd": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_void_p, c_void_p, c_int, _P, _P, _P,
                                               _P, _P, c_void_p, c_void_p, c_size_t, c_void_p]),
    "gdn_chunk_bwd_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int]),
    "gdn_causal_conv1d_silu": (c_int, [_P, _P, _P, _P, c_void_p]),
    "gdn_causal_conv1d_update": (c_int, [_P, _P, _P, _P, c_void_p]),
    "gdn_gates": (c_int, [_P, _P, _P, _P, _P, _P, c_void_p]),
    "gdn_rms_norm_gated": (c_int, [_P, _P, _P, ctypes.c_float, _P, c_void_p]),
    "gdn_recurrent_gated_delta_rule": (c_int, [_P, _P, _P, _P, _P, c_void_p, c_int, c_int, _P, c_void_p, c_void_p]),
    "gdn_chunk_sp_summary": (c_int, [_P, _P, _P, _P, _P, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t,
                                     c_void_p]),
    "gdn_chunk_sp_finish": (c_int, [_P, _P, _P, _P, _P, c_int, c_void_p, c_int, c_int, _P, c_void_p, c_void_p,
                                    c_size_t, c_void_p]),
    "gdn_model_add_rms_norm": (c_int, [_P, _P, _P, ctypes.c_float, _P, _P, c_void_p]),
    "gdn_model_attn_prep": (c_int, [_P, _P, _P, c_void_p, c_void_p, c_int, c_void_p, ctypes.c_float, _P, _P, _P,
                                    c_void_p]),
    "gdn_model_attention": (c_int, [_P, _P, _P, _P, c_void_p, _P, c_void_p]),
    "gdn_model_silu_mul": (c_int, [_P, _P, c_void_p]),
    "gdn_model_add_rms_norm_partials": (c_int, [c_void_p, c_int, c_int64, c_int64, _P, _P, ctypes.c_float, _P, _P,
                                                c_void_p]),
    "gdn_model_linear": (c_int, [_P, _P, _P, c_void_p, c_int, c_int, c_void_p]),
    "gdn_model_gdn_decode": (c_int, [_P, _P, _P, _P, _P, c_void_p, _P, ctypes.c_float, _P, c_int, c_void_p]),
    "gdn_model_set_programmatic_launch": (None, [c_int]),
    "gdn_launch_count": (ctypes.c_uint64, []),
    "gdn_set_phase_events": (None, [ctypes.POINTER(c_void_p), c_int]),
    "gdn_device_error": (ctypes.c_uint, [c_int]),
    "gdn_device_error_pending": (ctypes.c_uint, []),
    "gdn_selftest_bounded_wait": (c_int, [ctypes.c_uint64, c_void_p]),
    "gdn_last_error": (c_char_p, []),
    "gdn_status_name": (c_char_p, [c_int]),
    "gdn_abi_version": (c_int, []),
}

_lock = threading.Lock()
_lib = None


class GDNError(RuntimeError):
    """A failed call into the CUDA library; ``status`` is the gdn_status code."""

    def __init__(self, status: int, name: str, message: str):
        super().__init__(f"{name}: {message}")
        self.status = status


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the CUDA library with typed signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build it with `python -m llms_from_scratch_b200.build` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != GDN_OK:
        lib = load()
        raise GDNError(status, lib.gdn_status_name(status).decode(), lib.gdn_last_error().decode())
