"""The C-ABI library loads, exports every symbol include/*.h declares, and
rejects bad arguments with the reference's error behaviour -- all without a GPU
(validation runs before any CUDA call)."""
import ctypes
import glob
import os
import re

import pytest

from llms_from_scratch_b200 import _lib
from llms_from_scratch_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names.update(re.findall(r"GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = _declared_symbols()
    assert {"gdn_chunk_gated_delta_rule", "gdn_recurrent_gated_delta_rule", "gdn_chunk_workspace_bytes"} <= names


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(_declared_symbols()):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    # and the Python binding types every one of them
    assert _declared_symbols() <= set(_lib.SIGNATURES)


def test_abi_version_and_status_names(lib):
    assert lib.gdn_abi_version() == 1
    assert lib.gdn_status_name(0) == b"GDN_OK"
    assert lib.gdn_status_name(1) == b"GDN_ERR_INVALID_ARGUMENT"
    assert lib.gdn_status_name(99) == b"GDN_UNKNOWN_STATUS"


def test_workspace_size(lib):
    assert lib.gdn_chunk_workspace_bytes(0, 10, 1, 128, 128, 1) == 0
    a = lib.gdn_chunk_workspace_bytes(1, 64, 1, 128, 128, 1)
    assert a > 0 and a % 256 == 0
    assert lib.gdn_chunk_workspace_bytes(1, 65, 1, 128, 128, 1) == 2 * a
    assert lib.gdn_chunk_workspace_bytes(3, 4096, 16, 128, 128, 1) == 3 * 16 * 64 * a


def _t(shape, dtype=_lib.GDN_BF16, data=0x1000):
    d = _lib.GdnTensor()
    d.data = data
    d.dtype = dtype
    d.ndim = len(shape)
    st = 1
    strides = []
    for s in reversed(shape):
        strides.append(st)
        st *= s
    strides = list(reversed(strides))
    for i in range(4):
        d.shape[i] = shape[i] if i < len(shape) else 1
        d.stride[i] = strides[i] if i < len(shape) else 1
    return d


def _call_chunk(lib, q, k, v, g, b, out, chunk=64, ws=0x100000, ws_bytes=1 << 40):
    return lib.gdn_chunk_gated_delta_rule(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(g),
                                          ctypes.byref(b), chunk, None, 0, 1, ctypes.byref(out), None, ws,
                                          ws_bytes, None)


@pytest.mark.parametrize("case,needle", [
    ("chunk", "chunk_size must be 64"),
    ("dk", "key head dim must be 128"),
    ("dv", "value head dim must be 128"),
    ("gshape", "g has shape"),
    ("stride", "head dimension must be contiguous"),
    ("dtype", "unsupported dtype"),
])
def test_invalid_arguments_are_rejected_before_any_cuda_call(lib, case, needle):
    B, T, H = 1, 70, 2
    q, k, v = _t([B, T, H, 128]), _t([B, T, H, 128]), _t([B, T, H, 128])
    g, b = _t([B, T, H], _lib.GDN_F32), _t([B, T, H], _lib.GDN_F32)
    out = _t([B, T, H, 128])
    chunk = 64
    if case == "chunk":
        chunk = 32
    elif case == "dk":
        q, k = _t([B, T, H, 64]), _t([B, T, H, 64])
    elif case == "dv":
        v, out = _t([B, T, H, 64]), _t([B, T, H, 64])
    elif case == "gshape":
        g = _t([B, T + 1, H], _lib.GDN_F32)
    elif case == "stride":
        k.stride[3] = 2
    elif case == "dtype":
        v.dtype = 7
    rc = _call_chunk(lib, q, k, v, g, b, out, chunk=chunk)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT
    assert needle in lib.gdn_last_error().decode()
    with pytest.raises(_lib.GDNError, match="GDN_ERR_INVALID_ARGUMENT"):
        _lib.check(rc)


def _call_host(lib, q, k, v, g, b, out, slice_tokens=0, ws=0x100000, ws_bytes=1 << 40):
    return lib.gdn_chunk_gated_delta_rule_host(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(g),
                                               ctypes.byref(b), 64, None, 0, 1, ctypes.byref(out), None,
                                               slice_tokens, ws, ws_bytes, None)


@pytest.mark.parametrize("case,status,needle", [
    ("slice", _lib.GDN_ERR_INVALID_ARGUMENT, "slice_tokens"),
    ("dv", _lib.GDN_ERR_INVALID_ARGUMENT, "head dim must be 128"),
    ("gshape", _lib.GDN_ERR_INVALID_ARGUMENT, "differs from query"),
    ("unpacked", _lib.GDN_ERR_UNSUPPORTED, "packed [B][T][H][D]"),
    ("unpacked_g", _lib.GDN_ERR_UNSUPPORTED, "packed [B][T][H]"),
    ("workspace", _lib.GDN_ERR_WORKSPACE, "workspace of"),
])
def test_host_entry_rejects_bad_arguments_before_any_cuda_call(lib, case, status, needle):
    B, T, H = 2, 300, 2
    q, k, v, out = (_t([B, T, H, 128]) for _ in range(4))
    g, b = _t([B, T, H], _lib.GDN_F32), _t([B, T, H], _lib.GDN_F32)
    kw = {}
    if case == "slice":
        kw["slice_tokens"] = 100
    elif case == "dv":
        out = _t([B, T, H, 64])
    elif case == "gshape":
        b = _t([B, T, H + 1], _lib.GDN_F32)
    elif case == "unpacked":
        v.stride[1] = 2 * H * 128  # every other token of a wider buffer
    elif case == "unpacked_g":
        g.stride[2] = 2
    elif case == "workspace":
        kw["ws_bytes"] = 1024
    rc = _call_host(lib, q, k, v, g, b, out, **kw)
    assert rc == status
    assert needle in lib.gdn_last_error().decode()


def test_host_workspace_size(lib):
    f = lib.gdn_chunk_host_workspace_bytes
    assert f(1, 4096, 16, 128, 128, _lib.GDN_BF16, 100) == 0  # slice not a multiple of 64
    assert f(0, 4096, 16, 128, 128, _lib.GDN_BF16, 0) == 0
    a = f(1, 4096, 16, 128, 128, _lib.GDN_BF16, 0)
    b = f(1, 4096, 16, 128, 128, _lib.GDN_BF16, 1024)
    assert a == b > 0 and a % 256 == 0  # the default largest slice at B=1, H=16 is 1024 tokens (12 MiB of q/k/v)
    # one slice's chunk workspace + the state + g/beta of the whole sequence + two q/k/v and two out slices
    ws = lib.gdn_chunk_workspace_bytes(1, 1024, 16, 128, 128, _lib.GDN_BF16)
    rows = 1024 * 16
    assert a == ws + 16 * 128 * 128 * 4 + 2 * 4096 * 16 * 4 + 2 * 3 * rows * 256 + 2 * rows * 256
    # short sequences stage one slice rounded up to the chunk
    assert f(1, 100, 1, 128, 128, _lib.GDN_BF16, 0) == f(1, 128, 1, 128, 128, _lib.GDN_BF16, 0)


def _call_varlen(lib, q, k, v, g, b, out, cu=0x2000, num_seqs=2, chunk=64):
    return lib.gdn_chunk_gated_delta_rule_varlen(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(g),
                                                 ctypes.byref(b), cu, num_seqs, chunk, None, 0, 1,
                                                 ctypes.byref(out), None, 0x100000, 1 << 40, None)


@pytest.mark.parametrize("case,status,needle", [
    ("batch", _lib.GDN_ERR_INVALID_ARGUMENT, "B == 1"),
    ("num_seqs", _lib.GDN_ERR_INVALID_ARGUMENT, "num_seqs"),
    ("null", _lib.GDN_ERR_INVALID_ARGUMENT, "cu_seqlens is NULL"),
    ("chunk", _lib.GDN_ERR_INVALID_ARGUMENT, "chunk_size must be 64"),
    ("fp32", _lib.GDN_ERR_UNSUPPORTED, "bf16"),
])
def test_varlen_entry_rejects_bad_arguments_before_any_cuda_call(lib, case, status, needle):
    B, T, H = (2 if case == "batch" else 1), 300, 2
    dt = _lib.GDN_F32 if case == "fp32" else _lib.GDN_BF16
    q, k, v, out = (_t([B, T, H, 128], dt) for _ in range(4))
    g, b = _t([B, T, H], _lib.GDN_F32), _t([B, T, H], _lib.GDN_F32)
    kw = {}
    if case == "num_seqs":
        kw["num_seqs"] = 0
    elif case == "null":
        kw["cu"] = None
    elif case == "chunk":
        kw["chunk"] = 32
    rc = _call_varlen(lib, q, k, v, g, b, out, **kw)
    assert rc == status
    assert needle in lib.gdn_last_error().decode()


def test_varlen_workspace_size(lib):
    f = lib.gdn_chunk_varlen_workspace_bytes
    rec = 147456  # one tensor-core chunk record: M (32 KB) + Q' (16 KB) + b (64 KB) + o0 (32 KB)
    # tables (N + 1 bases, one sequence id per chunk, N sequence ranks) rounded to 256 B, then ceil(T/64) + N
    # records per head
    assert f(1000, 3, 4, 128, 128, _lib.GDN_BF16) == 256 + (16 + 3) * 4 * rec
    assert f(64, 1, 1, 128, 128, _lib.GDN_BF16) == 256 + 2 * rec
    big = f(100000, 500, 16, 128, 128, _lib.GDN_BF16)
    header = (4 * (501 + 1563 + 500 + 500) + 255) // 256 * 256
    assert big == header + (1563 + 500) * 16 * rec


@pytest.mark.parametrize("case,needle", [
    ("chunk", "chunk_size must be 64"),
    ("dq", "dq must be 4-D"),
    ("dg", "dg has shape"),
    ("dout", "out has shape"),
])
def test_bwd_entry_rejects_bad_arguments_before_any_cuda_call(lib, case, needle):
    B, T, H = 1, 70, 2
    q, k, v, do = (_t([B, T, H, 128]) for _ in range(4))
    dq, dk, dv = (_t([B, T, H, 128]) for _ in range(3))
    g, b, dg, db = (_t([B, T, H], _lib.GDN_F32) for _ in range(4))
    chunk = 64
    if case == "chunk":
        chunk = 16
    elif case == "dq":
        dq = _t([B, T, H])
    elif case == "dg":
        dg = _t([B, T + 1, H], _lib.GDN_F32)
    elif case == "dout":
        do = _t([B, T - 1, H, 128])
    rc = lib.gdn_chunk_gated_delta_rule_bwd(*(ctypes.byref(x) for x in (q, k, v, g, b, do)), chunk, None, None, 1,
                                            *(ctypes.byref(x) for x in (dq, dk, dv, dg, db)), None, 0x100000,
                                            1 << 40, None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT
    assert needle in lib.gdn_last_error().decode()


def test_bwd_workspace_size(lib):
    f = lib.gdn_chunk_bwd_workspace_bytes
    assert f(1, 0, 4, 128, 128, _lib.GDN_BF16) == 0
    # per (b, h, chunk): CUDA-core forward tiles (36,928 floats) + backward record (90,304 floats) + the
    # tensor-core forward record (147,456 bytes)
    per = (36928 + 90304) * 4 + 147456
    assert f(1, 64, 1, 128, 128, _lib.GDN_BF16) == per
    assert f(2, 4096, 16, 128, 128, _lib.GDN_F32) == 2 * 16 * 64 * per


def test_final_state_pointer_required(lib):
    B, T, H = 1, 8, 1
    q, k, v, out = (_t([B, T, H, 128]) for _ in range(4))
    g, b = _t([B, T, H], _lib.GDN_F32), _t([B, T, H], _lib.GDN_F32)
    rc = lib.gdn_recurrent_gated_delta_rule(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(g),
                                            ctypes.byref(b), None, 1, 1, ctypes.byref(out), None, None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT
    assert "final_state" in lib.gdn_last_error().decode()


def test_python_op_refuses_cpu_tensors_and_torch_backend():
    import torch

    from llms_from_scratch_b200 import fast_chunk_gated_delta_rule, fast_recurrent_gated_delta_rule
    q = torch.zeros(1, 4, 1, 128)
    g = torch.zeros(1, 4, 1)
    if not torch.cuda.is_available():  # CPU tensors go to the GPU through the host-buffer path
        with pytest.raises(RuntimeError, match="no CPU path"):
            fast_chunk_gated_delta_rule(q, q, q, g, g)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        fast_recurrent_gated_delta_rule(q, q, q, g, g, None, False)
    with pytest.raises(RuntimeError, match="pure-PyTorch"):
        fast_chunk_gated_delta_rule(q, q, q, g, g, backend="torch")
    with pytest.raises(RuntimeError, match="not available"):
        fast_chunk_gated_delta_rule(q, q, q, g, g, backend="nope")


def test_workspace_on_the_host_or_another_device_is_rejected():
    """A caller's workspace is handed to the kernels as a raw pointer, so it must be a CUDA buffer on the
    inputs' device; anything else raises instead of letting the kernels write through a foreign pointer."""
    import torch

    from llms_from_scratch_b200.ops import _workspace
    dev0 = torch.device("cuda", 0)
    with pytest.raises(RuntimeError, match="workspace is on cpu"):
        _workspace(torch.empty(1 << 10, dtype=torch.uint8), 16, dev0)
    with pytest.raises(RuntimeError, match="workspace is on"):
        _workspace(bytearray(64), 16, dev0)
    if torch.cuda.device_count() >= 2:
        with pytest.raises(RuntimeError, match="cuda:1"):
            _workspace(torch.empty(64, dtype=torch.uint8, device="cuda:1"), 16, dev0)


def test_torch_operator_library_registers_the_ops(lib):
    """torch.ops.gdn.chunk_fwd / decode_step (the drop-in's native entry) load and keep the reference's
    argument names; with CPU tensors they raise (there is no CPU path)."""
    import torch

    from llms_from_scratch_b200.build import build_torch_ops
    from llms_from_scratch_b200.ops import _torch_ops
    build_torch_ops()
    assert _torch_ops()
    schema = str(torch.ops.gdn.chunk_fwd.default._schema)
    for arg in ("Tensor query", "Tensor key", "Tensor value", "Tensor g", "Tensor beta", "int chunk_size=64",
                "Tensor? initial_state=None", "bool output_final_state=False", "bool use_qk_l2norm_in_kernel=False"):
        assert arg in schema, (arg, schema)
    assert "Tensor(a!)? out_state" in str(torch.ops.gdn.decode_step.default._schema)
    q, g = torch.zeros(1, 4, 1, 128), torch.zeros(1, 4, 1)
    with pytest.raises(RuntimeError, match="no CPU path"):
        torch.ops.gdn.chunk_fwd(q, q, q, g, g)
    with pytest.raises(RuntimeError, match="no CPU path"):
        torch.ops.gdn.decode_step(q, q, q, g, g, None, False)


def test_status_names_cover_every_status(lib):
    names = [lib.gdn_status_name(i).decode() for i in range(7)]
    assert names[6] == "GDN_ERR_KERNEL" and "GDN_UNKNOWN_STATUS" not in names


def test_compat_module_exports_reference_names():
    import importlib
    import sys
    sys.path.insert(0, os.path.join(ROOT, "llms_from_scratch_b200", "compat"))
    try:
        m = importlib.import_module("qwen3_5_cutedsl_kernels")
        for name in ("fast_chunk_gated_delta_rule", "get_backend", "_TRITON_OK", "_CUTE_OK", "l2norm"):
            assert hasattr(m, name)
        assert m.get_backend() in ("cuda",)
    finally:
        sys.path.pop(0)
