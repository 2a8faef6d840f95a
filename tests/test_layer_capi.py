"""The layer entry points of the C ABI reject bad arguments before any CUDA call
(so these run without a GPU), with the reference's error behaviour mapped to
gdn_status codes."""
import ctypes

import pytest

from llms_from_scratch_b200 import _lib
from llms_from_scratch_b200.build import build


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def _t(shape, dtype=_lib.GDN_BF16, data=0x1000, strides=None):
    d = _lib.GdnTensor()
    d.data = data
    d.dtype = dtype
    d.ndim = len(shape)
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= s
    st = list(reversed(st)) if strides is None else strides
    for i in range(4):
        d.shape[i] = shape[i] if i < len(shape) else 1
        d.stride[i] = st[i] if i < len(shape) else 1
    return d


def _r(x):
    return ctypes.byref(x) if x is not None else None


@pytest.mark.parametrize("case,status,needle", [
    ("wshape", _lib.GDN_ERR_INVALID_ARGUMENT, "weight: dim 1"),
    ("oshape", _lib.GDN_ERR_INVALID_ARGUMENT, "out: dim 1"),
    ("alias", _lib.GDN_ERR_INVALID_ARGUMENT, "must not alias"),
    ("unaligned", _lib.GDN_ERR_UNSUPPORTED, "16-byte aligned"),
    ("dtype", _lib.GDN_ERR_UNSUPPORTED, "share one dtype"),
    ("strided", _lib.GDN_ERR_INVALID_ARGUMENT, "last dimension must be contiguous"),
])
def test_conv_rejects_bad_arguments(lib, case, status, needle):
    B, T, C = 2, 10, 64
    x, w, out = _t([B, T, C]), _t([C, 4], data=0x2000), _t([B, T, C], data=0x8000)
    if case == "wshape":
        w = _t([C, 3])
    elif case == "oshape":
        out = _t([B, T + 1, C], data=0x8000)
    elif case == "alias":
        out = _t([B, T, C])
    elif case == "unaligned":
        x = _t([B, T, C], data=0x1008)
    elif case == "dtype":
        w = _t([C, 4], dtype=_lib.GDN_F32, data=0x2000)
    elif case == "strided":
        x = _t([B, T, C], strides=[T * C * 2, C * 2, 2])
    rc = lib.gdn_causal_conv1d_silu(_r(x), _r(w), _r(out), None, None)
    assert rc == status
    assert needle in lib.gdn_last_error().decode()


def test_conv_update_requires_the_state(lib):
    B, C = 3, 32
    x, w, out = _t([B, 1, C]), _t([C, 4], data=0x2000), _t([B, 1, C], data=0x8000)
    rc = lib.gdn_causal_conv1d_update(_r(x), None, _r(w), _r(out), None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT
    assert "conv_state is NULL" in lib.gdn_last_error().decode()
    s = _t([B, C, 3], data=0x4000)
    rc = lib.gdn_causal_conv1d_update(_r(x), _r(s), _r(w), _r(out), None)
    assert rc == _lib.GDN_ERR_INVALID_ARGUMENT


def test_gates_and_norm_reject_bad_shapes(lib):
    a, b = _t([1, 4, 16]), _t([1, 4, 16], data=0x2000)
    A, dt = _t([16], data=0x3000), _t([15], data=0x3100)
    g, beta = _t([1, 4, 16], _lib.GDN_F32, 0x4000), _t([1, 4, 16], data=0x5000)
    assert lib.gdn_gates(_r(a), _r(b), _r(A), _r(dt), _r(g), _r(beta), None) == _lib.GDN_ERR_INVALID_ARGUMENT
    assert "dt_bias" in lib.gdn_last_error().decode()
    x, z, w, o = _t([8, 64]), _t([8, 64], data=0x2000), _t([64], data=0x3000), _t([8, 64], data=0x4000)
    assert lib.gdn_rms_norm_gated(_r(x), _r(z), _r(w), 1e-6, _r(o), None) == _lib.GDN_ERR_INVALID_ARGUMENT
    assert "expected 128" in lib.gdn_last_error().decode()
    x, z, w, o = _t([8, 128]), _t([8, 128], data=0x2000), _t([128], data=0x3000), _t([8, 128], data=0x4000)
    assert lib.gdn_rms_norm_gated(_r(x), _r(z), _r(w), -1.0, _r(o), None) == _lib.GDN_ERR_INVALID_ARGUMENT


def test_python_layer_ops_refuse_cpu_tensors():
    import torch

    from llms_from_scratch_b200 import layer
    x = torch.zeros(1, 4, 64, dtype=torch.bfloat16)
    w = torch.zeros(64, 4, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer.causal_conv1d_silu(x, w)
    with pytest.raises(RuntimeError, match="bias must be None"):
        layer.causal_conv1d_fn(x.transpose(1, 2), w, bias=w[:, 0], activation="silu")
