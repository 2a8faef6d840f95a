"""CPU oracle for the GatedDeltaNet layer steps on either side of the gated delta rule.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the layer
kernels of ``llms_from_scratch_b200`` (``gdn_layer.cu``); only ``tests/``,
``__graft_entry__.smoke`` and ``bench.py``'s CPU legs may import it.  The product
path never calls it.

It restates, in numpy, the steps of ``Qwen3_5GatedDeltaNet.forward`` around the
chunked / recurrent rule (reference: qwen3_5_transformers.py):

* ``causal_conv1d_silu``   the prefill convolution: the depthwise ``nn.Conv1d``
  of :253-260 (kernel 4, ``padding=3``, no bias) followed by
  ``F.silu(conv(x)[:, :, :seq_len])`` (:356), plus the conv state the cache keeps,
  ``F.pad(mixed_qkv, (K - seq_len, 0))`` (:346-348);
* ``causal_conv1d_update`` ``torch_causal_conv1d_update`` (:85-101), the decode
  convolution against the cached state;
* ``gates``                ``beta = b.sigmoid()`` and
  ``g = -A_log.float().exp() * softplus(a.float() + dt_bias)`` (:377-379);
* ``rms_norm_gated``       ``Qwen3_5RMSNormGated.forward`` (:62-71).

Layouts: ``mixed_qkv`` token-major ``[B, T, C]`` (the ``in_proj_qkv`` output,
before the reference transposes it to ``[B, C, T]`` at :334); conv weight
``[C, K]`` (``conv1d.weight.squeeze(1)``); conv state ``[B, C, K]`` (the
reference's cache layout); a, b ``[B, T, H]``; A_log, dt_bias ``[H]``; the
norm's rows ``[N, D]``.

The layer runs in bf16 (the model casts itself to ``config.dtype``, :301-302).
For bf16 inputs every torch op rounds its result to bf16 once, computing in
fp32 inside: the conv output, the SiLU, the sigmoid, ``weight * x`` in the norm
and the final gated product are rounded, exactly as below.  The summation order
inside torch's conv and mean is not reproduced bit for bit; the fixtures made
by ``tests/golden/make_golden_layer.py`` from the reference's own torch code pin
how close the restatement is.
"""

from __future__ import annotations

import numpy as np

from .gdn_oracle import round_bf16, round_to

__all__ = ["causal_conv1d_silu", "causal_conv1d_update", "gates", "rms_norm_gated", "softplus"]


def _silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def causal_conv1d_silu(x, weight, in_dtype: str = "bf16"):
    """Prefill: ``y[b,t,c] = silu(sum_j w[c,j] x[b,t-3+j,c])`` with x = 0 before t = 0.

    Returns ``(y [B,T,C], conv_state [B,C,K])``; the state is the last K raw inputs,
    left-padded with zeros when T < K (:346-348).
    """
    x = np.asarray(x, np.float32)
    w = np.asarray(weight, np.float32)
    B, T, C = x.shape
    K = w.shape[1]
    xp = np.concatenate([np.zeros((B, K - 1, C), np.float32), x], axis=1)  # padding=K-1 on the left (:259)
    acc = np.zeros((B, T, C), np.float64)
    for j in range(K):
        acc += w[None, None, :, j].astype(np.float64) * xp[:, j:j + T, :].astype(np.float64)
    y = round_to(acc.astype(np.float32), in_dtype)          # conv output in the layer dtype
    y = round_to(_silu(y), in_dtype)                         # F.silu on that dtype (:356)
    if T >= K:
        state = x[:, T - K:, :]
    else:
        state = np.concatenate([np.zeros((B, K - T, C), np.float32), x], axis=1)
    return y, np.ascontiguousarray(state.transpose(0, 2, 1))


def causal_conv1d_update(x, conv_state, weight, in_dtype: str = "bf16"):
    """Decode: ``torch_causal_conv1d_update`` (:85-101).  x ``[B,T,C]`` (T new tokens),
    conv_state ``[B,C,K]``.  Returns ``(y [B,T,C], new_state [B,C,K])``."""
    x = np.asarray(x, np.float32)
    s = np.asarray(conv_state, np.float32)
    w = np.asarray(weight, np.float32)
    B, T, C = x.shape
    K = s.shape[2]
    hs = np.concatenate([s, x.transpose(0, 2, 1)], axis=2)   # cat([conv_state, x], -1) (:95)
    new_state = hs[:, :, -K:].copy()                          # conv_state.copy_(...) (:96)
    L = hs.shape[2]
    kw = w.shape[1]
    out = np.zeros((B, C, L - kw + 1), np.float64)
    for j in range(kw):
        out += w[None, :, j:j + 1].astype(np.float64) * hs[:, :, j:j + L - kw + 1].astype(np.float64)
    out = round_to(out[:, :, -T:].astype(np.float32), in_dtype)  # conv1d, padding 0 (:97)
    out = round_to(_silu(out), in_dtype)                          # F.silu(out[:, :, -seq_len:]) (:98)
    return np.ascontiguousarray(out.transpose(0, 2, 1)), new_state


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus with beta=1, threshold=20, in float32."""
    x = np.asarray(x, np.float32)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def gates(a, b, A_log, dt_bias, in_dtype: str = "bf16"):
    """``beta = b.sigmoid()`` in b's dtype; ``g = -exp(A_log.float()) * softplus(a.float() + dt_bias)``
    in fp32 (:377-379).  a, b ``[B,T,H]``; A_log, dt_bias ``[H]`` (values already in their dtypes)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    beta = round_to((np.float32(1.0) / (np.float32(1.0) + np.exp(-b))).astype(np.float32), in_dtype)
    sp = softplus(a + np.asarray(dt_bias, np.float32)[None, None, :])
    g = (-np.exp(np.asarray(A_log, np.float32))[None, None, :] * sp).astype(np.float32)
    return g, beta


def rms_norm_gated(x, gate, weight, eps: float = 1e-6, in_dtype: str = "bf16"):
    """``Qwen3_5RMSNormGated.forward`` (:62-71) over the last dim of ``x [N, D]``."""
    h = np.asarray(x, np.float32)
    var = (h.astype(np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    hn = (h * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))).astype(np.float32)
    n = round_to(hn, in_dtype)                                                  # .to(input_dtype)
    wn = round_to((np.asarray(weight, np.float32)[None, :] * n).astype(np.float32), in_dtype)  # weight * h
    out = (wn * _silu(np.asarray(gate, np.float32))).astype(np.float32)        # * F.silu(gate.float())
    return round_to(out, in_dtype)                                              # .to(input_dtype)
