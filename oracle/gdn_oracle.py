"""CPU oracle for the GatedDeltaNet chunked forward and recurrent step.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path in ``llms_from_scratch_b200``; only ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The product path never calls it and has no CPU fallback.

It is a numpy restatement of the two pure-PyTorch functions of the reference
(pbanavara/llms_from_scratch):

* ``chunk_gated_delta_rule``   follows ``torch_chunk_gated_delta_rule``
  (qwen3_5_transformers.py:110-187), which is also what
  ``fast_chunk_gated_delta_rule(backend="torch")`` runs
  (qwen3_5_cutedsl_kernels.py:483-491);
* ``recurrent_gated_delta_rule`` follows ``torch_recurrent_gated_delta_rule``
  (qwen3_5_transformers.py:190-229).

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against fixtures produced by the reference's own torch code
(``tests/golden/make_golden.py``).

Arrays are numpy; layouts follow the reference contract:
q, k ``[B, T, H, Dk]``, v ``[B, T, H, Dv]``, g, beta ``[B, T, H]``,
state ``[B, H, Dk, Dv]``, output ``[B, T, H, Dv]``.

``in_dtype`` names the dtype the reference tensors would have had ("fp32",
"bf16" or "fp16").  The reference runs ``l2norm`` *before* its fp32 cast
(qwen3_5_transformers.py:122-127), so for 16-bit inputs the normalised q/k are
rounded to that dtype; the oracle reproduces those roundings, and rounds the
output to ``in_dtype`` as the reference's final ``.to(initial_dtype)`` does
(qwen3_5_transformers.py:186, :228).  Intermediate arithmetic is float32 like
the reference, or float64 with ``acc=np.float64`` for a higher-precision
reference value.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "round_bf16",
    "round_fp16",
    "round_to",
    "bf16_bits",
    "from_bf16_bits",
    "l2norm",
    "chunk_gated_delta_rule",
    "recurrent_gated_delta_rule",
    "make_inputs",
]


# ---------------------------------------------------------------------------
# 16-bit rounding helpers (numpy has no bfloat16)
# ---------------------------------------------------------------------------

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    b = (b + 0x7FFF + lsb) & 0xFFFF0000
    out = b.astype(np.uint32).view(np.float32)
    # keep NaN as NaN (the add above could carry a NaN payload into Inf)
    return np.where(np.isnan(x), x, out)


def round_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, in_dtype: str) -> np.ndarray:
    if in_dtype == "fp32":
        return np.asarray(x, dtype=np.float32)
    if in_dtype == "bf16":
        return round_bf16(x)
    if in_dtype == "fp16":
        return round_fp16(x)
    raise ValueError(f"unknown dtype {in_dtype!r}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of float32 values already rounded to bf16."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# l2norm: qwen3_5_transformers.py:104-107 / qwen3_5_cutedsl_kernels.py:100-101
# ---------------------------------------------------------------------------

def l2norm(x: np.ndarray, in_dtype: str = "fp32", eps: float = 1e-6) -> np.ndarray:
    """``x * rsqrt(sum(x*x, -1) + eps)`` evaluated in ``in_dtype``.

    For 16-bit inputs torch evaluates each elementwise op in that dtype (the
    sum accumulates in float32 and is rounded once), so every intermediate is
    rounded here in the same places.
    """
    x = np.asarray(x, dtype=np.float32)
    if in_dtype == "fp32":
        inv = 1.0 / np.sqrt((x * x).sum(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
        return (x * inv.astype(np.float32)).astype(np.float32)
    sq = round_to(x * x, in_dtype)
    s = round_to(sq.sum(axis=-1, keepdims=True, dtype=np.float32), in_dtype)
    s = round_to(s + np.float32(eps), in_dtype)
    inv = round_to(1.0 / np.sqrt(s), in_dtype)
    return round_to(x * inv, in_dtype)


def _prep(query, key, value, g, beta, use_qk_l2norm, in_dtype, acc):
    """l2norm then transpose [B,T,H,*] -> [B,H,T,*] and cast (qwen3_5_transformers.py:122-127)."""
    query = round_to(query, in_dtype)
    key = round_to(key, in_dtype)
    value = round_to(value, in_dtype)
    if use_qk_l2norm:
        query = l2norm(query, in_dtype)
        key = l2norm(key, in_dtype)
    q = np.ascontiguousarray(np.swapaxes(query, 1, 2)).astype(acc)
    k = np.ascontiguousarray(np.swapaxes(key, 1, 2)).astype(acc)
    v = np.ascontiguousarray(np.swapaxes(value, 1, 2)).astype(acc)
    b = np.ascontiguousarray(np.swapaxes(np.asarray(beta, np.float32), 1, 2)).astype(acc)
    gg = np.ascontiguousarray(np.swapaxes(np.asarray(g, np.float32), 1, 2)).astype(acc)
    return q, k, v, gg, b


# ---------------------------------------------------------------------------
# Chunked rule: qwen3_5_transformers.py:110-187
# ---------------------------------------------------------------------------

def chunk_gated_delta_rule(
    query,
    key,
    value,
    g,
    beta,
    chunk_size: int = 64,
    initial_state=None,
    output_final_state: bool = False,
    use_qk_l2norm_in_kernel: bool = False,
    in_dtype: str = "fp32",
    acc=np.float32,
):
    """Chunked gated delta rule; returns ``(out [B,T,H,Dv], state [B,H,Dk,Dv] or None)``.

    Step by step as in the reference:
      * pad T to a multiple of ``chunk_size`` with zeros (:131-137);
      * ``q *= 1/sqrt(Dk)`` (:138-139); ``k_beta = k*beta``, ``v_beta = v*beta`` (:141-142);
      * per-chunk cumulative sum of g (:151) and the lower decay mask
        ``exp(gc_i - gc_j)`` (:152);
      * ``attn = -(k_beta k^T * decay)`` strictly lower (:153), forward
        substitution (:154-157), ``+ I`` (:158);
      * ``u = attn v_beta`` (:159), ``w = attn (k_beta * exp(gc))`` (:160);
      * the chunk loop (:170-180) with the causal intra-chunk attention (incl.
        the diagonal), ``v_new = u - w S``, output and state update.
    """
    q, k, v, gg, b = _prep(query, key, value, g, beta, use_qk_l2norm_in_kernel, in_dtype, acc)
    B, H, T, Dk = k.shape
    Dv = v.shape[-1]
    C = chunk_size
    pad = (C - T % C) % C
    if pad:
        q = np.pad(q, ((0, 0), (0, 0), (0, pad), (0, 0)))
        k = np.pad(k, ((0, 0), (0, 0), (0, pad), (0, 0)))
        v = np.pad(v, ((0, 0), (0, 0), (0, pad), (0, 0)))
        b = np.pad(b, ((0, 0), (0, 0), (0, pad)))
        gg = np.pad(gg, ((0, 0), (0, 0), (0, pad)))
    Tp = T + pad
    NC = Tp // C
    q = q * acc(1.0 / np.sqrt(Dk))
    v_beta = v * b[..., None]
    k_beta = k * b[..., None]
    q, k, v, k_beta, v_beta = [x.reshape(B, H, NC, C, x.shape[-1]) for x in (q, k, v, k_beta, v_beta)]
    gc = np.cumsum(gg.reshape(B, H, NC, C), axis=-1, dtype=acc)

    lower_incl = np.tril(np.ones((C, C), dtype=bool))
    strict_lower = np.tril(np.ones((C, C), dtype=bool), k=-1)
    diff = gc[..., :, None] - gc[..., None, :]
    # tril().exp().tril(): entries above the diagonal become exp(0)=1 and are
    # then zeroed again, so the mask is exp(diff) on and below the diagonal.
    decay = np.where(lower_incl, np.exp(np.where(lower_incl, diff, 0)), 0).astype(acc)

    attn = -np.einsum("...ik,...jk->...ij", k_beta, k) * decay
    attn = np.where(strict_lower, attn, 0).astype(acc)
    for i in range(1, C):
        row = attn[..., i, :i].copy()
        sub = attn[..., :i, :i].copy()
        attn[..., i, :i] = row + (row[..., :, None] * sub).sum(-2)
    attn = attn + np.eye(C, dtype=acc)
    u = attn @ v_beta
    w = attn @ (k_beta * np.exp(gc)[..., None])

    if initial_state is None:
        S = np.zeros((B, H, Dk, Dv), dtype=acc)
    else:
        S = np.asarray(initial_state, dtype=np.float32).astype(acc).copy()
    out = np.zeros((B, H, NC, C, Dv), dtype=acc)
    for c in range(NC):
        q_c, k_c, u_c, w_c, gc_c = q[:, :, c], k[:, :, c], u[:, :, c], w[:, :, c], gc[:, :, c]
        a_qk = np.where(lower_incl, (q_c @ np.swapaxes(k_c, -1, -2)) * decay[:, :, c], 0).astype(acc)
        v_new = u_c - w_c @ S
        o_inter = (q_c * np.exp(gc_c)[..., None]) @ S
        out[:, :, c] = o_inter + a_qk @ v_new
        g_last = gc_c[..., -1]
        k_dec = k_c * np.exp(g_last[..., None] - gc_c)[..., None]
        S = S * np.exp(g_last)[..., None, None] + np.swapaxes(k_dec, -1, -2) @ v_new

    out = out.reshape(B, H, Tp, Dv)[:, :, :T]
    out = np.ascontiguousarray(np.swapaxes(out, 1, 2))
    out = round_to(out.astype(np.float32), in_dtype) if acc == np.float32 else out
    return out, (S if output_final_state else None)


# ---------------------------------------------------------------------------
# Recurrent rule: qwen3_5_transformers.py:190-229
# ---------------------------------------------------------------------------

def recurrent_gated_delta_rule(
    query,
    key,
    value,
    g,
    beta,
    initial_state,
    output_final_state: bool,
    use_qk_l2norm_in_kernel: bool = False,
    in_dtype: str = "fp32",
    acc=np.float32,
):
    """Token-by-token gated delta rule (:213-224):
    ``S *= exp(g); kv = S^T k; delta = beta (v - kv); S += k delta^T; o = S^T q``."""
    q, k, v, gg, b = _prep(query, key, value, g, beta, use_qk_l2norm_in_kernel, in_dtype, acc)
    B, H, T, Dk = k.shape
    Dv = v.shape[-1]
    q = q * acc(1.0 / np.sqrt(Dk))
    if initial_state is None:
        S = np.zeros((B, H, Dk, Dv), dtype=acc)
    else:
        S = np.asarray(initial_state, dtype=np.float32).astype(acc).copy()
    out = np.zeros((B, H, T, Dv), dtype=acc)
    for t in range(T):
        S = S * np.exp(gg[:, :, t])[..., None, None]
        kv = (S * k[:, :, t][..., :, None]).sum(-2)
        delta = (v[:, :, t] - kv) * b[:, :, t][..., None]
        S = S + k[:, :, t][..., :, None] * delta[..., None, :]
        out[:, :, t] = (S * q[:, :, t][..., :, None]).sum(-2)
    out = np.ascontiguousarray(np.swapaxes(out, 1, 2))
    out = round_to(out.astype(np.float32), in_dtype) if acc == np.float32 else out
    return out, (S if output_final_state else None)


# ---------------------------------------------------------------------------
# Seeded synthetic inputs with the distributions of the benchmark configs
# ---------------------------------------------------------------------------

def make_inputs(B, T, H, D=128, seed=0, in_dtype="fp32", init_state_std=0.0, normalize_qk=True):
    """q,k ~ N(0,1) then L2-normalised per head vector; v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = -softplus(N(0,1)); optional initial state
    ~ N(0, init_state_std).  q/k/v are rounded to ``in_dtype``; g, beta and
    the state stay float32.  numpy's PCG64 stream makes these reproducible
    on any machine."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, D), dtype=np.float32)
    k = rng.standard_normal((B, T, H, D), dtype=np.float32)
    v = rng.standard_normal((B, T, H, D), dtype=np.float32)
    if normalize_qk:
        q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
        k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H), dtype=np.float32)))).astype(np.float32)
    a = rng.standard_normal((B, T, H), dtype=np.float32)
    g = (-np.logaddexp(0.0, a)).astype(np.float32)
    state = None
    if init_state_std > 0:
        state = (rng.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(init_state_std)).astype(np.float32)
    q, k, v = (round_to(x, in_dtype) for x in (q, k, v))
    return q, k, v, g, beta, state
