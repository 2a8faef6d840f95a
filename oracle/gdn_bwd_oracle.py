"""CPU oracle for the backward pass of the chunked gated delta rule.

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA backward in
``llms_from_scratch_b200``; only ``tests/``, ``__graft_entry__.smoke`` and
``bench.py``'s CPU legs may import it.  The product path never calls it.

The reference (pbanavara/llms_from_scratch) is inference-only: it has no
backward kernel.  Its pure-PyTorch forward ``torch_chunk_gated_delta_rule``
(qwen3_5_transformers.py:110-187) is differentiable, so the gradients autograd
takes through that function define the backward; ``tests/golden/make_golden_bwd.py``
records them and ``tests/test_bwd_oracle_golden.py`` pins this module to them (to the
reference's own fp32 round-off: the function casts to float32, :122-127).

This is the chunk-form backward written out by hand, chunk by chunk in reverse,
with the forward of ``gdn_oracle.chunk_gated_delta_rule`` recomputed on the
way.  Per chunk (64 tokens; Q = q^ Dk^-1/2, E_ij = e^(gc_i - gc_j),
L = -(beta k^ k^T) * E strictly lower, T = (I - L)^-1, u = T beta v,
w = T beta e^gc k^, Kd = k^ e^(gc_last - gc), Aqk = (Q k^T) * E incl. the
diagonal, Qg = Q e^gc, v_new = u - w S_c):

  forward   o_c = Qg S_c + Aqk v_new          S_{c+1} = e^gc_last S_c + Kd^T v_new
  backward  dv_new = Kd dS_{c+1} + Aqk^T do_c
            dS_c   = e^gc_last dS_{c+1} + Qg^T do_c - w^T dv_new
                   = M_c^T dS_{c+1} + Q'_c^T do_c   (M_c = e^gc_last I - Kd^T w, Q'_c = Qg - Aqk w)
            du = dv_new, dw = -dv_new S_c^T, d(beta v) = T^T du, d(beta e^gc k^) = T^T dw,
            dT = du (beta v)^T + dw (beta e^gc k^)^T, dL = (T^T dT T^T) strictly lower,
            then the elementwise chain rule through E, beta, e^gc and the l2norm.

Gradients come back in the reference layouts: dq, dk, dv ``[B,T,H,D]``,
dg, dbeta ``[B,T,H]``, dh0 ``[B,H,Dk,Dv]``.  The l2norm's derivative is taken
exactly (``x_hat = x (sum x^2 + 1e-6)^-1/2``); for 16-bit inputs the forward
values are rounded as the reference rounds them (``gdn_oracle._prep``) and the
derivative is taken at those values.
"""

from __future__ import annotations

import numpy as np

from .gdn_oracle import _prep, round_to

__all__ = ["chunk_gated_delta_rule_bwd"]


def _l2norm_bwd(x, dxh, eps=1e-6):
    """x_hat = x r, r = (sum x^2 + eps)^-1/2  ->  dx = r (dx_hat - x_hat (x_hat . dx_hat))."""
    r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) + eps)
    xh = x * r
    return r * (dxh - xh * (xh * dxh).sum(-1, keepdims=True))


def chunk_gated_delta_rule_bwd(
    query,
    key,
    value,
    g,
    beta,
    d_out,
    initial_state=None,
    d_final_state=None,
    chunk_size: int = 64,
    use_qk_l2norm_in_kernel: bool = False,
    in_dtype: str = "fp32",
    acc=np.float64,
):
    """Returns ``(dq, dk, dv, dg, dbeta, dh0)`` for ``chunk_gated_delta_rule``'s outputs receiving
    ``d_out [B,T,H,Dv]`` and (optionally) its final state receiving ``d_final_state [B,H,Dk,Dv]``."""
    q, k, v, gg, b = _prep(query, key, value, g, beta, use_qk_l2norm_in_kernel, in_dtype, acc)
    B, H, T, Dk = k.shape
    Dv = v.shape[-1]
    C = chunk_size
    pad = (C - T % C) % C
    do = np.ascontiguousarray(np.swapaxes(np.asarray(d_out, np.float64), 1, 2)).astype(acc)
    padt = ((0, 0), (0, 0), (0, pad), (0, 0))
    q, k, v, do = (np.pad(x, padt) for x in (q, k, v, do))
    b = np.pad(b, ((0, 0), (0, 0), (0, pad)))
    gg = np.pad(gg, ((0, 0), (0, 0), (0, pad)))
    NC = (T + pad) // C
    s = acc(1.0 / np.sqrt(Dk))
    rs = lambda x: x.reshape(B, H, NC, C, x.shape[-1])  # noqa: E731
    Q, K, V, dO = rs(q * s), rs(k), rs(v), rs(do)
    beta_c = b.reshape(B, H, NC, C)
    gc = np.cumsum(gg.reshape(B, H, NC, C), axis=-1, dtype=acc)
    incl = np.tril(np.ones((C, C), dtype=bool))
    strict = np.tril(np.ones((C, C), dtype=bool), k=-1)
    eye = np.eye(C, dtype=acc)
    tr = lambda x: np.swapaxes(x, -1, -2)  # noqa: E731

    # forward recompute, chunk quantities and chunk-start states
    E = np.where(incl, np.exp(np.where(incl, gc[..., :, None] - gc[..., None, :], 0)), 0)
    G = K @ tr(K)
    Lm = np.where(strict, -(beta_c[..., :, None] * G) * E, 0)
    Tm = np.linalg.solve(eye - Lm, np.broadcast_to(eye, Lm.shape))
    egc = np.exp(gc)
    vb = V * beta_c[..., None]
    kbe = K * (beta_c * egc)[..., None]
    U = Tm @ vb
    W = Tm @ kbe
    P = Q @ tr(K)
    Aqk = np.where(incl, P * E, 0)
    Qg = Q * egc[..., None]
    gl = gc[..., -1]
    ekd = np.exp(gl[..., None] - gc)
    Kd = K * ekd[..., None]
    gamma = np.exp(gl)
    S = np.zeros((B, H, Dk, Dv), acc) if initial_state is None else np.asarray(initial_state, np.float64).astype(acc)
    states = []
    for c in range(NC):
        states.append(S)
        vn = U[:, :, c] - W[:, :, c] @ S
        S = gamma[:, :, c, None, None] * S + tr(Kd[:, :, c]) @ vn

    dS = np.zeros((B, H, Dk, Dv), acc) if d_final_state is None else np.asarray(d_final_state, np.float64).astype(acc)
    dQ = np.zeros_like(Q)
    dK = np.zeros_like(K)
    dV = np.zeros_like(V)
    dbeta = np.zeros_like(beta_c)
    dgc = np.zeros_like(gc)
    for c in reversed(range(NC)):
        Sc = states[c]
        sl = (slice(None), slice(None), c)
        Kc, Qc, Vc, doc, Tc, Ec, Lc, Ac = K[sl], Q[sl], V[sl], dO[sl], Tm[sl], E[sl], Lm[sl], Aqk[sl]
        bc, ec, kdc, Wc = beta_c[sl], egc[sl], Kd[sl], W[sl]
        vn = U[sl] - Wc @ Sc
        dvn = kdc @ dS + tr(Ac) @ doc
        dQg = doc @ tr(Sc)
        dA = np.where(incl, doc @ tr(vn), 0)
        dKd = vn @ tr(dS)
        dgamma = (Sc * dS).sum((-1, -2))
        dS_prev = gamma[sl][..., None, None] * dS + tr(Qg[sl]) @ doc - tr(Wc) @ dvn
        dw = -dvn @ tr(Sc)
        d_vb = tr(Tc) @ dvn
        d_kbe = tr(Tc) @ dw
        dT = dvn @ tr(vb[sl]) + dw @ tr(kbe[sl])
        dL = np.where(strict, tr(Tc) @ dT @ tr(Tc), 0)
        # Aqk = P * E (incl.):  P = Q K^T
        dP = dA * Ec
        dQc = dP @ Kc + ec[..., None] * dQg
        dKc = tr(dP) @ Qc
        # L = -(beta_i G_ij) E_ij (strict)
        dG = np.where(strict, -(bc[..., :, None] * Ec) * dL, 0)
        dKc = dKc + dG @ Kc + tr(dG) @ Kc
        dbc = np.where(strict, -G[sl] * Ec * dL, 0).sum(-1)
        # E_ij = e^(gc_i - gc_j) in both
        R = Ac * dA + Lc * dL
        dgcc = R.sum(-1) - R.sum(-2)
        dgcc = dgcc + (Qg[sl] * dQg).sum(-1)
        # beta e^gc k^
        dKc = dKc + (bc * ec)[..., None] * d_kbe
        dbc = dbc + (Kc * ec[..., None] * d_kbe).sum(-1)
        dgcc = dgcc + (kbe[sl] * d_kbe).sum(-1)
        # Kd = k^ e^(gc_last - gc)
        dKc = dKc + ekd[sl][..., None] * dKd
        kd_dot = (kdc * dKd).sum(-1)
        dgcc = dgcc - kd_dot
        dgl = kd_dot.sum(-1) + gamma[sl] * dgamma
        dgcc[..., -1] += dgl
        # beta v
        dV[sl] = bc[..., None] * d_vb
        dbc = dbc + (Vc * d_vb).sum(-1)
        dQ[sl] = dQc
        dK[sl] = dKc
        dbeta[sl] = dbc
        dgc[sl] = dgcc
        dS = dS_prev

    dg = np.flip(np.cumsum(np.flip(dgc, -1), -1), -1)  # gc_i = sum_{t<=i} g_t
    unc = lambda x: np.ascontiguousarray(np.swapaxes(x.reshape(B, H, NC * C, x.shape[-1])[:, :, :T], 1, 2))  # noqa: E731
    dq_hat = unc(dQ) * s
    dk_hat = unc(dK)
    dv = unc(dV)
    if use_qk_l2norm_in_kernel:
        qin = np.asarray(query, np.float64)
        kin = np.asarray(key, np.float64)
        qin = round_to(qin.astype(np.float32), in_dtype).astype(np.float64)
        kin = round_to(kin.astype(np.float32), in_dtype).astype(np.float64)
        dq = _l2norm_bwd(qin, dq_hat)
        dk = _l2norm_bwd(kin, dk_hat)
    else:
        dq, dk = dq_hat, dk_hat
    dgo = np.ascontiguousarray(np.swapaxes(dg.reshape(B, H, NC * C)[:, :, :T], 1, 2))
    dbo = np.ascontiguousarray(np.swapaxes(dbeta.reshape(B, H, NC * C)[:, :, :T], 1, 2))
    return dq, dk, dv, dgo, dbo, dS
