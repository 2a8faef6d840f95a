"""A Qwen3.5-0.8B-shaped hybrid decoder that drives the GatedDeltaNet path end to end.

The reference builds this model from torch modules (``Qwen3_5Model``,
qwen3_5.py:240-283: embedding, 24 blocks of which every fourth is full
attention and the rest are ``Qwen3_5GatedDeltaNet``, final RMSNorm, LM head)
and generates greedily by re-running the whole prefix for every new token
(qwen3_5.py:483-495, benchmark.py:318-335): it has no cache (its
``Qwen3_5DynamicCache`` is an empty placeholder, qwen3_5_transformers.py:50-53).

``Qwen35Decoder`` runs the same architecture on the sm_100a library with a
cache, the way the GatedDeltaNet layer's own cache contract
(qwen3_5_transformers.py:312-326, :343-348, :401-402) intends:

* prefill: the prompt goes through every layer once; the linear-attention
  layers run the prefill convolution (which also fills the conv state) and the
  chunked rule with ``output_final_state=True`` (the recurrent state); the
  full-attention layers write their keys and values into a KV cache;
* decode: each new token runs the conv update, the gates and the recurrent
  rule in place on those states, and attends over the KV cache.  One decode
  step is a fixed sequence of kernels over static buffers, so it is captured
  once in a CUDA graph and replayed per token (the position lives on the
  device and the step advances it).

The projections are plain bf16 GEMMs (cuBLAS through ``torch.nn.functional.
linear``) on weights fused per layer ([qkv | z | b | a], [W_query | W_key |
W_value], [fc1 | fc2]); everything else is this package's kernels.  Weights are
random (``random_weights``): the Qwen3.5-0.8B checkpoint is not available to
this build, so this serves the benchmark's config 4 (random N(0, 0.02)
weights) and the parity tests against the reference's model on the same
weights.
"""

from __future__ import annotations

import ctypes
import math
from types import SimpleNamespace
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import _lib, layer
from .ops import _desc, check_device_errors, fast_chunk_gated_delta_rule, fast_recurrent_gated_delta_rule

# Qwen3.5-0.8B's text stack (qwen3_5.py:287-320) at the benchmark's vocabulary size (151,936).
QWEN3_5_0_8B = {
    "vocab_size": 151_936,
    "emb_dim": 1_024,
    "n_heads": 8,
    "n_layers": 24,
    "hidden_dim": 3_584,
    "head_dim": 256,
    "qk_norm": True,
    "n_kv_groups": 2,
    "rope_base": 10_000_000.0,
    "partial_rotary_factor": 0.25,
    "rms_norm_eps": 1e-6,
    "linear_conv_kernel_dim": 4,
    "linear_key_head_dim": 128,
    "linear_value_head_dim": 128,
    "linear_num_key_heads": 16,
    "linear_num_value_heads": 16,
    "layer_types": (["linear_attention"] * 3 + ["full_attention"]) * 6,
}


def parameter_shapes(cfg: dict) -> List[tuple]:
    """``(name, shape)`` of every parameter, named as the reference's ``Qwen3_5Model`` names them
    (qwen3_5.py:117-283, qwen3_5_transformers.py:231-300), so its ``load_state_dict`` takes them."""
    E, V, F_ = cfg["emb_dim"], cfg["vocab_size"], cfg["hidden_dim"]
    Hq, Hkv, Dh = cfg["n_heads"], cfg["n_kv_groups"], cfg["head_dim"]
    Hk, Hv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
    Dk, Dv, K = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"], cfg["linear_conv_kernel_dim"]
    C = 2 * Hk * Dk + Hv * Dv
    shapes = [("tok_emb.weight", (V, E))]
    for i, kind in enumerate(cfg["layer_types"]):
        p = f"trf_blocks.{i}."
        m = p + "token_mixer."
        if kind == "full_attention":
            shapes += [(m + "W_query.weight", (2 * Hq * Dh, E)), (m + "W_key.weight", (Hkv * Dh, E)),
                       (m + "W_value.weight", (Hkv * Dh, E)), (m + "out_proj.weight", (E, Hq * Dh)),
                       (m + "q_norm.weight", (Dh,)), (m + "k_norm.weight", (Dh,))]
        else:
            shapes += [(m + "dt_bias", (Hv,)), (m + "A_log", (Hv,)), (m + "conv1d.weight", (C, 1, K)),
                       (m + "norm.weight", (Dv,)), (m + "out_proj.weight", (E, Hv * Dv)),
                       (m + "in_proj_qkv.weight", (C, E)), (m + "in_proj_z.weight", (Hv * Dv, E)),
                       (m + "in_proj_b.weight", (Hv, E)), (m + "in_proj_a.weight", (Hv, E))]
        shapes += [(p + "ff.fc1.weight", (F_, E)), (p + "ff.fc2.weight", (F_, E)), (p + "ff.fc3.weight", (E, F_)),
                   (p + "norm1.weight", (E,)), (p + "norm2.weight", (E,))]
    shapes += [("final_norm.weight", (E,)), ("out_head.weight", (V, E))]
    return shapes


def random_weights(cfg: dict, seed: int = 0, std: float = 0.02, device="cpu") -> Dict[str, torch.Tensor]:
    """Seeded random weights in bf16: every parameter ~ N(0, std) drawn in ``parameter_shapes`` order from
    one generator on ``device``, except the gated RMS norm's scale, which keeps the reference's
    initialisation (ones, qwen3_5_transformers.py:57-59) because it multiplies the normalised output
    directly: N(0, 0.02) there would scale every linear-attention layer's contribution down fifty-fold.
    The RMSNorms take ``1 + weight`` (qwen3_5.py:60-63), so N(0, std) is near one.  Host draws are
    reproducible on any machine (the parity fixtures use them); device draws are faster but are other
    values."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = {}
    for name, shape in parameter_shapes(cfg):
        if name.endswith("token_mixer.norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
        else:
            out[name] = (torch.randn(shape, generator=gen, device=device) * std).to(torch.bfloat16)
    return out


def weight_checksum(weights: Dict[str, torch.Tensor]) -> float:
    """The float64 sum of |w| over every parameter: identifies a weight set, e.g. shows that
    ``random_weights`` drew the same values on two machines."""
    return float(sum(v.double().abs().sum().item() for v in weights.values()))


def rope_tables(cfg: dict, max_len: int):
    """cos / sin ``[max_len, rotary_dim]`` fp32, computed as ``compute_rope_params`` does (qwen3_5.py:66-90)."""
    Dh = cfg["head_dim"]
    rot = int(Dh * cfg.get("partial_rotary_factor", 1.0))
    rot = max(2, rot - (rot % 2))
    inv_freq = 1.0 / (cfg["rope_base"] ** (torch.arange(0, rot, 2, dtype=torch.float32)[: rot // 2].float() / rot))
    pos = torch.arange(max_len, dtype=torch.float32)
    ang = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    ang = torch.cat([ang, ang], dim=1)
    return torch.cos(ang), torch.sin(ang), rot


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def add_rms_norm(x, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None):
    """``RMSNorm(x + residual)`` with the (1 + weight) scale (``gdn_model_add_rms_norm``); returns
    ``(normed, x + residual)`` (the new residual stream written into ``residual``) or ``(normed, x)``.
    ``x`` may be a ``Partial`` (then ``residual`` is required and shapes follow it)."""
    if isinstance(x, Partial):
        ns, rows, D = x.buf.shape
        r2 = residual.reshape(rows, D)
        o = torch.empty((rows, D), dtype=residual.dtype, device=residual.device) if out is None else out.reshape(rows, D)
        dr, dw, do = _desc(r2), _desc(weight), _desc(o)
        _lib.check(_lib.load().gdn_model_add_rms_norm_partials(x.buf.data_ptr(), ns, rows, D, ctypes.byref(dr),
                                                               ctypes.byref(dw), float(eps), ctypes.byref(do),
                                                               ctypes.byref(dr), _stream(residual.device)))
        return o.reshape(residual.shape), residual
    D = x.shape[-1]
    x2 = x.reshape(-1, D)
    o = torch.empty_like(x2) if out is None else out.reshape(-1, D)
    r2 = residual.reshape(-1, D) if residual is not None else None
    lib = _lib.load()
    dx, dw, do = _desc(x2), _desc(weight), _desc(o)
    if r2 is not None:
        dr = _desc(r2)
        rc = lib.gdn_model_add_rms_norm(ctypes.byref(dx), ctypes.byref(dr), ctypes.byref(dw), float(eps),
                                        ctypes.byref(do), ctypes.byref(dr), _stream(x.device))
    else:
        rc = lib.gdn_model_add_rms_norm(ctypes.byref(dx), None, ctypes.byref(dw), float(eps), ctypes.byref(do),
                                        None, _stream(x.device))
    _lib.check(rc)
    return o.reshape(x.shape), (residual if residual is not None else x)


EPI_STORE, EPI_SILU_MUL, EPI_PARTIAL = 0, 1, 2
DECODE_MAX_ROWS = 32  # gdn_model_linear's batch limit


class Partial:
    """fp32 split-K partial sums ``[nsplit, rows, dim]`` of a projection, summed (in plane order) and rounded
    to bf16 by the ``add_rms_norm`` that consumes them."""

    def __init__(self, buf: torch.Tensor):
        self.buf = buf


def linear(x: torch.Tensor, w: torch.Tensor, epilogue: int = EPI_STORE, ksplit: int = 1):
    """``x [M, K] @ w.T`` for a decode batch (M <= 32) on ``gdn_model_linear``: bf16 ``[M, N]``
    (``EPI_STORE``), the FFN's ``SiLU(fc1) * fc2`` ``[M, N / 2]`` from fc1/fc2 rows interleaved in groups of 8
    (``EPI_SILU_MUL``), or a ``Partial`` over ``ksplit`` CTAs along K (``EPI_PARTIAL``)."""
    M, N = x.shape[0], w.shape[0]
    lib = _lib.load()
    dx, dw = _desc(x), _desc(w)
    if epilogue == EPI_PARTIAL:
        buf = torch.empty((ksplit, M, N), dtype=torch.float32, device=x.device)
        _lib.check(lib.gdn_model_linear(ctypes.byref(dx), ctypes.byref(dw), None, buf.data_ptr(), int(ksplit),
                                        EPI_PARTIAL, _stream(x.device)))
        return Partial(buf)
    out = torch.empty((M, N // 2 if epilogue == EPI_SILU_MUL else N), dtype=x.dtype, device=x.device)
    do = _desc(out)
    _lib.check(lib.gdn_model_linear(ctypes.byref(dx), ctypes.byref(dw), ctypes.byref(do), None, 1, int(epilogue),
                                    _stream(x.device)))
    return out


def interleave_fc12(fc1: torch.Tensor, fc2: torch.Tensor) -> torch.Tensor:
    """fc1 / fc2 ``[F, E]`` as one ``[2F, E]`` weight in row groups of 8 (fc1 rows 8j..8j+7, then fc2 rows
    8j..8j+7): the layout ``EPI_SILU_MUL`` pairs."""
    F_, E = fc1.shape
    return torch.stack([fc1.view(F_ // 8, 8, E), fc2.view(F_ // 8, 8, E)], 1).reshape(2 * F_, E).contiguous()


def silu_mul(u: torch.Tensor) -> torch.Tensor:
    """``SiLU(u[..., :F]) * u[..., F:]`` (``gdn_model_silu_mul``)."""
    W = u.shape[-1]
    u2 = u.reshape(-1, W)
    o = torch.empty((u2.shape[0], W // 2), dtype=u.dtype, device=u.device)
    du, do = _desc(u2), _desc(o)
    _lib.check(_lib.load().gdn_model_silu_mul(ctypes.byref(du), ctypes.byref(do), _stream(u.device)))
    return o.reshape(*u.shape[:-1], W // 2)


def gated_norm(core: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``Qwen3_5RMSNormGated`` over ``[M, H, 128]`` views (``gdn_rms_norm_gated``): the gate z stays a strided
    view of the fused projection."""
    out = torch.empty(core.shape, dtype=core.dtype, device=core.device)
    dx, dz, dw, do = _desc(core), _desc(z), _desc(weight), _desc(out)
    _lib.check(_lib.load().gdn_rms_norm_gated(ctypes.byref(dx), ctypes.byref(dz), ctypes.byref(dw), float(eps),
                                              ctypes.byref(do), _stream(core.device)))
    return out


def gdn_decode(proj: torch.Tensor, conv_state: torch.Tensor, conv_w: torch.Tensor, A_log: torch.Tensor,
               dt_bias: torch.Tensor, state: torch.Tensor, norm_w: torch.Tensor, eps: float,
               prefetch_state: bool = False) -> torch.Tensor:
    """One decode token of a GatedDeltaNet layer from its fused input projection ``proj [B, 3HD + HD + 2H]``
    (``gdn_model_gdn_decode``: conv update, gates, recurrent rule and gated norm in one kernel; ``conv_state``
    and ``state`` updated in place); returns the normed output ``[B, H*128]``.  ``prefetch_state``: no kernel
    that may still run writes ``state`` (the decoder's steps guarantee it), so its loads start early."""
    B = proj.shape[0]
    H = A_log.shape[0]
    out = torch.empty((B, H * 128), dtype=proj.dtype, device=proj.device)
    d = [_desc(t) for t in (proj, conv_state, conv_w, A_log, dt_bias, norm_w, out)]
    _lib.check(_lib.load().gdn_model_gdn_decode(ctypes.byref(d[0]), ctypes.byref(d[1]), ctypes.byref(d[2]),
                                                ctypes.byref(d[3]), ctypes.byref(d[4]), state.data_ptr(),
                                                ctypes.byref(d[5]), float(eps), ctypes.byref(d[6]),
                                                int(bool(prefetch_state)), _stream(proj.device)))
    return out


class Qwen35Cache:
    """Decode state of a batch: per linear-attention layer the conv state ``[B, C, 4]`` (the layer dtype) and
    the recurrent state ``[B, H, Dk, Dv]`` fp32 -- the ``conv_states`` / ``recurrent_states`` /
    ``has_previous_state`` contract of the reference's layer (qwen3_5_transformers.py:312-326, :343-348,
    :401-402) -- and per full-attention layer a key and a value cache ``[B, Hkv, max_len, Dh]``.  ``pos`` is
    the position of the next token, on the device (one int32)."""

    def __init__(self, cfg: dict, batch: int, max_len: int, device, dtype=torch.bfloat16):
        Hk, Hv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        Dk, Dv, K = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"], cfg["linear_conv_kernel_dim"]
        C = 2 * Hk * Dk + Hv * Dv
        self.batch, self.max_len = batch, max_len
        self.conv_states: Dict[int, torch.Tensor] = {}
        self.recurrent_states: Dict[int, torch.Tensor] = {}
        self.key_cache: Dict[int, torch.Tensor] = {}
        self.value_cache: Dict[int, torch.Tensor] = {}
        for i, kind in enumerate(cfg["layer_types"]):
            if kind == "linear_attention":
                self.conv_states[i] = torch.zeros(batch, C, K, dtype=dtype, device=device)
                self.recurrent_states[i] = torch.zeros(batch, Hv, Dk, Dv, dtype=torch.float32, device=device)
            else:
                shape = (batch, cfg["n_kv_groups"], max_len, cfg["head_dim"])
                self.key_cache[i] = torch.zeros(shape, dtype=dtype, device=device)
                self.value_cache[i] = torch.zeros(shape, dtype=dtype, device=device)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        self.has_previous_state = False


class Qwen35Decoder:
    """The Qwen3.5-shaped decoder on this package's kernels (module docstring).  ``weights`` maps the
    reference's parameter names (``parameter_shapes``) to tensors; they are copied to ``device`` in bf16 and
    fused per layer."""

    def __init__(self, cfg: dict, weights: Dict[str, torch.Tensor], device="cuda", max_len: int = 256):
        self.cfg = dict(cfg)
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_len = max_len
        self.eps = cfg.get("rms_norm_eps", 1e-6)
        bf = torch.bfloat16

        def w(name):
            return weights[name].to(device=self.device, dtype=bf).contiguous()

        self.emb = w("tok_emb.weight")
        self.head = w("out_head.weight")
        self.final_norm = w("final_norm.weight")
        Hk, Hv = cfg["linear_num_key_heads"], cfg["linear_num_value_heads"]
        Dk, Dv = cfg["linear_key_head_dim"], cfg["linear_value_head_dim"]
        self.gdn = SimpleNamespace(Hk=Hk, Hv=Hv, Dk=Dk, Dv=Dv, key_dim=Hk * Dk, value_dim=Hv * Dv,
                                   C=2 * Hk * Dk + Hv * Dv)
        if Hv != Hk:
            raise NotImplementedError("the decoder runs equal key and value head counts (Qwen3.5-0.8B: 16 / 16)")
        self.layers = []
        for i, kind in enumerate(cfg["layer_types"]):
            p = f"trf_blocks.{i}."
            m = p + "token_mixer."
            L = SimpleNamespace(kind=kind, idx=i, norm1=w(p + "norm1.weight"), norm2=w(p + "norm2.weight"),
                                fc12=interleave_fc12(w(p + "ff.fc1.weight"), w(p + "ff.fc2.weight")),
                                fc3=w(p + "ff.fc3.weight"))
            if kind == "linear_attention":
                L.w_in = torch.cat([w(m + "in_proj_qkv.weight"), w(m + "in_proj_z.weight"),
                                    w(m + "in_proj_b.weight"), w(m + "in_proj_a.weight")]).contiguous()
                L.conv_w = w(m + "conv1d.weight").squeeze(1).contiguous()
                L.A_log, L.dt_bias = w(m + "A_log"), w(m + "dt_bias")
                L.gnorm, L.w_out = w(m + "norm.weight"), w(m + "out_proj.weight")
            else:
                L.w_qkv = torch.cat([w(m + "W_query.weight"), w(m + "W_key.weight"),
                                     w(m + "W_value.weight")]).contiguous()
                L.qn, L.kn, L.w_out = w(m + "q_norm.weight"), w(m + "k_norm.weight"), w(m + "out_proj.weight")
            self.layers.append(L)
        cos, sin, self.rot = rope_tables(cfg, max_len)
        self.rope_cos = cos.to(self.device).contiguous()
        self.rope_sin = sin.to(self.device).contiguous()
        self._graph = None

    # ------------------------------------------------------------------ mixers

    def _proj(self, h: torch.Tensor, w: torch.Tensor, epilogue: int = EPI_STORE, ksplit: int = 1):
        """``h [..., K] -> [..., N]``: the decode kernel (``linear``) for at most 32 rows, the library GEMM
        otherwise; ``EPI_SILU_MUL`` applies the FFN activation to fc1/fc2 interleaved rows either way, and
        ``EPI_PARTIAL`` may return a ``Partial`` (any consumer takes both forms through ``add_rms_norm``)."""
        lead = h.shape[:-1]
        x = h.reshape(-1, h.shape[-1])
        if x.shape[0] <= DECODE_MAX_ROWS:
            y = linear(x, w, epilogue, ksplit)
            return y if isinstance(y, Partial) else y.view(*lead, y.shape[-1])
        y = F.linear(x, w)
        if epilogue == EPI_SILU_MUL:
            u = y.unflatten(-1, (-1, 2, 8))
            y = (F.silu(u[..., 0, :]) * u[..., 1, :]).flatten(-2)
        return y.view(*lead, y.shape[-1])

    def _gdn(self, L, h: torch.Tensor, cache: Qwen35Cache, decode: bool) -> torch.Tensor:
        g_ = self.gdn
        B, T, _ = h.shape
        proj = self._proj(h, L.w_in)  # [B, T, C + value_dim + 2 Hv]
        C, Vd, Hv = g_.C, g_.value_dim, g_.Hv
        mixed = proj[..., :C]
        z = proj[..., C:C + Vd]
        b = proj[..., C + Vd:C + Vd + Hv]
        a = proj[..., C + Vd + Hv:C + Vd + 2 * Hv]
        conv_state = cache.conv_states[L.idx]
        if decode and T == 1:  # one token: conv update, gates, recurrent rule and gated norm in one kernel
            # the state was last written by this layer's call in the previous step, before the step's
            # embedding (a plain launch): its loads may start while the projection before runs
            normed = gdn_decode(proj.reshape(B, -1), conv_state, L.conv_w, L.A_log, L.dt_bias,
                                cache.recurrent_states[L.idx], L.gnorm, self.eps, prefetch_state=True)
            return self._proj(normed.view(B, 1, Vd), L.w_out, EPI_PARTIAL, 8)
        if decode:  # torch_causal_conv1d_update against the cached state (qwen3_5_transformers.py:337-343)
            conv = layer.causal_conv1d_update(mixed.transpose(1, 2), conv_state, L.conv_w, None, "silu")
            conv = conv.transpose(1, 2)
        else:  # prefill conv + SiLU; the last four inputs become the conv state (:346-356)
            conv = layer.causal_conv1d_silu(mixed, L.conv_w, conv_state=conv_state)
        g, beta = layer.gates(a, b, L.A_log, L.dt_bias)
        kd = g_.key_dim
        q = conv[..., :kd].unflatten(-1, (g_.Hk, g_.Dk))
        k = conv[..., kd:2 * kd].unflatten(-1, (g_.Hk, g_.Dk))
        v = conv[..., 2 * kd:].unflatten(-1, (Hv, g_.Dv))
        state = cache.recurrent_states[L.idx]
        if decode:  # recurrent rule, state updated in place (:396-402)
            core, _ = fast_recurrent_gated_delta_rule(q, k, v, g, beta, state, True, use_qk_l2norm_in_kernel=True,
                                                      out_state=state)
        else:  # chunked rule over the prompt, final state into the cache (:384-392, :401-402)
            core, final = fast_chunk_gated_delta_rule(q, k, v, g, beta, initial_state=None, output_final_state=True,
                                                      use_qk_l2norm_in_kernel=True)
            state.copy_(final)
        normed = gated_norm(core.reshape(B * T, Hv, g_.Dv), z.reshape(B * T, Hv, g_.Dv), L.gnorm, self.eps)
        return self._proj(normed.reshape(B, T, Vd), L.w_out, EPI_PARTIAL, 8)

    def _attention(self, L, h: torch.Tensor, cache: Qwen35Cache) -> torch.Tensor:
        cfg = self.cfg
        B, T, _ = h.shape
        Hq, Hkv, Dh = cfg["n_heads"], cfg["n_kv_groups"], cfg["head_dim"]
        qkv = self._proj(h, L.w_qkv)  # [B, T, Hq (q | gate) + Hkv k + Hkv v]
        q = torch.empty((B, T, Hq, Dh), dtype=h.dtype, device=h.device)
        kc, vc = cache.key_cache[L.idx], cache.value_cache[L.idx]
        lib = _lib.load()
        dqkv, dqn, dkn, dq, dkc, dvc = (_desc(x) for x in (qkv, L.qn, L.kn, q, kc, vc))
        _lib.check(lib.gdn_model_attn_prep(ctypes.byref(dqkv), ctypes.byref(dqn), ctypes.byref(dkn),
                                           self.rope_cos.data_ptr(), self.rope_sin.data_ptr(), self.rot,
                                           cache.pos.data_ptr(), float(self.eps), ctypes.byref(dq), ctypes.byref(dkc),
                                           ctypes.byref(dvc), _stream(h.device)))
        gate = qkv[..., :Hq * 2 * Dh].unflatten(-1, (Hq, 2 * Dh))[..., Dh:]
        ctx = torch.empty((B, T, Hq * Dh), dtype=h.dtype, device=h.device)
        dg, dctx = _desc(gate), _desc(ctx)
        _lib.check(lib.gdn_model_attention(ctypes.byref(dq), ctypes.byref(dkc), ctypes.byref(dvc), ctypes.byref(dg),
                                           cache.pos.data_ptr(), ctypes.byref(dctx), _stream(h.device)))
        return self._proj(ctx, L.w_out, EPI_PARTIAL, 8)

    # ------------------------------------------------------------------ model

    def forward(self, ids: torch.Tensor, cache: Qwen35Cache, decode: bool) -> torch.Tensor:
        """Logits of the last position, ``[B, vocab]`` bf16, for tokens ``ids [B, T]`` at positions
        ``cache.pos ..``; updates the cache and advances ``cache.pos`` by T (on the device)."""
        B, T = ids.shape
        x = F.embedding(ids, self.emb)
        h, res = add_rms_norm(x, self.layers[0].norm1, self.eps)
        res = res.clone()  # the residual stream is written in place from here on
        delta = None
        for li, L in enumerate(self.layers):
            if li > 0:
                h, res = add_rms_norm(delta, L.norm1, self.eps, residual=res)
            mix = self._attention(L, h, cache) if L.kind == "full_attention" else self._gdn(L, h, cache, decode)
            h, res = add_rms_norm(mix, L.norm2, self.eps, residual=res)
            delta = self._proj(self._proj(h, L.fc12, EPI_SILU_MUL), L.fc3, EPI_PARTIAL, 8)
        h, res = add_rms_norm(delta, self.final_norm, self.eps, residual=res)
        hl = h[:, -1]
        # the 151,936-row head: the decode kernel at batch <= 8 (52 us against cuBLAS's 55 at batch 1),
        # cuBLAS above (55 us against 69 at batch 32)
        logits = self._proj(hl, self.head) if hl.shape[0] <= 8 else F.linear(hl, self.head)
        cache.pos.add_(T)  # after the head, so the norm -> head launches stay programmatically chained
        return logits

    def new_cache(self, batch: int) -> Qwen35Cache:
        return Qwen35Cache(self.cfg, batch, self.max_len, self.device)

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, cache: Qwen35Cache) -> torch.Tensor:
        """Run the prompt ``ids [B, T]`` (int64 on the device) into ``cache`` from position 0 (whatever it held
        before is replaced); logits ``[B, vocab]``."""
        check_device_errors(self.device)
        cache.pos.zero_()
        logits = self.forward(ids, cache, decode=False)
        cache.has_previous_state = True
        return logits

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, cache: Qwen35Cache) -> torch.Tensor:
        """One token per sequence (``tokens [B]``) through the recurrent path; logits ``[B, vocab]``."""
        if not cache.has_previous_state:
            raise RuntimeError("decode_step needs a prefilled cache")
        return self.forward(tokens.view(-1, 1), cache, decode=True)

    @torch.no_grad()
    def capture_decode(self, cache: Qwen35Cache):
        """Capture one greedy decode step over static buffers in a CUDA graph: replaying it reads the
        token in ``self.step_tokens [B]``, runs the step, and writes the greedy next token back there (and
        the step's logits to ``self.step_logits``), so successive replays decode without the host."""
        B = cache.batch
        self.step_tokens = torch.zeros(B, dtype=torch.int64, device=self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        saved = [(t, t.clone()) for t in self._cache_tensors(cache)]
        with torch.cuda.stream(stream):  # warm-up on the side stream (allocations, library set-up)
            for _ in range(2):
                self.decode_step(self.step_tokens, cache)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            self.step_logits = self.decode_step(self.step_tokens, cache)
            self.step_tokens.copy_(self.step_logits.argmax(-1))
        for t, s in saved:  # the warm-up and capture ran the step: put the cache back
            t.copy_(s)
        torch.cuda.synchronize(self.device)
        self._graph, self._graph_cache = graph, cache
        return graph

    @staticmethod
    def _cache_tensors(cache: Qwen35Cache):
        return (list(cache.conv_states.values()) + list(cache.recurrent_states.values())
                + list(cache.key_cache.values()) + list(cache.value_cache.values()) + [cache.pos])

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, steps: int, use_graph: bool = True,
                 cache: Optional[Qwen35Cache] = None, teacher: Optional[torch.Tensor] = None):
        """Greedy generation: the prompt ``ids [B, T0]``, then ``steps`` decode steps.  Returns
        ``(tokens [B, steps + 1], cache)``: tokens[:, 0] comes from the prefill's logits, tokens[:, i] from
        decode step i.  ``teacher [B, steps]`` feeds given tokens to the decode steps instead of the greedy
        ones (the returned tokens stay the greedy choices)."""
        B = ids.shape[0]
        if cache is None:
            cache = self.new_cache(B)
        if ids.shape[1] + steps > self.max_len:
            raise RuntimeError(f"prompt + steps ({ids.shape[1] + steps}) exceeds max_len {self.max_len}")
        out = torch.empty((B, steps + 1), dtype=torch.int64, device=self.device)
        logits = self.prefill(ids, cache)
        out[:, 0] = logits.argmax(-1)
        if use_graph and teacher is None:
            if self._graph is None or self._graph_cache is not cache:
                self.capture_decode(cache)
            self.step_tokens.copy_(out[:, 0])
            for i in range(steps):
                self._graph.replay()
                out[:, i + 1] = self.step_tokens
        else:
            tok = out[:, 0]
            for i in range(steps):
                feed = tok if teacher is None else teacher[:, i]
                logits = self.decode_step(feed, cache)
                tok = logits.argmax(-1)
                out[:, i + 1] = tok
        return out, cache


def parity_logits(decoder: Qwen35Decoder, ids: torch.Tensor, feed: torch.Tensor):
    """Teacher-forced logits ``[B, n + 1, vocab]`` (fp32): the prefill's last-position logits, then the logits
    of n decode steps fed ``feed [B, n]`` -- what the parity tests compare with the reference's model."""
    cache = decoder.new_cache(ids.shape[0])
    rows = [decoder.prefill(ids, cache).float()]
    for i in range(feed.shape[1]):
        rows.append(decoder.decode_step(feed[:, i], cache).float())
    return torch.stack(rows, 1)


def count_parameters(cfg: dict) -> int:
    return sum(math.prod(s) for _, s in parameter_shapes(cfg))
