/*
 * gdn_model.h - kernels of the Qwen3.5-shaped decoder that drives the
 * GatedDeltaNet path end to end (prefill through the chunked rule, then
 * token-by-token decode through the recurrent rule with cached states).
 *
 * The reference's model (qwen3_5.py) has no cache: its generation loop
 * re-runs the whole prefix for every new token (qwen3_5.py:483-495,
 * benchmark.py:318-335), and its full-attention layer is plain torch ops
 * (qwen3_5.py:145-183).  These entry points are the steps of that model the
 * GatedDeltaNet kernels of gdn_b200.h do not already cover, written for a
 * decoder that keeps a KV cache for the full-attention layers:
 *
 *   gdn_model_add_rms_norm  TransformerBlock's residual add and RMSNorm
 *                           (qwen3_5.py:224-237, :49-63)
 *   gdn_model_attn_prep     q/k RMSNorm, partial RoPE and the KV-cache append
 *                           (qwen3_5.py:148-166, :66-114)
 *   gdn_model_attention     causal softmax attention over the cache and the
 *                           sigmoid output gate (qwen3_5.py:167-183)
 *   gdn_model_silu_mul      FeedForward's SiLU(fc1) * fc2 (qwen3_5.py:42-46)
 *
 * All tensors are bf16 device memory (the model dtype), views with a
 * contiguous last dimension; calls are asynchronous on `stream`, allocate
 * nothing, and return a gdn_status (gdn_last_error() has the message).
 * Results are rounded to bf16 where the reference's bf16 torch ops round them.
 */
#ifndef GDN_MODEL_H
#define GDN_MODEL_H

#include "gdn_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out = RMSNorm(h) with h = x (+ residual): h * rsqrt(mean(h^2) + eps) * (1 + weight) in fp32, rounded to
 * bf16 (qwen3_5.py:49-63).  x, out [N, D] (D a multiple of 8, at most 8192); weight [D].  With `residual`
 * non-NULL, h = bf16(x + residual) (the block's `x = x + shortcut`, qwen3_5.py:231, :236) and h is written
 * to `residual_out` (which may alias x or residual). */
GDN_API int gdn_model_add_rms_norm(const gdn_tensor* x, const gdn_tensor* residual, const gdn_tensor* weight, float eps,
                                   gdn_tensor* out, gdn_tensor* residual_out, void* stream);

/* Full-attention prologue for T new tokens at positions pos[0] .. pos[0] + T - 1 (pos: one device int32, so
 * a captured decode step can advance it): from the fused projection qkv [B, T, Hq*2*Dh + 2*Hkv*Dh] (per
 * token: Hq blocks of [query Dh | gate Dh] (qwen3_5.py:148-151), then Hkv keys, then Hkv values),
 *   q_out [B, T, Hq, Dh]   = RoPE(RMSNorm_q(query))
 *   k_cache[b, h, p, :]    = RoPE(RMSNorm_k(key)),   v_cache[b, h, p, :] = value
 * RMSNorm as in gdn_model_add_rms_norm with q_norm_w / k_norm_w [Dh]; RoPE rotates the first rope_dim dims
 * with the tables rope_cos / rope_sin [max_len, rope_dim] fp32 (qwen3_5.py:66-114).  Caches are
 * [B, Hkv, max_len, Dh]; positions at or past max_len are not written. */
GDN_API int gdn_model_attn_prep(const gdn_tensor* qkv, const gdn_tensor* q_norm_w, const gdn_tensor* k_norm_w,
                                const float* rope_cos, const float* rope_sin, int rope_dim, const int32_t* pos,
                                float eps, gdn_tensor* q_out, gdn_tensor* k_cache, gdn_tensor* v_cache,
                                void* stream);

/* Causal attention of the T new queries q [B, T, Hq, Dh] over the cache (query t sees positions
 * 0 .. pos[0] + t; Hq / Hkv query heads share a KV head), softmax(q k^T / sqrt(Dh)) v, then times
 * sigmoid(gate) (gate [B, T, Hq, Dh], a view of the projection): out [B, T, Hq * Dh].  The score, the
 * softmax weights, the context and the gated output are rounded to bf16 as the reference's bf16 ops round
 * them (qwen3_5.py:171-182).  max_len (the cache length) is at most 16384. */
GDN_API int gdn_model_attention(const gdn_tensor* q, const gdn_tensor* k_cache, const gdn_tensor* v_cache,
                                const gdn_tensor* gate, const int32_t* pos, gdn_tensor* out, void* stream);

/* out = bf16(bf16(SiLU(x[:, :F])) * x[:, F:]) for x [N, 2F] (the fused fc1 | fc2 projection), out [N, F]
 * (qwen3_5.py:42-46); F a multiple of 8. */
GDN_API int gdn_model_silu_mul(const gdn_tensor* x, gdn_tensor* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_MODEL_H */
