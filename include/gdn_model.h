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

/* Every kernel below is launched with programmatic stream serialization (programmatic dependent launch):
 * the next kernel in the stream may be scheduled while the previous one runs and read its weights, but
 * waits for the previous grid to complete before it reads anything else or writes (griddepcontrol.wait), so
 * results do not depend on it.  In a captured decode step this overlaps each kernel's launch and weight
 * prefetch with the tail of the one before.  enable = 0 launches them plainly (for comparison). */
GDN_API void gdn_model_set_programmatic_launch(int enable);

/* out = RMSNorm(h) with h = x (+ residual): h * rsqrt(mean(h^2) + eps) * (1 + weight) in fp32, rounded to
 * bf16 (qwen3_5.py:49-63).  x, out [N, D] (D a multiple of 8, at most 8192); weight [D].  With `residual`
 * non-NULL, h = bf16(x + residual) (the block's `x = x + shortcut`, qwen3_5.py:231, :236) and h is written
 * to `residual_out` (which may alias x or residual). */
GDN_API int gdn_model_add_rms_norm(const gdn_tensor* x, const gdn_tensor* residual, const gdn_tensor* weight, float eps,
                                   gdn_tensor* out, gdn_tensor* residual_out, void* stream);

/* gdn_model_add_rms_norm with x given as the fp32 partial sums of a split-K projection
 * (gdn_model_linear, GDN_MODEL_EPI_PARTIAL): x = bf16(sum over the nsplit planes [nsplit][rows][dim], in
 * plane order), the bf16 output the reference's Linear rounds to. */
GDN_API int gdn_model_add_rms_norm_partials(const float* partial, int nsplit, int64_t rows, int64_t dim,
                                            const gdn_tensor* residual, const gdn_tensor* weight, float eps,
                                            gdn_tensor* out, gdn_tensor* residual_out, void* stream);

/* A decode-step projection, out = x W^T (the reference's bias-free bf16 nn.Linear, qwen3_5.py:38-40,
 * :131-134; qwen3_5_transformers.py:252-300), for x [M, K] with M <= 32 (the decode batch; prefill
 * projections use a library GEMM) and W [N, K] read once: W's rows stream through the tensor cores
 * (mma.sync m16n8k16) with K split over the warps of a CTA; N a multiple of 16, K of 64.  epilogue:
 *   GDN_MODEL_EPI_STORE     out [M, N] bf16;
 *   GDN_MODEL_EPI_SILU_MUL  W holds fc1 and fc2 interleaved in row groups of 8 (rows 16j..16j+7 = fc1 rows
 *                           8j..8j+7, rows 16j+8..16j+15 = fc2 rows 8j..8j+7): out [M, N/2] =
 *                           SiLU(fc1 x) * (fc2 x), rounded as FeedForward rounds it (qwen3_5.py:42-46);
 *   GDN_MODEL_EPI_PARTIAL   K split over `ksplit` CTAs, fp32 partial sums into partial [ksplit][M][N]
 *                           (consumed by gdn_model_add_rms_norm_partials); out unused. */
#define GDN_MODEL_EPI_STORE 0
#define GDN_MODEL_EPI_SILU_MUL 1
#define GDN_MODEL_EPI_PARTIAL 2
GDN_API int gdn_model_linear(const gdn_tensor* x, const gdn_tensor* w, gdn_tensor* out, float* partial, int ksplit,
                             int epilogue, void* stream);

/* One decode token of a GatedDeltaNet layer after its input projection, fused: the conv update
 * (torch_causal_conv1d_update, qwen3_5_transformers.py:85-101), the gates (:377-379), the recurrent rule with
 * q/k l2-normalised (:190-229, :396-410) on the cached state, and the gated RMS norm with z (:56-71, :413-415).
 *   proj        [B, 3*H*128 + H*128 + 2H]: the layer's fused input projection row (mixed q|k|v, z, b, a)
 *   conv_state  [B, 3*H*128, 4] updated in place;  conv_w [3*H*128, 4];  A_log, dt_bias [H]
 *   state       fp32 [B, H, 128, 128] updated in place;  norm_w [128]
 *   out         [B, H*128]: the normed output (the input of out_proj)
 * The same roundings as the separate gdn_causal_conv1d_update, gdn_gates, gdn_recurrent_gated_delta_rule and
 * gdn_rms_norm_gated calls; equal key and value head counts (Qwen3.5: 16 / 16).
 *   prefetch_state  nonzero: the caller guarantees that no kernel that may still be running when this one
 *                   starts writes `state` (in a decode step the state is written only by this layer's call
 *                   of the previous step, and a plainly launched kernel -- the step's embedding -- lies in
 *                   between), so the kernel starts loading it before the kernel launched just before it
 *                   completes.  0: it waits for that kernel first, like every other input. */
GDN_API int gdn_model_gdn_decode(const gdn_tensor* proj, gdn_tensor* conv_state, const gdn_tensor* conv_w,
                                 const gdn_tensor* A_log, const gdn_tensor* dt_bias, float* state,
                                 const gdn_tensor* norm_w, float eps, gdn_tensor* out, int prefetch_state,
                                 void* stream);

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
