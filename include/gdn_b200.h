/*
 * gdn_b200.h - C ABI of the B200 (sm_100a) GatedDeltaNet kernels.
 *
 * The reference (pbanavara/llms_from_scratch) exposes this path as two Python
 * callables; every entry point below names the reference interface it replaces:
 *
 *   fast_chunk_gated_delta_rule      qwen3_5_cutedsl_kernels.py:462-473
 *   torch_chunk_gated_delta_rule     qwen3_5_transformers.py:110-120
 *   torch_recurrent_gated_delta_rule qwen3_5_transformers.py:190-192
 * and the layer steps on either side of the rule (Qwen3_5GatedDeltaNet.forward):
 *   prefill conv1d + SiLU            qwen3_5_transformers.py:346-356
 *   torch_causal_conv1d_update       qwen3_5_transformers.py:85-101
 *   gates g, beta                    qwen3_5_transformers.py:377-379
 *   Qwen3_5RMSNormGated              qwen3_5_transformers.py:56-71
 *
 * Conventions (same as the reference):
 *   query, key   [B, T, H, Dk]      value, out  [B, T, H, Dv]
 *   g, beta      [B, T, H]          g is the per-token log-decay (not cumsummed)
 *   states       [B, H, Dk, Dv]     float32, row-major, contiguous
 * `out` has query's dtype.  Dk = Dv = 128 and chunk_size = 64 are required.
 * Tensors may be strided in B, T and H; the innermost (head) dimension must be
 * contiguous.  All calls are asynchronous on `stream` (a cudaStream_t; NULL is
 * the legacy default stream) and allocate no device memory: the chunked
 * forward takes a caller-owned workspace of gdn_chunk_workspace_bytes() bytes.
 *
 * Every function returns a gdn_status; gdn_last_error() gives a message for
 * the most recent failure on the calling host thread.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_ABI_VERSION 1

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

typedef enum {
    GDN_OK = 0,
    GDN_ERR_INVALID_ARGUMENT = 1, /* shape, stride, dtype or flag not supported (Python: ValueError) */
    GDN_ERR_UNSUPPORTED = 2,      /* valid request this build cannot run (Python: RuntimeError)    */
    GDN_ERR_WORKSPACE = 3,        /* workspace missing, too small or misaligned                    */
    GDN_ERR_CUDA = 4,             /* a CUDA runtime call or kernel launch failed                   */
    GDN_ERR_DEVICE = 5,           /* the current device is not an sm_100 GPU                       */
    GDN_ERR_KERNEL = 6            /* a kernel reported a failure in the device error word; the
                                     outputs of the call that set it are not valid                  */
} gdn_status;

typedef enum { GDN_F32 = 0, GDN_BF16 = 1, GDN_F16 = 2 } gdn_dtype;

/* A strided view of device memory (host memory for gdn_chunk_gated_delta_rule_host).
 * Unused trailing dims have size 1. */
typedef struct {
    void* data;        /* device pointer                                   */
    int32_t dtype;     /* gdn_dtype                                        */
    int32_t ndim;      /* 3 for g/beta, 4 for q/k/v/out                     */
    int64_t shape[4];
    int64_t stride[4]; /* in elements                                      */
} gdn_tensor;

/* Chunked gated delta rule forward (prefill).
 *
 * Replaces fast_chunk_gated_delta_rule(query, key, value, g, beta, chunk_size,
 * initial_state, output_final_state, use_qk_l2norm_in_kernel)
 * (qwen3_5_cutedsl_kernels.py:462-473) and its oracle
 * torch_chunk_gated_delta_rule (qwen3_5_transformers.py:110-187).
 *   initial_state  NULL for a zero state (qwen3_5_transformers.py:161-165)
 *   final_state    written when output_final_state != 0; may alias initial_state
 *   workspace      >= gdn_chunk_workspace_bytes(...) bytes, 256-byte aligned
 */
GDN_API int gdn_chunk_gated_delta_rule(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                               const gdn_tensor* g, const gdn_tensor* beta, int chunk_size,
                               const float* initial_state, int output_final_state,
                               int use_qk_l2norm_in_kernel, gdn_tensor* out, float* final_state,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes gdn_chunk_gated_delta_rule needs for this problem. */
GDN_API size_t gdn_chunk_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype);

/* Chunked forward for callers that cannot allocate device memory.
 *
 * No counterpart in the reference (its Python op allocates freely).  Same
 * arguments and results as gdn_chunk_gated_delta_rule, minus the workspace:
 * for callers that cannot call cudaMalloc when they run the op -- runtimes that
 * plan every device buffer ahead of time, plugins whose host framework owns all
 * allocations, code running while other components hold the free memory.
 * Scratch comes from a fixed array of GDN_NOALLOC_SCRATCH_BYTES (64 MiB)
 * compiled into the library, which every GPU that loads it holds until exit.
 *   - Problems whose workspace (gdn_chunk_workspace_bytes) exceeds that return
 *     GDN_ERR_WORKSPACE without launching anything.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current) and caches it; make that
 *     first call before any stream capture.
 *   - All calls share the array and it keeps the last call's contents; nothing
 *     in it needs to start at zero.  Calls that overlap on the GPU (other
 *     streams or host threads) race on it: order them on one stream.
 *   - Calls no cudaMalloc, cudaFree or other allocating routine. */
#define GDN_NOALLOC_SCRATCH_BYTES (64ull << 20)
GDN_API int gdn_chunk_gated_delta_rule_noalloc(const gdn_tensor* query, const gdn_tensor* key,
                                               const gdn_tensor* value, const gdn_tensor* g,
                                               const gdn_tensor* beta, int chunk_size,
                                               const float* initial_state, int output_final_state,
                                               int use_qk_l2norm_in_kernel, gdn_tensor* out,
                                               float* final_state, void* stream);

/* Chunked forward over HOST buffers, the copies overlapped with the compute.
 *
 * No counterpart in the reference: its op takes device tensors
 * (qwen3_5_cutedsl_kernels.py:462-473), so a caller holding host data copies
 * everything in, runs the op, and copies everything out, one after the other.
 * This call does the copies itself, cut into time slices of at most
 * `slice_tokens` (a multiple of chunk_size; 0 = about 12 MiB of q/k/v per
 * slice, e.g. 1024 tokens at B=1, H=16 bf16): slice s+1's inputs cross PCIe
 * while slice s computes and slice s-1's outputs come back, on two copy streams
 * of the library's own ordered against `stream` by events.
 *   query/key/value/g/beta/out  views of HOST memory, packed [B][T][H][D] and
 *               [B][T][H] (only the batch stride free; GDN_ERR_UNSUPPORTED
 *               otherwise); page-locked (cudaHostAlloc / cudaHostRegister) for
 *               the copies to overlap, pageable memory works but serialises.
 *   initial_state, final_state  host [B,H,Dk,Dv] fp32 or NULL, as in
 *               gdn_chunk_gated_delta_rule; may alias.
 *   workspace   DEVICE memory of gdn_chunk_host_workspace_bytes(...) bytes,
 *               256-byte aligned (sized for out in the query dtype and 4-byte
 *               g/beta: wider out or g/beta than that need more and get
 *               GDN_ERR_WORKSPACE).
 * Asynchronous like the device call: the results are in host memory once
 * `stream` has reached the end of this call's work.  The slices start on chunk
 * boundaries and carry the state in fp32, so the results equal one
 * gdn_chunk_gated_delta_rule call on the whole sequence. */
GDN_API int gdn_chunk_gated_delta_rule_host(const gdn_tensor* query, const gdn_tensor* key,
                                            const gdn_tensor* value, const gdn_tensor* g, const gdn_tensor* beta,
                                            int chunk_size, const float* initial_state, int output_final_state,
                                            int use_qk_l2norm_in_kernel, gdn_tensor* out, float* final_state,
                                            int64_t slice_tokens, void* workspace, size_t workspace_bytes,
                                            void* stream);

/* Device workspace bytes of gdn_chunk_gated_delta_rule_host (0 for an empty problem
 * or a slice_tokens that is negative or not a multiple of 64). */
GDN_API size_t gdn_chunk_host_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype,
                                              int64_t slice_tokens);

/* Packed variable-length sequences (prefill of a batch of prompts).
 *
 * The reference's op has no varlen form: its vLLM patch falls back to FLA when
 * cu_seqlens holds more than one sequence (vllm_inference.py:97-108).  This is
 * the interface vLLM's ChunkGatedDeltaRule hands to its kernels: q/k/v/g/beta
 * are [1, T, H, *] with sequence n at tokens [cu_seqlens[n], cu_seqlens[n+1]);
 * every sequence starts its own chunks, its own state (initial_state and
 * final_state [num_seqs,H,Dk,Dv] fp32, NULL = zeros / not written) and gives
 * exactly the results of a separate gdn_chunk_gated_delta_rule call on it.
 *   cu_seqlens  DEVICE int32 [num_seqs + 1], 0 = cu[0] <= cu[1] <= ... <= cu[num_seqs] = T;
 *               read on the device only (no host synchronisation).  Offsets that
 *               break this set device error bit 8 and no chunk is processed.
 *   workspace   >= gdn_chunk_varlen_workspace_bytes(T, num_seqs, ...) bytes, 256-byte aligned.
 * bf16 q/k/v/out with 16-byte aligned rows only (GDN_ERR_UNSUPPORTED otherwise). */
GDN_API int gdn_chunk_gated_delta_rule_varlen(const gdn_tensor* query, const gdn_tensor* key,
                                              const gdn_tensor* value, const gdn_tensor* g, const gdn_tensor* beta,
                                              const int32_t* cu_seqlens, int64_t num_seqs, int chunk_size,
                                              const float* initial_state, int output_final_state,
                                              int use_qk_l2norm_in_kernel, gdn_tensor* out, float* final_state,
                                              void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of gdn_chunk_gated_delta_rule_varlen (T = total tokens). */
GDN_API size_t gdn_chunk_varlen_workspace_bytes(int64_t T, int64_t num_seqs, int64_t H, int64_t Dk, int64_t Dv,
                                                int qkv_dtype);

/* Sequence parallelism: one long sequence split into contiguous time shards,
 * one shard per GPU.  No counterpart in the reference, which runs the chunk
 * loop on one device (qwen3_5_cutedsl_kernels.py:427-453); these two calls are
 * the per-shard halves of gdn_chunk_gated_delta_rule.
 *
 * The state at the end of a shard is an affine map of the state at its start,
 * S_end = transition @ S_start + local_state (transition [B,H,Dk,Dk], local_state
 * [B,H,Dk,Dv], fp32).  gdn_chunk_sp_summary computes both for this shard and
 * leaves its chunk records in `workspace`; after the shards' summaries are
 * exchanged and composed into this shard's start state, gdn_chunk_sp_finish
 * (same inputs, same untouched workspace) writes the shard's outputs and its
 * end state.  bf16 q/k/v/out with 16-byte aligned rows only (GDN_ERR_UNSUPPORTED
 * otherwise); T > 0. */
GDN_API int gdn_chunk_sp_summary(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                 const gdn_tensor* g, const gdn_tensor* beta, int chunk_size,
                                 int use_qk_l2norm_in_kernel, float* transition, float* local_state,
                                 void* workspace, size_t workspace_bytes, void* stream);
GDN_API int gdn_chunk_sp_finish(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                const gdn_tensor* g, const gdn_tensor* beta, int chunk_size,
                                const float* initial_state, int output_final_state, int use_qk_l2norm_in_kernel,
                                gdn_tensor* out, float* final_state, const void* workspace, size_t workspace_bytes,
                                void* stream);

/* Backward of gdn_chunk_gated_delta_rule (the reference is inference-only; these are the gradients
 * autograd takes through its torch forward, qwen3_5_transformers.py:110-187).  Given the forward's
 * inputs and the gradients of its outputs (d_out [B,T,H,Dv], any float dtype) and of its final state
 * (d_final_state [B,H,Dk,Dv] fp32, or NULL for none), writes dq, dk, dv [B,T,H,D] and dg, dbeta
 * [B,T,H] in their descriptors' dtypes and, if dh0 is not NULL, the gradient of the initial state
 * (fp32 [B,H,Dk,Dv]).  Forward recompute, a reverse state scan and three per-chunk kernels; with bf16
 * q/k/v/d_out (16-byte aligned rows) the recompute's state scan and the reverse scan run on the tensor
 * cores (bf16 operands, fp32 accumulation), otherwise everything runs in fp32 on CUDA cores.  The
 * workspace holds the recomputed forward and the chunk gradients.
 * Replaces: torch autograd through torch_chunk_gated_delta_rule (qwen3_5_transformers.py:110-187). */
GDN_API size_t gdn_chunk_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv,
                                             int qkv_dtype);
GDN_API int gdn_chunk_gated_delta_rule_bwd(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                           const gdn_tensor* g, const gdn_tensor* beta, const gdn_tensor* d_out,
                                           int chunk_size, const float* initial_state, const float* d_final_state,
                                           int use_qk_l2norm_in_kernel, gdn_tensor* dq, gdn_tensor* dk,
                                           gdn_tensor* dv, gdn_tensor* dg, gdn_tensor* dbeta, float* dh0,
                                           void* workspace, size_t workspace_bytes, void* stream);

/* Token-by-token recurrent rule (decode step when T == 1).
 *
 * Replaces torch_recurrent_gated_delta_rule(query, key, value, g, beta,
 * initial_state, output_final_state, use_qk_l2norm_in_kernel)
 * (qwen3_5_transformers.py:190-229).  final_state may alias initial_state
 * (in-place decode).  No workspace.
 */
GDN_API int gdn_recurrent_gated_delta_rule(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                   const gdn_tensor* g, const gdn_tensor* beta, const float* initial_state,
                                   int output_final_state, int use_qk_l2norm_in_kernel, gdn_tensor* out,
                                   float* final_state, void* stream);

/* GatedDeltaNet layer steps on either side of the rule (Qwen3_5GatedDeltaNet.forward,
 * qwen3_5_transformers.py:304-419).  Each result is rounded to the layer dtype
 * as the reference's bf16 torch ops round it.  Views are device memory with a
 * contiguous last dimension.
 *
 * gdn_causal_conv1d_silu replaces the prefill convolution
 * F.silu(self.conv1d(mixed_qkv)[:, :, :seq_len]) (:356; depthwise Conv1d with
 * kernel 4, padding 3, no bias, :253-260) and, when conv_state is non-NULL, the
 * cache's conv state F.pad(mixed_qkv, (4 - seq_len, 0)) (:346-348).
 *   x [B,T,C]  the in_proj_qkv output, token-major (the reference transposes it
 *              to [B,C,T], :334); out [B,T,C] must not alias x; both need
 *              16-byte aligned rows and C a multiple of 8 (bf16/fp16) or 4 (fp32)
 *   weight [C,4] (conv1d.weight.squeeze(1)); conv_state [B,C,4] or NULL.
 * q/k/v are then the channel ranges [0,Dk·H), [Dk·H, 2Dk·H), [2Dk·H, C) of out,
 * views the chunk entry points take as they are. */
GDN_API int gdn_causal_conv1d_silu(const gdn_tensor* x, const gdn_tensor* weight, gdn_tensor* out,
                                   gdn_tensor* conv_state, void* stream);

/* Decode convolution: replaces torch_causal_conv1d_update(x, conv_state, weight,
 * None, "silu") (:85-101).  x [B,T,C] (T new tokens, token-major), conv_state
 * [B,C,4] read and updated in place, weight [C,4], out [B,T,C]. */
GDN_API int gdn_causal_conv1d_update(const gdn_tensor* x, gdn_tensor* conv_state, const gdn_tensor* weight,
                                     gdn_tensor* out, void* stream);

/* Gates: replaces beta = b.sigmoid() and g = -A_log.float().exp() *
 * F.softplus(a.float() + dt_bias) (:377-379).  a, b, g, beta [B,T,H]; A_log,
 * dt_bias [H] (one dtype).  g is computed in fp32 and beta rounded to beta's
 * dtype (the reference keeps it in b's dtype). */
GDN_API int gdn_gates(const gdn_tensor* a, const gdn_tensor* b, const gdn_tensor* A_log, const gdn_tensor* dt_bias,
                      gdn_tensor* g, gdn_tensor* beta, void* stream);

/* Gated RMS norm: replaces Qwen3_5RMSNormGated.forward(x, gate) (:62-71) over rows
 * of 128 (head_v_dim).  x, gate, out [N,128], or [M,H,128] views (each with its
 * own strides: e.g. the gate z as a strided view of a wider projection, :331-332);
 * weight [128]; one dtype. */
GDN_API int gdn_rms_norm_gated(const gdn_tensor* x, const gdn_tensor* gate, const gdn_tensor* weight, float eps,
                               gdn_tensor* out, void* stream);

/* Instrumentation (no counterpart in the reference, which times whole calls
 * with CUDA events, benchmark.py:82-100).
 *
 * gdn_launch_count: number of kernels this library has launched in this
 * process (all devices, all threads).
 *
 * gdn_set_phase_events: when `events` is non-NULL, every later call on this
 * host thread records events[0] on its stream before its first kernel and
 * events[i] after its i-th kernel (i = 1..n-1 must cover the kernels of the
 * call: 2 for the chunked forward, 1 for the recurrent rule and each layer
 * step).  Entries are
 * cudaEvent_t handles.  Pass NULL to stop. */
GDN_API uint64_t gdn_launch_count(void);
GDN_API void gdn_set_phase_events(void* const* events, int n);

/* Sticky error bits of the current device.  A kernel whose bounded wait on an
 * internal barrier gives up (a bug, never expected) sets a bit here and exits
 * cleanly instead of hanging: 1 = chunk prep, 2 = chunk scan.  8 = packed
 * sequence offsets that were not a valid cu_seqlens.  16 = the wait of
 * gdn_selftest_bounded_wait.  The outputs of a call that set a bit are not
 * valid.  Synchronous (it copies the word from the device); `clear` != 0
 * resets the word and its host mirror.
 *
 * The library caches the device addresses of this word (and of the fixed
 * scratch of gdn_chunk_gated_delta_rule_noalloc) per device ordinal for the
 * life of the process: resetting a device (cudaDeviceReset, or a primary
 * context reset) after the first call on it is not supported. */
GDN_API unsigned int gdn_device_error(int clear);

/* The current device's error bits as the kernels mirror them into page-locked
 * host memory: reads host memory only (no synchronisation), so a caller can
 * check it before every call.  Reflects the kernels that have finished: a call
 * that failed on the device shows up here once its kernels have run (and
 * gdn_device_error(1) then returns and clears the bits).  The mirror is a page
 * of this library's host data, page-locked and mapped into each device by the
 * first call on that device that sets up the error word (the chunked forward
 * and its variants, the backward, the self-test below), which also writes the
 * mirror's address to the device with one synchronous copy: make that first
 * call before any stream capture.  Returns 0 before that call, or if the page
 * could not be page-locked.  No counterpart in the reference (its torch ops
 * raise synchronously). */
GDN_API unsigned int gdn_device_error_pending(void);

/* Test hook: launches one kernel on `stream` whose bounded wait on a barrier
 * that nothing arms runs out after timeout_ns (1e3 .. 1e8 ns); it then sets bit
 * 16 of the error word (and its mirror) and returns, exactly as a chunk kernel
 * whose wait gave up would.  Lets a caller check that a timed-out wait
 * surfaces as an error and leaves the context usable.  No counterpart in the
 * reference. */
GDN_API int gdn_selftest_bounded_wait(uint64_t timeout_ns, void* stream);

/* Message for the most recent failure on this host thread ("" if none). */
GDN_API const char* gdn_last_error(void);

/* Name of a gdn_status value. */
GDN_API const char* gdn_status_name(int status);

/* GDN_ABI_VERSION of the loaded library. */
GDN_API int gdn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
