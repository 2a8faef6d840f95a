// Kernels of the Qwen3.5-shaped decoder that drives the GatedDeltaNet path
// (include/gdn_model.h): the residual add + RMSNorm, the full-attention
// prologue (q/k RMSNorm, partial RoPE, KV-cache append), causal attention over
// the cache with the sigmoid output gate, and the FFN's SiLU(fc1) * fc2.  The
// projections themselves are plain GEMMs (cuBLAS through torch).
//
// All operands are bf16 rows handled 8 elements (16 bytes) per lane; sums run
// in fp32 and each result is rounded to bf16 where the reference's bf16 torch
// ops round it (qwen3_5.py:35-183).  These kernels are small and latency-bound
// at decode sizes (a few MB per call): one CTA per row / per (token, head), no
// shared state between CTAs, every index bounded by the shapes checked on the
// host.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "../../include/gdn_model.h"
#include "gdn_internal.h"

namespace gdn {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void load8(const bf16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void store8(bf16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

// --------------------------------------------------------------------------- residual add + RMSNorm

struct AddNormArgs {
    const bf16* x;
    int64_t x_s;
    const bf16* r;  // residual or null
    int64_t r_s;
    const bf16* w;
    bf16* out;
    int64_t o_s;
    bf16* ro;       // residual_out (with r)
    int64_t ro_s;
    int D;
    float eps;
};

// One CTA per row, D / 8 threads (a multiple of 32), 8 elements a thread.
__global__ void __launch_bounds__(1024) gdn_model_add_rms_norm_kernel(AddNormArgs a) {
    __shared__ float part[32];
    const int64_t row = blockIdx.x;
    const int c = threadIdx.x * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    float h[8];
    load8(a.x + row * a.x_s + c, h);
    if (a.r) {
        float r[8];
        load8(a.r + row * a.r_s + c, r);
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = rbf(h[i] + r[i]);
        store8(a.ro + row * a.ro_s + c, h);  // this thread's elements were read above (aliasing is safe)
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(h[i], h[i], ss);
    ss = warp_sum(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float v = lane < nwarps ? part[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) part[0] = v;
    }
    __syncthreads();
    const float inv = rsqrtf(part[0] / (float)a.D + a.eps);
    float w[8], o[8];
    load8(a.w + c, w);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(h[i], inv), 1.0f + w[i]);
    store8(a.out + row * a.o_s + c, o);
}

// --------------------------------------------------------------------------- attention prologue

constexpr int kDh = 256;  // head_dim of Qwen3.5's full-attention layers

struct PrepArgs {
    const bf16* qkv;
    int64_t q_sb, q_st;
    const bf16* qn;
    const bf16* kn;
    const float* cos;
    const float* sin;
    int rope_dim;
    const int* pos;
    float eps;
    bf16* q_out;
    int64_t o_sb, o_st, o_sh;
    bf16* kc;
    int64_t kc_sb, kc_sh, kc_sp;
    bf16* vc;
    int64_t vc_sb, vc_sh, vc_sp;
    int Hq, Hkv, L;
};

// grid (T, B); warp w < Hq: query head w; then Hkv key heads, then Hkv value heads.  Lane l holds dims
// 8l .. 8l+7; the RoPE partner of dim d < rope_dim/2 is d + rope_dim/2, rope_dim/16 lanes away.
__global__ void __launch_bounds__(1024) gdn_model_attn_prep_kernel(PrepArgs a) {
    const int t = blockIdx.x, b = blockIdx.y;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = a.pos[0] + t;
    if (p < 0 || p >= a.L) return;
    const bf16* tok = a.qkv + (int64_t)b * a.q_sb + (int64_t)t * a.q_st;
    const bf16* src;
    const bf16* nw;
    bf16* dst;
    if (w < a.Hq) {
        src = tok + (int64_t)w * 2 * kDh;
        nw = a.qn;
        dst = a.q_out + (int64_t)b * a.o_sb + (int64_t)t * a.o_st + (int64_t)w * a.o_sh;
    } else if (w < a.Hq + a.Hkv) {
        const int kh = w - a.Hq;
        src = tok + (int64_t)a.Hq * 2 * kDh + (int64_t)kh * kDh;
        nw = a.kn;
        dst = a.kc + (int64_t)b * a.kc_sb + (int64_t)kh * a.kc_sh + (int64_t)p * a.kc_sp;
    } else {
        const int vh = w - a.Hq - a.Hkv;
        src = tok + (int64_t)a.Hq * 2 * kDh + (int64_t)(a.Hkv + vh) * kDh;
        dst = a.vc + (int64_t)b * a.vc_sb + (int64_t)vh * a.vc_sh + (int64_t)p * a.vc_sp;
        *reinterpret_cast<uint4*>(dst + 8 * lane) = *reinterpret_cast<const uint4*>(src + 8 * lane);
        return;
    }
    float x[8], g[8];
    load8(src + 8 * lane, x);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)kDh + a.eps);
    load8(nw + 8 * lane, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = rbf(__fmul_rn(__fmul_rn(x[i], inv), 1.0f + g[i]));  // RMSNorm -> bf16
    const int half_lanes = a.rope_dim / 16;
    float partner[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], half_lanes);
    if (8 * lane < a.rope_dim) {
        const bool first = 8 * lane < a.rope_dim / 2;
        const float* cr = a.cos + (int64_t)p * a.rope_dim + 8 * lane;
        const float* sr = a.sin + (int64_t)p * a.rope_dim + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float rot = first ? -partner[i] : partner[i];
            x[i] = __fadd_rn(__fmul_rn(x[i], cr[i]), __fmul_rn(rot, sr[i]));
        }
    }
    store8(dst + 8 * lane, x);
}

// --------------------------------------------------------------------------- attention

struct AttnArgs {
    const bf16* q;
    int64_t q_sb, q_st, q_sh;
    const bf16* kc;
    int64_t kc_sb, kc_sh, kc_sp;
    const bf16* vc;
    int64_t vc_sb, vc_sh, vc_sp;
    const bf16* gate;
    int64_t g_sb, g_st, g_sh;
    const int* pos;
    bf16* out;
    int64_t o_sb, o_st;
    int Hq, Hkv, L;
    float scale;
};

constexpr int kAttnWarps = 4;

__device__ __forceinline__ float block_reduce4(float v, float* buf, bool is_max) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = is_max ? warp_max(v) : warp_sum(v);
    if (lane == 0) buf[warp] = v;
    __syncthreads();
    float r = buf[0];
#pragma unroll
    for (int i = 1; i < kAttnWarps; ++i) r = is_max ? fmaxf(r, buf[i]) : r + buf[i];
    __syncthreads();
    return r;
}

// grid (T, Hq, B), 4 warps.  Scores: warp w takes keys w, w+4, ...; each key is a warp-wide dot product
// (8 dims a lane).  Weights: softmax over smem.  Context: the same key split, each warp accumulating
// its keys' weighted values, then the four partial rows summed in smem.
__global__ void __launch_bounds__(kAttnWarps * 32) gdn_model_attention_kernel(AttnArgs a) {
    extern __shared__ float sm[];
    float* sc = sm;                       // [L] scores, then weights
    float* red = sm + a.L;                // [4][256] partial contexts
    float* buf = red + kAttnWarps * kDh;  // [4] reduction scratch
    const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kh = h / (a.Hq / a.Hkv);
    int p = a.pos[0] + t;
    if (p >= a.L) p = a.L - 1;
    if (p < 0) p = 0;
    float q[8];
    load8(a.q + (int64_t)b * a.q_sb + (int64_t)t * a.q_st + (int64_t)h * a.q_sh + 8 * lane, q);
    const bf16* kbase = a.kc + (int64_t)b * a.kc_sb + (int64_t)kh * a.kc_sh + 8 * lane;
    const bf16* vbase = a.vc + (int64_t)b * a.vc_sb + (int64_t)kh * a.vc_sh + 8 * lane;
    for (int j = warp; j <= p; j += kAttnWarps) {
        float k[8];
        load8(kbase + (int64_t)j * a.kc_sp, k);
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(q[i], k[i], d);
        d = warp_sum(d);
        if (lane == 0) sc[j] = rbf(rbf(d) * a.scale);  // bf16 scores, scaled in bf16
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) m = fmaxf(m, sc[j]);
    m = block_reduce4(m, buf, true);
    float s = 0.f;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) s += expf(sc[j] - m);
    s = block_reduce4(s, buf, false);
    const float inv_s = 1.0f / s;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) sc[j] = rbf(expf(sc[j] - m) * inv_s);  // fp32 softmax -> bf16
    __syncthreads();
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = warp; j <= p; j += kAttnWarps) {
        float v[8];
        load8(vbase + (int64_t)j * a.vc_sp, v);
        const float wj = sc[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(wj, v[i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * kDh + 8 * lane + i] = acc[i];
    __syncthreads();
    const bf16* grow = a.gate + (int64_t)b * a.g_sb + (int64_t)t * a.g_st + (int64_t)h * a.g_sh;
    bf16* orow = a.out + (int64_t)b * a.o_sb + (int64_t)t * a.o_st + (int64_t)h * kDh;
    for (int d = threadIdx.x; d < kDh; d += blockDim.x) {
        float c = red[d];
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) c += red[w * kDh + d];
        c = rbf(c);
        const float gt = __bfloat162float(grow[d]);
        const float sg = rbf(1.0f / (1.0f + expf(-gt)));
        orow[d] = __float2bfloat16_rn(c * sg);
    }
}

// --------------------------------------------------------------------------- SiLU(fc1) * fc2

struct SiluArgs {
    const bf16* x;
    int64_t x_s;
    bf16* out;
    int64_t o_s;
    int64_t N;
    int F;
};

__global__ void __launch_bounds__(256) gdn_model_silu_mul_kernel(SiluArgs a) {
    const int per_row = a.F / 8;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= a.N * per_row) return;
    const int64_t row = idx / per_row;
    const int c = (int)(idx % per_row) * 8;
    float u[8], g[8], o[8];
    load8(a.x + row * a.x_s + c, u);
    load8(a.x + row * a.x_s + a.F + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = rbf(u[i] / (1.0f + expf(-u[i]))) * g[i];
    store8(a.out + row * a.o_s + c, o);
}

// --------------------------------------------------------------------------- host side

int bad(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
int bad(const char* fmt, ...) {
    char msg[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    return set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s", msg);
}

// A bf16 view of `ndim` dims (shape checked against want, -1 = any) whose base and every stride but the last
// are 16-byte multiples and whose last dim is contiguous.
int view(const char* name, const gdn_tensor* t, int ndim, const int64_t* want) {
    if (!t) return bad("%s is NULL", name);
    if (t->ndim != ndim) return bad("%s must be %d-D, got ndim=%d", name, ndim, t->ndim);
    if (t->dtype != GDN_BF16) return set_last_error(GDN_ERR_UNSUPPORTED, "%s must be bf16", name);
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) {
        if (t->shape[i] < 0) return bad("%s has a negative dimension", name);
        if (want && want[i] >= 0 && t->shape[i] != want[i])
            return bad("%s: dim %d is %lld, expected %lld", name, i, (long long)t->shape[i], (long long)want[i]);
        n *= t->shape[i];
    }
    if (t->stride[ndim - 1] != 1) return bad("%s: the last dimension must be contiguous", name);
    if (n > 0 && !t->data) return bad("%s has a NULL data pointer", name);
    if (reinterpret_cast<uintptr_t>(t->data) & 15) return bad("%s must be 16-byte aligned", name);
    for (int i = 0; i < ndim - 1; ++i)
        if (t->stride[i] % 8) return bad("%s: strides must be multiples of 8 elements", name);
    return GDN_OK;
}

int launched(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        return set_last_error(GDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    note_launch();
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" {

int gdn_model_add_rms_norm(const gdn_tensor* x, const gdn_tensor* residual, const gdn_tensor* weight, float eps,
                           gdn_tensor* out, gdn_tensor* residual_out, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("x", x, 2, nullptr))) return rc;
    const int64_t N = x->shape[0], D = x->shape[1];
    if (D % 256 || D > 8192) return bad("the row length must be a multiple of 256 and at most 8192, got %lld", (long long)D);
    const int64_t shp[2] = {N, D}, wshp[1] = {D};
    if ((rc = view("weight", weight, 1, wshp)) || (rc = view("out", out, 2, shp))) return rc;
    if (residual) {
        if ((rc = view("residual", residual, 2, shp))) return rc;
        if (!residual_out) return bad("residual_out is NULL");
        if ((rc = view("residual_out", residual_out, 2, shp))) return rc;
    }
    if (!(eps >= 0.f)) return bad("eps must be >= 0");
    if (N > 0x7fffffffLL) return bad("too many rows");
    if (N == 0) return GDN_OK;
    AddNormArgs a{reinterpret_cast<const bf16*>(x->data), x->stride[0],
                  residual ? reinterpret_cast<const bf16*>(residual->data) : nullptr, residual ? residual->stride[0] : 0,
                  reinterpret_cast<const bf16*>(weight->data), reinterpret_cast<bf16*>(out->data), out->stride[0],
                  residual ? reinterpret_cast<bf16*>(residual_out->data) : nullptr,
                  residual ? residual_out->stride[0] : 0, (int)D, eps};
    gdn_model_add_rms_norm_kernel<<<(unsigned)N, (unsigned)(D / 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return launched(cudaGetLastError(), "add_rms_norm launch");
}

int gdn_model_attn_prep(const gdn_tensor* qkv, const gdn_tensor* q_norm_w, const gdn_tensor* k_norm_w,
                        const float* rope_cos, const float* rope_sin, int rope_dim, const int32_t* pos, float eps,
                        gdn_tensor* q_out, gdn_tensor* k_cache, gdn_tensor* v_cache, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("q_out", q_out, 4, nullptr))) return rc;
    const int64_t B = q_out->shape[0], T = q_out->shape[1], Hq = q_out->shape[2];
    if (q_out->shape[3] != kDh) return bad("head_dim must be %d, got %lld", kDh, (long long)q_out->shape[3]);
    if ((rc = view("k_cache", k_cache, 4, nullptr))) return rc;
    const int64_t Hkv = k_cache->shape[1], L = k_cache->shape[2];
    const int64_t cshp[4] = {B, Hkv, L, kDh};
    if ((rc = view("k_cache", k_cache, 4, cshp)) || (rc = view("v_cache", v_cache, 4, cshp))) return rc;
    if (Hkv <= 0 || Hq % Hkv || Hq + 2 * Hkv > 32) return bad("need Hq a multiple of Hkv and Hq + 2 Hkv <= 32");
    const int64_t qshp[3] = {B, T, (Hq * 2 + Hkv * 2) * kDh};
    const int64_t nshp[1] = {kDh};
    if ((rc = view("qkv", qkv, 3, qshp)) || (rc = view("q_norm_w", q_norm_w, 1, nshp)) ||
        (rc = view("k_norm_w", k_norm_w, 1, nshp)))
        return rc;
    if (rope_dim != 16 && rope_dim != 32 && rope_dim != 64 && rope_dim != 128 && rope_dim != 256)
        return bad("rope_dim must be 16, 32, 64, 128 or 256, got %d", rope_dim);
    if (!rope_cos || !rope_sin || !pos) return bad("rope tables and pos must be device pointers");
    if (!(eps >= 0.f)) return bad("eps must be >= 0");
    if (B > 65535 || T > 0x7fffffffLL || L > 0x7fffffffLL) return bad("B must be <= 65535");
    if (B * T == 0) return GDN_OK;
    PrepArgs a{reinterpret_cast<const bf16*>(qkv->data), qkv->stride[0], qkv->stride[1],
               reinterpret_cast<const bf16*>(q_norm_w->data), reinterpret_cast<const bf16*>(k_norm_w->data),
               rope_cos, rope_sin, rope_dim, pos, eps, reinterpret_cast<bf16*>(q_out->data), q_out->stride[0],
               q_out->stride[1], q_out->stride[2], reinterpret_cast<bf16*>(k_cache->data), k_cache->stride[0],
               k_cache->stride[1], k_cache->stride[2], reinterpret_cast<bf16*>(v_cache->data), v_cache->stride[0],
               v_cache->stride[1], v_cache->stride[2], (int)Hq, (int)Hkv, (int)L};
    gdn_model_attn_prep_kernel<<<dim3((unsigned)T, (unsigned)B), (unsigned)(32 * (Hq + 2 * Hkv)), 0,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return launched(cudaGetLastError(), "attn_prep launch");
}

int gdn_model_attention(const gdn_tensor* q, const gdn_tensor* k_cache, const gdn_tensor* v_cache,
                        const gdn_tensor* gate, const int32_t* pos, gdn_tensor* out, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("q", q, 4, nullptr))) return rc;
    const int64_t B = q->shape[0], T = q->shape[1], Hq = q->shape[2];
    if (q->shape[3] != kDh) return bad("head_dim must be %d, got %lld", kDh, (long long)q->shape[3]);
    if ((rc = view("k_cache", k_cache, 4, nullptr))) return rc;
    const int64_t Hkv = k_cache->shape[1], L = k_cache->shape[2];
    const int64_t cshp[4] = {B, Hkv, L, kDh};
    if ((rc = view("k_cache", k_cache, 4, cshp)) || (rc = view("v_cache", v_cache, 4, cshp))) return rc;
    if (Hkv <= 0 || Hq % Hkv) return bad("Hq must be a multiple of Hkv");
    if (L <= 0 || L > 16384) return bad("the cache length must be in [1, 16384], got %lld", (long long)L);
    const int64_t gshp[4] = {B, T, Hq, kDh};
    const int64_t oshp[3] = {B, T, Hq * kDh};
    if ((rc = view("gate", gate, 4, gshp)) || (rc = view("out", out, 3, oshp))) return rc;
    if (!pos) return bad("pos must be a device pointer");
    if (B > 65535 || Hq > 65535 || T > 0x7fffffffLL) return bad("B and Hq must be <= 65535");
    if (B * T == 0) return GDN_OK;
    AttnArgs a{reinterpret_cast<const bf16*>(q->data), q->stride[0], q->stride[1], q->stride[2],
               reinterpret_cast<const bf16*>(k_cache->data), k_cache->stride[0], k_cache->stride[1],
               k_cache->stride[2], reinterpret_cast<const bf16*>(v_cache->data), v_cache->stride[0],
               v_cache->stride[1], v_cache->stride[2], reinterpret_cast<const bf16*>(gate->data), gate->stride[0],
               gate->stride[1], gate->stride[2], pos, reinterpret_cast<bf16*>(out->data), out->stride[0],
               out->stride[1], (int)Hq, (int)Hkv, (int)L, (float)(1.0 / sqrt((double)kDh))};
    const size_t smem = ((size_t)L + kAttnWarps * kDh + kAttnWarps) * sizeof(float);
    if (smem > 48 * 1024) {  // above the default limit only (short caches need no attribute call)
        cudaError_t e = cudaFuncSetAttribute(gdn_model_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return launched(e, "attention attribute");
    }
    gdn_model_attention_kernel<<<dim3((unsigned)T, (unsigned)Hq, (unsigned)B), kAttnWarps * 32, smem,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return launched(cudaGetLastError(), "attention launch");
}

int gdn_model_silu_mul(const gdn_tensor* x, gdn_tensor* out, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("x", x, 2, nullptr))) return rc;
    const int64_t N = x->shape[0], F2 = x->shape[1];
    if (F2 % 16) return bad("x must be [N, 2F] with F a multiple of 8, got width %lld", (long long)F2);
    const int64_t oshp[2] = {N, F2 / 2};
    if ((rc = view("out", out, 2, oshp))) return rc;
    const int64_t work = N * (F2 / 16);
    if (work == 0) return GDN_OK;
    if (work > (int64_t)0x7fffffff * 256) return bad("x too large");
    SiluArgs a{reinterpret_cast<const bf16*>(x->data), x->stride[0], reinterpret_cast<bf16*>(out->data),
               out->stride[0], N, (int)(F2 / 2)};
    gdn_model_silu_mul_kernel<<<(unsigned)((work + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return launched(cudaGetLastError(), "silu_mul launch");
}

}  // extern "C"
