// GatedDeltaNet layer steps on either side of the gated delta rule
// (Qwen3_5GatedDeltaNet.forward, qwen3_5_transformers.py:304-419):
//   * the prefill causal depthwise conv1d (kernel 4) + SiLU over the mixed q/k/v
//     projection, and the conv state the cache keeps (:346-356);
//   * the decode convolution against that state, torch_causal_conv1d_update (:85-101);
//   * the gates beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias) (:377-379);
//   * the gated RMS norm after the rule, Qwen3_5RMSNormGated (:56-71).
// All four are HBM-bound elementwise/row passes.  The convolutions read the
// projection in its token-major [B,T,C] layout (the reference transposes it to
// [B,C,T] for torch's conv1d, :334, and back, :358) and write the conv output in
// the same layout, so q/k/v are strided views of it that the chunk kernels take
// without a copy.  Each thread owns 16 bytes of channels (8 bf16) and walks a run
// of tokens with the three previous inputs in registers.
//
// Numerics follow the reference's bf16 ops, each result rounded to the layer
// dtype once: the conv sum (bf16 x bf16 products are exact in fp32, accumulated
// with FMAs in tap order), then SiLU in fp32; the norm's mean of squares in fp32,
// then the three roundings of Qwen3_5RMSNormGated.  SiLU and sigmoid use the
// fast exponential and division; against an exactly computed fp32 value that can
// move a bf16 rounding by one unit in rare cases (measured in the tests).
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kConvK = 4;          // linear_conv_kernel_dim of Qwen3.5
constexpr int kConvThreads = 128;  // channel groups per CTA
constexpr int kConvTokens = 8;     // tokens per thread (prefill), all their loads issued at once

struct ConvParams {
    const void* x;       // [B,T,C], channels contiguous
    int64_t x_sb, x_st;
    const void* w;       // [C,K], row stride w_sc
    int64_t w_sc;
    void* out;           // [B,T,C], channels contiguous
    int64_t o_sb, o_st;
    void* state;         // [B,C,K] conv state (prefill: written; update: read and written); may be null
    int64_t s_sb, s_sc;
    int B, C;
    int64_t T;
    int dtype;           // of x, w, out and state
};

template <typename E> struct Elem;
// Per-dtype load / store / round-to-dtype, with pair forms (one packed conversion for two values).
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float ld(const __nv_bfloat16& v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 st(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    static __device__ __forceinline__ void rnd2(float& a, float& b) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        a = __low2float(h);
        b = __high2float(h);
    }
    static __device__ __forceinline__ void st2(__nv_bfloat16* dst, float a, float b) {
        *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
    }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float ld(const __half& v) { return __half2float(v); }
    static __device__ __forceinline__ __half st(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ float rnd(float x) { return __half2float(__float2half_rn(x)); }
    static __device__ __forceinline__ void rnd2(float& a, float& b) {
        const __half2 h = __floats2half2_rn(a, b);
        a = __low2float(h);
        b = __high2float(h);
    }
    static __device__ __forceinline__ void st2(__half* dst, float a, float b) {
        *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(a, b);
    }
};
template <> struct Elem<float> {
    static __device__ __forceinline__ float ld(const float& v) { return v; }
    static __device__ __forceinline__ float st(float x) { return x; }
    static __device__ __forceinline__ float rnd(float x) { return x; }
    static __device__ __forceinline__ void rnd2(float&, float&) {}
    static __device__ __forceinline__ void st2(float* dst, float a, float b) {
        dst[0] = a;
        dst[1] = b;
    }
};

// x * sigmoid(x) in fp32 (F.silu computes in fp32 for 16-bit tensors), from e^-y = 2^(-y log2 e) and
// 1 / (1 + e^-y) on the hardware's approximate base-2 exponential and reciprocal.  For very negative y
// the denominator overflows to inf and the result is -0, the limit; inputs are finite.
__device__ __forceinline__ float silu_f32(float y) {
    constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-y * kLog2e));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return y * r;
}

// conv output of one channel: sum_j w_j x_j in tap order, rounded to the layer dtype, then SiLU
// rounded again (:356 / :97-98).
template <typename E>
__device__ __forceinline__ float conv_silu(const float (&w)[kConvK], float x0, float x1, float x2, float x3) {
    float acc = w[0] * x0;
    acc = fmaf(w[1], x1, acc);
    acc = fmaf(w[2], x2, acc);
    acc = fmaf(w[3], x3, acc);
    return Elem<E>::rnd(silu_f32(Elem<E>::rnd(acc)));
}

// Prefill: thread = V consecutive channels (8 bytes) x kConvTokens tokens.  The run's loads (and the
// three inputs before it: zero before t = 0, the conv's left padding) are all in flight before the
// first output; each input is converted to fp32 once and slides through a three-deep window.  A warp
// covers 32 x 8 contiguous bytes of channels per token.
template <typename E>
__global__ void __launch_bounds__(kConvThreads) gdn_conv_silu_kernel(ConvParams p) {
    constexpr int V = 8 / sizeof(E);
    using Vec = uint2;
    const int cg = blockIdx.x * kConvThreads + threadIdx.x;
    const int c0 = cg * V;
    if (c0 >= p.C) return;
    const int b = blockIdx.z;
    const int64_t t0 = (int64_t)blockIdx.y * kConvTokens;
    if (t0 >= p.T) return;

    const E* xb = reinterpret_cast<const E*>(p.x) + (int64_t)b * p.x_sb + c0;
    E* ob = reinterpret_cast<E*>(p.out) + (int64_t)b * p.o_sb + c0;
    constexpr int N = kConvTokens + kConvK - 1;  // inputs t0-3 .. t0+kConvTokens-1
    Vec xs[N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
        const int64_t t = t0 - (kConvK - 1) + k;
        xs[k] = (t >= 0 && t < p.T) ? *reinterpret_cast<const Vec*>(xb + t * p.x_st) : make_uint2(0u, 0u);
    }
    float w[V][kConvK];
    const E* wp = reinterpret_cast<const E*>(p.w);
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
        for (int j = 0; j < kConvK; ++j) w[i][j] = Elem<E>::ld(wp[(int64_t)(c0 + i) * p.w_sc + j]);

    float win[kConvK - 1][V];  // inputs t-3, t-2, t-1 in fp32
#pragma unroll
    for (int k = 0; k < kConvK - 1; ++k) {
        const E* e = reinterpret_cast<const E*>(&xs[k]);
#pragma unroll
        for (int i = 0; i < V; ++i) win[k][i] = Elem<E>::ld(e[i]);
    }
#pragma unroll
    for (int k = kConvK - 1; k < N; ++k) {
        const int64_t t = t0 - (kConvK - 1) + k;
        if (t >= p.T) break;
        const E* e = reinterpret_cast<const E*>(&xs[k]);
        Vec r;
        E* re = reinterpret_cast<E*>(&r);
#pragma unroll
        for (int i = 0; i < V; i += 2) {  // channel pairs: one packed rounding for the conv, one for the output
            const float x0 = Elem<E>::ld(e[i]), x1 = Elem<E>::ld(e[i + 1]);
            float y0 = fmaf(w[i][3], x0, fmaf(w[i][2], win[2][i], fmaf(w[i][1], win[1][i], w[i][0] * win[0][i])));
            float y1 = fmaf(w[i + 1][3], x1,
                            fmaf(w[i + 1][2], win[2][i + 1], fmaf(w[i + 1][1], win[1][i + 1], w[i + 1][0] * win[0][i + 1])));
            Elem<E>::rnd2(y0, y1);
            Elem<E>::st2(re + i, silu_f32(y0), silu_f32(y1));
#pragma unroll
            for (int c = i; c < i + 2; ++c) {
                win[0][c] = win[1][c];
                win[1][c] = win[2][c];
            }
            win[2][i] = x0;
            win[2][i + 1] = x1;
        }
        *reinterpret_cast<Vec*>(ob + t * p.o_st) = r;
    }
    // the cache's conv state: the last K raw inputs, zero-padded on the left when T < K (:346-348)
    if (p.state && blockIdx.y == gridDim.y - 1) {
        E* sb = reinterpret_cast<E*>(p.state) + (int64_t)b * p.s_sb;
#pragma unroll
        for (int k = 0; k < kConvK; ++k) {
            const int64_t t = p.T - kConvK + k;
            float v[V];
            if (t >= 0) {
                const Vec u = *reinterpret_cast<const Vec*>(xb + t * p.x_st);
                const E* e = reinterpret_cast<const E*>(&u);
#pragma unroll
                for (int i = 0; i < V; ++i) v[i] = Elem<E>::ld(e[i]);
            } else {
#pragma unroll
                for (int i = 0; i < V; ++i) v[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < V; ++i) sb[(int64_t)(c0 + i) * p.s_sc + k] = Elem<E>::st(v[i]);
        }
    }
}

// Decode: thread = one (sequence, channel); the K-wide state slides over the T new tokens
// (torch_causal_conv1d_update: cat([state, x]), keep the last K, conv without padding, :95-98).
template <typename E>
__global__ void __launch_bounds__(256) gdn_conv_update_kernel(ConvParams p) {
    const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (i >= (int64_t)p.B * p.C) return;
    const int b = (int)(i / p.C), c = (int)(i % p.C);
    const E* wp = reinterpret_cast<const E*>(p.w) + (int64_t)c * p.w_sc;
    float w[kConvK], s[kConvK];
    E* sp = reinterpret_cast<E*>(p.state) + (int64_t)b * p.s_sb + (int64_t)c * p.s_sc;
#pragma unroll
    for (int j = 0; j < kConvK; ++j) {
        w[j] = Elem<E>::ld(wp[j]);
        s[j] = Elem<E>::ld(sp[j]);
    }
    const E* xp = reinterpret_cast<const E*>(p.x) + (int64_t)b * p.x_sb + c;
    E* op = reinterpret_cast<E*>(p.out) + (int64_t)b * p.o_sb + c;
    for (int64_t t = 0; t < p.T; ++t) {
        const float xn = Elem<E>::ld(xp[t * p.x_st]);
        op[t * p.o_st] = Elem<E>::st(conv_silu<E>(w, s[1], s[2], s[3], xn));
        s[0] = s[1];
        s[1] = s[2];
        s[2] = s[3];
        s[3] = xn;
    }
#pragma unroll
    for (int j = 0; j < kConvK; ++j) sp[j] = Elem<E>::st(s[j]);
}

struct GateParams {
    View3 a, b;          // [B,T,H]
    const void* A_log;   // [H]
    const void* dt_bias; // [H]
    int64_t A_st, dt_st;
    int p_dtype;         // of A_log and dt_bias
    View3 g, beta;       // outputs: g (any float dtype; fp32 as the reference), beta (b's dtype in the reference)
    int B, H;
    int64_t T;
};

// beta = sigmoid(b) rounded to beta's dtype; g = -exp(A_log) softplus(a + dt_bias) in fp32 (:377-379).
__global__ void __launch_bounds__(256) gdn_gates_kernel(GateParams p) {
    const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (i >= (int64_t)p.B * p.T * p.H) return;
    const int h = (int)(i % p.H);
    const int64_t t = (i / p.H) % p.T;
    const int b = (int)(i / ((int64_t)p.H * p.T));
    const float a = load_elem(p.a.p, (int64_t)b * p.a.sb + t * p.a.st + (int64_t)h * p.a.sh, p.a.dtype);
    const float bb = load_elem(p.b.p, (int64_t)b * p.b.sb + t * p.b.st + (int64_t)h * p.b.sh, p.b.dtype);
    const float A_log = load_elem(p.A_log, (int64_t)h * p.A_st, p.p_dtype);
    const float dt = load_elem(p.dt_bias, (int64_t)h * p.dt_st, p.p_dtype);
    const float x = a + dt;
    const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, beta 1, threshold 20
    store_elem(const_cast<void*>(p.g.p), (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype, -expf(A_log) * sp);
    store_elem(const_cast<void*>(p.beta.p), (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype,
               __fdividef(1.0f, 1.0f + __expf(-bb)));
}

struct NormParams {
    const void* x;      // rows of D; row r = (group r / H, head r % H) at (r / H) * x_sg + (r % H) * x_sr
    int64_t x_sr;
    const void* gate;
    int64_t g_sr;
    const void* w;      // [D]
    void* out;
    int64_t o_sr;
    int64_t N;          // rows
    float eps;
    int64_t x_sg, g_sg, o_sg;  // group strides ([M, H, D] views; == the row strides for [N, D] views)
    int H;              // rows per group (1 for [N, D] views)
};

__device__ __forceinline__ int64_t norm_row_offset(int64_t r, int H, int64_t s_group, int64_t s_row) {
    return H == 1 ? r * s_row : (r / H) * s_group + (r % H) * s_row;
}

constexpr int kNormD = 128;  // head_v_dim

// Qwen3_5RMSNormGated (:62-71):
//   n = round(x * rsqrt(mean(x^2) + eps)); wn = round(weight * n); out = round(wn * silu(gate)).
// Vector form: each lane owns 16 bytes of a row (8 bf16), 128 / V lanes per row, several rows per warp.
template <typename E>
__device__ __forceinline__ void norm_finish(float (&h)[16 / sizeof(E)], const float (&z)[16 / sizeof(E)],
                                            const float (&w)[16 / sizeof(E)], float inv, float (&o)[16 / sizeof(E)]) {
#pragma unroll
    for (int e = 0; e < (int)(16 / sizeof(E)); ++e) {
        const float n = Elem<E>::rnd(h[e] * inv);
        const float wn = Elem<E>::rnd(w[e] * n);
        o[e] = wn * silu_f32(z[e]);
    }
}

template <typename E>
__global__ void __launch_bounds__(256) gdn_rms_norm_gated_vec_kernel(NormParams p) {
    constexpr int V = 16 / sizeof(E);       // elements per lane
    constexpr int LPR = kNormD / V;         // lanes per row (16 for bf16, 32 for fp32)
    constexpr int RPW = 32 / LPR;           // rows per warp
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR, l = lane % LPR;
    const int64_t row = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * RPW + sub;
    const bool live = row < p.N;
    const int64_t r = live ? row : 0;
    const uint4 xu = *reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(p.x) +
                                                      norm_row_offset(r, p.H, p.x_sg, p.x_sr) + V * l);
    const uint4 gu = *reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(p.gate) +
                                                      norm_row_offset(r, p.H, p.g_sg, p.g_sr) + V * l);
    const uint4 wu = *reinterpret_cast<const uint4*>(reinterpret_cast<const E*>(p.w) + V * l);
    const E* xe = reinterpret_cast<const E*>(&xu);
    const E* ge = reinterpret_cast<const E*>(&gu);
    const E* we = reinterpret_cast<const E*>(&wu);
    float h[V], z[V], w[V], o[V];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < V; ++e) {
        h[e] = Elem<E>::ld(xe[e]);
        z[e] = Elem<E>::ld(ge[e]);
        w[e] = Elem<E>::ld(we[e]);
        ss = fmaf(h[e], h[e], ss);
    }
#pragma unroll
    for (int o2 = LPR / 2; o2 > 0; o2 >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
    const float inv = rsqrtf(ss * (1.0f / kNormD) + p.eps);
    norm_finish<E>(h, z, w, inv, o);
    if (!live) return;
    uint4 ou;
    E* oe = reinterpret_cast<E*>(&ou);
#pragma unroll
    for (int e = 0; e < V; ++e) oe[e] = Elem<E>::st(o[e]);
    *reinterpret_cast<uint4*>(reinterpret_cast<E*>(p.out) + norm_row_offset(row, p.H, p.o_sg, p.o_sr) + V * l) = ou;
}

// Scalar form for rows that are not 16-byte aligned: one warp per row, 4 elements per lane.
template <typename E>
__global__ void __launch_bounds__(256) gdn_rms_norm_gated_kernel(NormParams p) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.N) return;
    const E* xr = reinterpret_cast<const E*>(p.x) + norm_row_offset(row, p.H, p.x_sg, p.x_sr) + 4 * lane;
    const E* gr = reinterpret_cast<const E*>(p.gate) + norm_row_offset(row, p.H, p.g_sg, p.g_sr) + 4 * lane;
    const E* wr = reinterpret_cast<const E*>(p.w) + 4 * lane;
    float h[4], z[4], w[4];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        h[e] = Elem<E>::ld(xr[e]);
        z[e] = Elem<E>::ld(gr[e]);
        w[e] = Elem<E>::ld(wr[e]);
        ss = fmaf(h[e], h[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * (1.0f / kNormD) + p.eps);
    E* orow = reinterpret_cast<E*>(p.out) + norm_row_offset(row, p.H, p.o_sg, p.o_sr) + 4 * lane;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float n = Elem<E>::rnd(h[e] * inv);
        const float wn = Elem<E>::rnd(w[e] * n);
        orow[e] = Elem<E>::st(wn * silu_f32(z[e]));
    }
}

}  // namespace


// ---------------------------------------------------------------------------------------- host side

namespace {

size_t esz(int dtype) { return dtype == GDN_F32 ? 4 : 2; }
bool float_dtype(int d) { return d == GDN_F32 || d == GDN_BF16 || d == GDN_F16; }

int bad(const char* fmt, const char* name) { return set_last_error(GDN_ERR_INVALID_ARGUMENT, fmt, name); }

// [d0, d1, d2] view with a contiguous last dim (shape checked against `want`, -1 = any).
int check_view(const char* name, const gdn_tensor* t, int ndim, const int64_t* want) {
    if (!t) return bad("%s is NULL", name);
    if (t->ndim != ndim) return set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s must be %d-D, got ndim=%d", name, ndim, t->ndim);
    if (!float_dtype(t->dtype)) return set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s has unsupported dtype code %d", name, t->dtype);
    for (int i = 0; i < ndim; ++i) {
        if (t->shape[i] < 0) return bad("%s has a negative dimension", name);
        if (want[i] >= 0 && t->shape[i] != want[i])
            return set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s: dim %d is %lld, expected %lld", name, i,
                                  (long long)t->shape[i], (long long)want[i]);
    }
    if (t->stride[ndim - 1] != 1) return bad("%s: the last dimension must be contiguous", name);
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= t->shape[i];
    if (n > 0 && !t->data) return bad("%s has a NULL data pointer", name);
    return GDN_OK;
}

// The 16-byte vector path of the prefill convolution: base and row strides on 16-byte boundaries.
bool vec16(const gdn_tensor* t) {
    const int64_t v = 16 / (int64_t)esz(t->dtype);
    if (reinterpret_cast<uintptr_t>(t->data) & 15) return false;
    for (int i = 0; i < t->ndim - 1; ++i)
        if (t->stride[i] % v) return false;
    return true;
}

int conv_checks(const gdn_tensor* x, const gdn_tensor* weight, const gdn_tensor* out, const gdn_tensor* state,
                bool state_required, ConvParams* p) {
    int rc;
    const int64_t any3[3] = {-1, -1, -1};
    if ((rc = check_view("x", x, 3, any3))) return rc;
    const int64_t B = x->shape[0], T = x->shape[1], C = x->shape[2];
    const int64_t wshape[2] = {C, kConvK};
    if ((rc = check_view("weight", weight, 2, wshape))) return rc;
    const int64_t oshape[3] = {B, T, C};
    if ((rc = check_view("out", out, 3, oshape))) return rc;
    if (state || state_required) {
        const int64_t sshape[3] = {B, C, kConvK};
        if ((rc = check_view("conv_state", state, 3, sshape))) return rc;
    }
    if (weight->dtype != x->dtype || out->dtype != x->dtype || (state && state->dtype != x->dtype))
        return set_last_error(GDN_ERR_UNSUPPORTED, "x, weight, out and conv_state must share one dtype");
    if (B * C > 0x7fffffffLL) return bad("%s: B*C too large", "x");
    const char* xb = reinterpret_cast<const char*>(x->data);
    const char* ob = reinterpret_cast<const char*>(out->data);
    if (B * T * C > 0 && xb == ob) return bad("%s must not alias x", "out");
    *p = ConvParams{};
    p->x = x->data;
    p->x_sb = x->stride[0];
    p->x_st = x->stride[1];
    p->w = weight->data;
    p->w_sc = weight->stride[0];
    p->out = out->data;
    p->o_sb = out->stride[0];
    p->o_st = out->stride[1];
    p->state = state ? state->data : nullptr;
    p->s_sb = state ? state->stride[0] : 0;
    p->s_sc = state ? state->stride[1] : 0;
    p->B = (int)B;
    p->C = (int)C;
    p->T = T;
    p->dtype = x->dtype;
    return GDN_OK;
}

template <typename E>
cudaError_t launch_conv_silu(const ConvParams& p, cudaStream_t st) {
    constexpr int V = 8 / sizeof(E);
    dim3 grid((unsigned)((p.C / V + kConvThreads - 1) / kConvThreads), (unsigned)((p.T + kConvTokens - 1) / kConvTokens),
              (unsigned)p.B);
    gdn_conv_silu_kernel<E><<<grid, kConvThreads, 0, st>>>(p);
    return cudaGetLastError();
}

template <typename E>
cudaError_t launch_conv_update(const ConvParams& p, cudaStream_t st) {
    const int64_t n = (int64_t)p.B * p.C;
    gdn_conv_update_kernel<E><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p);
    return cudaGetLastError();
}

template <typename E>
cudaError_t launch_norm(const NormParams& p, bool vec, cudaStream_t st) {
    if (vec) {
        constexpr int rows_per_cta = 8 * (32 / (kNormD / (16 / (int)sizeof(E))));
        gdn_rms_norm_gated_vec_kernel<E><<<(unsigned)((p.N + rows_per_cta - 1) / rows_per_cta), 256, 0, st>>>(p);
    } else {
        gdn_rms_norm_gated_kernel<E><<<(unsigned)((p.N + 7) / 8), 256, 0, st>>>(p);
    }
    return cudaGetLastError();
}

int launched(cudaError_t e, const char* what) {
    if (e != cudaSuccess) return set_last_error(GDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    note_launch();
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

extern "C" {

int gdn_causal_conv1d_silu(const gdn_tensor* x, const gdn_tensor* weight, gdn_tensor* out, gdn_tensor* conv_state,
                           void* stream) {
    gdn::ConvParams p;
    int rc = gdn::conv_checks(x, weight, out, conv_state, false, &p);
    if (rc) return rc;
    if (!gdn::vec16(x) || !gdn::vec16(out) || p.C % (int64_t)(16 / gdn::esz(p.dtype)))
        return gdn::set_last_error(GDN_ERR_UNSUPPORTED,
                                   "x and out need 16-byte aligned rows and C a multiple of 16 bytes of elements");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if ((int64_t)p.B * p.C == 0) return GDN_OK;
    if (p.T == 0) {  // no tokens: the conv state is all padding
        if (!conv_state) return GDN_OK;
        if (conv_state->stride[1] != gdn::kConvK || conv_state->stride[0] != (int64_t)p.C * gdn::kConvK)
            return gdn::set_last_error(GDN_ERR_UNSUPPORTED, "an empty sequence needs a packed conv_state");
        cudaError_t e = cudaMemsetAsync(conv_state->data, 0, (size_t)p.B * p.C * gdn::kConvK * gdn::esz(p.dtype), st);
        return e == cudaSuccess ? GDN_OK : gdn::set_last_error(GDN_ERR_CUDA, "conv_state reset: %s", cudaGetErrorName(e));
    }
    gdn::phase_event(0, st);
    cudaError_t e = p.dtype == GDN_BF16  ? gdn::launch_conv_silu<__nv_bfloat16>(p, st)
                    : p.dtype == GDN_F16 ? gdn::launch_conv_silu<__half>(p, st)
                                         : gdn::launch_conv_silu<float>(p, st);
    rc = gdn::launched(e, "conv1d launch");
    gdn::phase_event(1, st);
    return rc;
}

int gdn_causal_conv1d_update(const gdn_tensor* x, gdn_tensor* conv_state, const gdn_tensor* weight, gdn_tensor* out,
                             void* stream) {
    gdn::ConvParams p;
    int rc = gdn::conv_checks(x, weight, out, conv_state, true, &p);
    if (rc) return rc;
    if ((int64_t)p.B * p.C == 0 || p.T == 0) return GDN_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    gdn::phase_event(0, st);
    cudaError_t e = p.dtype == GDN_BF16  ? gdn::launch_conv_update<__nv_bfloat16>(p, st)
                    : p.dtype == GDN_F16 ? gdn::launch_conv_update<__half>(p, st)
                                         : gdn::launch_conv_update<float>(p, st);
    rc = gdn::launched(e, "conv1d update launch");
    gdn::phase_event(1, st);
    return rc;
}

int gdn_gates(const gdn_tensor* a, const gdn_tensor* b, const gdn_tensor* A_log, const gdn_tensor* dt_bias,
              gdn_tensor* g, gdn_tensor* beta, void* stream) {
    int rc;
    const int64_t any3[3] = {-1, -1, -1};
    if ((rc = gdn::check_view("a", a, 3, any3))) return rc;
    const int64_t shp[3] = {a->shape[0], a->shape[1], a->shape[2]};
    const int64_t hshape[1] = {a->shape[2]};
    if ((rc = gdn::check_view("b", b, 3, shp)) || (rc = gdn::check_view("A_log", A_log, 1, hshape)) ||
        (rc = gdn::check_view("dt_bias", dt_bias, 1, hshape)) || (rc = gdn::check_view("g", g, 3, shp)) ||
        (rc = gdn::check_view("beta", beta, 3, shp)))
        return rc;
    if (A_log->dtype != dt_bias->dtype) return gdn::set_last_error(GDN_ERR_UNSUPPORTED, "A_log and dt_bias must share one dtype");
    const int64_t n = shp[0] * shp[1] * shp[2];
    if (n == 0) return GDN_OK;
    gdn::GateParams p{};
    p.a = {a->data, a->stride[0], a->stride[1], a->stride[2], a->dtype};
    p.b = {b->data, b->stride[0], b->stride[1], b->stride[2], b->dtype};
    p.A_log = A_log->data;
    p.dt_bias = dt_bias->data;
    p.A_st = 1;
    p.dt_st = 1;
    p.p_dtype = A_log->dtype;
    p.g = {g->data, g->stride[0], g->stride[1], g->stride[2], g->dtype};
    p.beta = {beta->data, beta->stride[0], beta->stride[1], beta->stride[2], beta->dtype};
    p.B = (int)shp[0];
    p.T = shp[1];
    p.H = (int)shp[2];
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    gdn::phase_event(0, st);
    gdn::gdn_gates_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(p);
    rc = gdn::launched(cudaGetLastError(), "gates launch");
    gdn::phase_event(1, st);
    return rc;
}

int gdn_rms_norm_gated(const gdn_tensor* x, const gdn_tensor* gate, const gdn_tensor* weight, float eps,
                       gdn_tensor* out, void* stream) {
    int rc;
    if (!x) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "x is NULL");
    const int nd = x->ndim;
    if (nd != 2 && nd != 3)
        return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "x must be [N,128] or [M,H,128], got ndim=%d", nd);
    const int64_t rows2[2] = {-1, gdn::kNormD};
    const int64_t rows3[3] = {-1, -1, gdn::kNormD};
    if ((rc = gdn::check_view("x", x, nd, nd == 2 ? rows2 : rows3))) return rc;
    const int64_t shp[3] = {x->shape[0], x->shape[1], nd == 2 ? -1 : gdn::kNormD};
    const int64_t wshape[1] = {gdn::kNormD};
    if ((rc = gdn::check_view("gate", gate, nd, shp)) || (rc = gdn::check_view("weight", weight, 1, wshape)) ||
        (rc = gdn::check_view("out", out, nd, shp)))
        return rc;
    if (gate->dtype != x->dtype || weight->dtype != x->dtype || out->dtype != x->dtype)
        return gdn::set_last_error(GDN_ERR_UNSUPPORTED, "x, gate, weight and out must share one dtype");
    if (!(eps >= 0.f)) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "eps must be >= 0");
    const int64_t H = nd == 2 ? 1 : x->shape[1];
    const int64_t N = x->shape[0] * H;
    if (N == 0) return GDN_OK;
    if (H > 0x7fffffffLL) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "x: too many rows per group");
    const int r = nd - 2;  // index of the row-stride dim
    gdn::NormParams p{x->data, x->stride[r], gate->data, gate->stride[r], weight->data, out->data, out->stride[r],
                      N, eps, x->stride[0], gate->stride[0], out->stride[0], (int)H};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    gdn::phase_event(0, st);
    const bool vec = gdn::vec16(x) && gdn::vec16(gate) && gdn::vec16(out) && gdn::vec16(weight);
    cudaError_t e = x->dtype == GDN_BF16  ? gdn::launch_norm<__nv_bfloat16>(p, vec, st)
                    : x->dtype == GDN_F16 ? gdn::launch_norm<__half>(p, vec, st)
                                          : gdn::launch_norm<float>(p, vec, st);
    rc = gdn::launched(e, "gated RMS norm launch");
    gdn::phase_event(1, st);
    return rc;
}

}  // extern "C"
