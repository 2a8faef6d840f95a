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

#include <atomic>
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

// Programmatic dependent launch: every kernel here is launched with programmatic stream serialization, so
// the next kernel of a decode step may be scheduled while this one runs.  A kernel reads nothing the
// previous kernel may write, and writes nothing, before griddep_wait() (which returns once the previous
// grid has completed and its memory is visible); before it, it may only read weights.  Right after the
// wait it lets the next kernel launch.  Launched without the attribute, both are no-ops.
__device__ __forceinline__ void griddep_wait_and_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

std::atomic<int> g_pdl{1};

// Launch with programmatic stream serialization (the next kernel of the stream may start while this one runs;
// see griddep_wait_and_release), unless switched off by gdn_model_set_programmatic_launch(0).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl.load(std::memory_order_relaxed) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// --------------------------------------------------------------------------- residual add + RMSNorm

struct AddNormArgs {
    const bf16* x;
    int64_t x_s;
    const float* xp;  // or: x = bf16(sum of nsplit fp32 planes [nsplit][N][D]) (a split-K GEMM's partials)
    int nsplit;
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
    float w[8];
    load8(a.w + c, w);  // the weight only: nothing the previous kernel writes is read before the wait
    griddep_wait_and_release();
    float h[8];
    if (a.xp) {
        const int64_t plane = (int64_t)gridDim.x * a.D;
        const float* src = a.xp + row * a.D + c;
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = 0.f;
        for (int sp = 0; sp < a.nsplit; ++sp) {  // fixed order: deterministic
            const float4 u = *reinterpret_cast<const float4*>(src + sp * plane);
            const float4 v = *reinterpret_cast<const float4*>(src + sp * plane + 4);
            h[0] += u.x, h[1] += u.y, h[2] += u.z, h[3] += u.w, h[4] += v.x, h[5] += v.y, h[6] += v.z, h[7] += v.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = rbf(h[i]);  // the projection's bf16 output
    } else {
        load8(a.x + row * a.x_s + c, h);
    }
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
    float o[8];
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
    griddep_wait_and_release();
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
    griddep_wait_and_release();
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
    griddep_wait_and_release();
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

// --------------------------------------------------------------------------- skinny GEMM (decode projections)

// out[m, n] = sum_k x[m, k] W[n, k] for a decode batch (M <= 32 rows of x) against a weight W [N, K] read
// exactly once: the projections of a decode step are weight-bandwidth-bound, so the kernel is built to keep
// weight bytes in flight.  A CTA owns 64 rows of W (a 16-row tile per warp) and one of `ksplit` K ranges;
// its threads stream the range through a shared-memory ring of kStages 64-column blocks (the 64 W rows and
// the M rows of x of each block, cp.async in 16-byte pieces; piece p of row r sits at slot p ^ (r & 7), so
// the fragment reads are conflict-free), and each warp multiplies its tile on the tensor cores with
// mma.sync m16n8k16 (W rows as A, x rows as B, one n8 tile per 8 batch rows).  Inside each 64-column block
// the K order is permuted identically for W and x: lane c of a fragment takes columns 16c .. 16c+15, which
// hold its k positions {2c, 2c+1, 2c+8, 2c+9} of the four k16 steps, so a lane reads 32 contiguous bytes of
// a row.  Epilogues:
//   kStore    out[m, n] in bf16 (the output rounding of the reference's bf16 Linear), ksplit = 1;
//   kSiluMul  W interleaves fc1 / fc2 rows in groups of 8 (rows 16j..16j+7 = fc1 rows 8j.., 16j+8..16j+15 =
//             fc2 rows 8j..): out[m, 8j + i] = bf16(bf16(SiLU(bf16(fc1))) * bf16(fc2)) (qwen3_5.py:42-46),
//             ksplit = 1;
//   kPartial  fp32 partial sums of K range s into partial[s][m][n] (the consumer sums the planes in order:
//             gdn_model_add_rms_norm_partials), so no atomics and a deterministic result.
enum : int { kStore = 0, kSiluMul = 1, kPartial = 2 };
constexpr int kGemmMaxM = 32;
constexpr int kStages = 10;

// NW warps per CTA own 16 NW rows of W; a stage holds those rows' and x's 64 columns (bf16)
template <int MT, int NW>
constexpr int gemm_stage_bytes() { return 16 * NW * 128 + 8 * MT * 128; }
template <int MT>
constexpr int gemm_warps() { return MT >= 3 ? 2 : 4; }  // wide batches: more, smaller CTAs

struct GemmArgs {
    const bf16* x;
    int64_t x_s;
    const bf16* w;
    int64_t w_s;
    bf16* out;
    int64_t o_s;
    float* partial;  // [ksplit][M][N]
    int M, N, K;
    int ksplit;
    int kblocks_per_split;
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void lds128(uint4& v, uint32_t addr) {
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
}

template <int MT, int EPI>
__global__ void __launch_bounds__(gemm_warps<MT>() * 32) gdn_model_gemm_kernel(GemmArgs a) {
    extern __shared__ __align__(128) unsigned char gsm_raw[];
    constexpr int NW = gemm_warps<MT>();
    constexpr int kThreads = 32 * NW;
    constexpr int kGemmRows = 16 * NW;
    constexpr int kWStage = kGemmRows * 128;
    constexpr int kStage = gemm_stage_bytes<MT, NW>();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int rows0 = blockIdx.x * kGemmRows;                 // first W row of this CTA
    const int split = blockIdx.y;
    const int kb0 = split * a.kblocks_per_split;
    const int nkb = min(a.kblocks_per_split, a.K / 64 - kb0);
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(gsm_raw);
    // copy plan of one stage: W pieces i = tid + 128 j (j < 4): row i / 8 (rows past N are skipped), piece i % 8;
    // x pieces i = tid + 128 j (j < MT*8*8/128): row i / 8 (rows past M are zero-filled)
    constexpr int kXPieces = MT * 8 * 8;
    auto issue_w = [&](int b) {
        const uint32_t st = ring + (uint32_t)(b % kStages) * kStage;
        const int64_t k0 = (int64_t)(kb0 + b) * 64;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + kThreads * j, r = i >> 3, pc = i & 7;
            const int n = rows0 + r;
            const uint32_t d = st + r * 128 + ((pc ^ (r & 7)) << 4);
            const bf16* src = a.w + (int64_t)(n < a.N ? n : 0) * a.w_s + k0 + pc * 8;
            const uint32_t bytes = n < a.N ? 16u : 0u;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
        }
    };
    auto issue_x = [&](int b) {
        const uint32_t st = ring + (uint32_t)(b % kStages) * kStage;
        const int64_t k0 = (int64_t)(kb0 + b) * 64;
#pragma unroll
        for (int j = 0; j < (kXPieces + kThreads - 1) / kThreads; ++j) {
            const int i = tid + kThreads * j;
            if (i < kXPieces) {
                const int r = i >> 3, pc = i & 7;
                const uint32_t d = st + kWStage + r * 128 + ((pc ^ (r & 7)) << 4);
                const bf16* src = a.x + (int64_t)(r < a.M ? r : 0) * a.x_s + k0 + pc * 8;
                const uint32_t bytes = r < a.M ? 16u : 0u;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
            }
        }
    };
    // the first blocks' weights before the wait (weights are never written by a kernel of the step), x after
#pragma unroll
    for (int b = 0; b < kStages - 1; ++b)
        if (b < nkb) issue_w(b);
    griddep_wait_and_release();
#pragma unroll
    for (int b = 0; b < kStages - 1; ++b)
        if (b < nkb) issue_x(b);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // the prologue's blocks, then the steady pipeline
    float acc[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
    // fragment reads: W rows 16 warp + g and + 8, x rows 8t + g; column pieces 2c and 2c + 1
    const int wr = 16 * warp + g;
    const uint32_t wa0 = (uint32_t)(wr * 128 + (((2 * c) ^ (wr & 7)) << 4));
    const uint32_t wa1 = (uint32_t)(wr * 128 + (((2 * c + 1) ^ (wr & 7)) << 4));
    const uint32_t wb0 = wa0 + 8 * 128, wb1 = wa1 + 8 * 128;  // row wr + 8 has the same (row & 7)
    const uint32_t xa0 = (uint32_t)(kWStage + g * 128 + (((2 * c) ^ g) << 4));
    const uint32_t xa1 = (uint32_t)(kWStage + g * 128 + (((2 * c + 1) ^ g) << 4));
    for (int b = 0; b < nkb; ++b) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
        __syncthreads();  // block b has landed for every thread, and every warp is done with block b - 1's stage
        if (b + kStages - 1 < nkb) {  // refills the stage block b - 1 used
            issue_w(b + kStages - 1);
            issue_x(b + kStages - 1);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint32_t st = ring + (uint32_t)(b % kStages) * kStage;
        uint4 ra[2], rb[2];
        lds128(ra[0], st + wa0);
        lds128(ra[1], st + wa1);
        lds128(rb[0], st + wb0);
        lds128(rb[1], st + wb1);
        const uint32_t* A0 = reinterpret_cast<const uint32_t*>(ra);
        const uint32_t* A1 = reinterpret_cast<const uint32_t*>(rb);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            uint4 xb[2];
            lds128(xb[0], st + xa0 + t * 8 * 128);
            lds128(xb[1], st + xa1 + t * 8 * 128);
            const uint32_t* B = reinterpret_cast<const uint32_t*>(xb);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t af[4] = {A0[2 * s], A1[2 * s], A0[2 * s + 1], A1[2 * s + 1]};
                mma_bf16_16816(acc[t], af, B[2 * s], B[2 * s + 1]);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    const int n0 = rows0 + 16 * warp;
    if (n0 >= a.N) return;
    // C fragment: acc[t][0] = (row g, col 2c), [1] = (g, 2c+1), [2] = (g+8, 2c), [3] = (g+8, 2c+1); rows are
    // W rows n0 + ..., cols batch rows 8t + ...
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        const int m0 = 8 * t + 2 * c;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int m = m0 + j;
            if (m >= a.M) continue;
            if (EPI == kSiluMul) {
                const float u = rbf(acc[t][j]), gt = rbf(acc[t][2 + j]);
                a.out[(int64_t)m * a.o_s + n0 / 2 + g] = __float2bfloat16_rn(rbf(u / (1.0f + expf(-u))) * gt);
            } else if (EPI == kPartial) {
                float* P = a.partial + ((size_t)split * a.M + m) * a.N;
                P[n0 + g] = acc[t][j];
                P[n0 + g + 8] = acc[t][2 + j];
            } else {
                a.out[(int64_t)m * a.o_s + n0 + g] = __float2bfloat16_rn(acc[t][j]);
                a.out[(int64_t)m * a.o_s + n0 + g + 8] = __float2bfloat16_rn(acc[t][2 + j]);
            }
        }
    }
}

template <int MT, int EPI>
cudaError_t launch_gemm_mt(const GemmArgs& a, cudaStream_t st) {
    constexpr int NW = gemm_warps<MT>();
    constexpr int kGemmRows = 16 * NW;
    constexpr int smem = kStages * gemm_stage_bytes<MT, NW>();
    static std::atomic<uint64_t> attr_done{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (smem > 48 * 1024 && !(attr_done.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(gdn_model_gemm_kernel<MT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit, std::memory_order_release);
    }
    const dim3 grid((unsigned)((a.N + kGemmRows - 1) / kGemmRows), (unsigned)a.ksplit);
    return launch_k(gdn_model_gemm_kernel<MT, EPI>, grid, dim3(NW * 32), smem, st, a);
}

template <int EPI>
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t st) {
    switch ((a.M + 7) / 8) {
        case 1: return launch_gemm_mt<1, EPI>(a, st);
        case 2: return launch_gemm_mt<2, EPI>(a, st);
        case 3: return launch_gemm_mt<3, EPI>(a, st);
        default: return launch_gemm_mt<4, EPI>(a, st);
    }
}

// --------------------------------------------------------------------------- fused GatedDeltaNet decode step

// One decode token of a GatedDeltaNet layer after its input projection, in one kernel: the conv update
// (torch_causal_conv1d_update, qwen3_5_transformers.py:85-101), the gates (:377-379), the recurrent rule
// (:190-229, q/k l2-normalised in the kernel) on the cached state, and the gated RMS norm with z
// (Qwen3_5RMSNormGated, :56-71).  One 256-thread CTA per (sequence, head) owns the head's 384 conv channels
// (q, k, v) and its whole 128 x 128 fp32 state: the state loads are issued first and land while the
// conv and gates run; the state layout and arithmetic are those of gdn_recurrent_kernel (warp w: rows
// 16w..16w+15, lane l: columns 4l..4l+3, half the rows in registers, half in shared memory).  Every
// intermediate is rounded where the separate kernels round it (conv output and SiLU to bf16, beta to
// bf16, the rule's output to bf16 before the norm).
struct GdnDecodeArgs {
    const bf16* proj;   // [B, C + Hv*Dv + 2 Hv]: mixed qkv | z | b | a (the fused in_proj row)
    int64_t proj_s;
    bf16* conv_state;   // [B, C, 4]
    int64_t cs_sb;
    const bf16* conv_w; // [C, 4]
    const bf16* A_log;  // [H]
    const bf16* dt_bias;
    float* state;       // [B, H, 128, 128], updated in place
    const bf16* norm_w; // [128]
    float eps;
    bf16* out;          // [B, H * 128]
    int64_t out_s;
    int H, C;
    int prefetch_state;  // the state is not written by any kernel that may still run (see the C ABI)
};

constexpr int kDecThreads = 256;
constexpr int kDecWarps = 8;
constexpr int kDecRows = 16;      // state rows per warp
constexpr int kDecRegRows = 8;    // rows 0-7 of a warp in registers, 8-15 in shared memory

__device__ __forceinline__ float silu_fast(float y) {
    constexpr float kLog2e = 1.4426950408889634f;
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-y * kLog2e));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return y * r;
}

__global__ void __launch_bounds__(kDecThreads, 4) gdn_model_gdn_decode_kernel(GdnDecodeArgs a) {
    __shared__ __align__(16) float4 srows[kDecWarps][kDecRows - kDecRegRows][32];  // 32 KiB
    __shared__ __align__(16) float qs[128];
    __shared__ __align__(16) float ks[128];
    __shared__ __align__(16) float vs[128];
    __shared__ float gb[2];
    __shared__ __align__(16) float red[kDecWarps][128];   // kv partials
    __shared__ __align__(16) float red2[kDecWarps][128];  // o partials (their own array: no barrier between the two)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
    const int r0 = kDecRows * warp, c0 = 4 * lane;
    if (!a.prefetch_state) griddep_wait_and_release();
    // 1. the state: shared-memory rows by cp.async, register rows by plain loads, all in flight now (with
    //    prefetch_state, while the kernel before this one still runs)
    float* st = a.state + (int64_t)bh * 128 * 128 + c0;
#pragma unroll
    for (int r = 0; r < kDecRows - kDecRegRows; ++r)
        cp_async16_rec(&srows[warp][r][lane], st + (int64_t)(r0 + kDecRegRows + r) * 128);
    cp_async_commit_rec();
    float S[kDecRegRows][4];
#pragma unroll
    for (int r = 0; r < kDecRegRows; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(st + (int64_t)(r0 + r) * 128);
        S[r][0] = v.x, S[r][1] = v.y, S[r][2] = v.z, S[r][3] = v.w;
    }
    if (a.prefetch_state) griddep_wait_and_release();  // the projection row and conv state come from here on
    // 2. conv update of the head's q / k / v channels (window [s1, s2, s3, x]), conv + SiLU rounded to bf16
    const bf16* prow = a.proj + (int64_t)b * a.proj_s;
    const int key_dim = a.H * 128;
    for (int i = tid; i < 384; i += kDecThreads) {
        const int part = i >> 7, j = i & 127;  // 0 = q, 1 = k, 2 = v
        const int ch = part * key_dim + h * 128 + j;
        bf16* sp = a.conv_state + (int64_t)b * a.cs_sb + (int64_t)ch * 4;
        const uint2 su = *reinterpret_cast<const uint2*>(sp);
        const uint2 wu = *reinterpret_cast<const uint2*>(a.conv_w + (int64_t)ch * 4);
        const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&su);
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wu);
        const float2 sa = __bfloat1622float2(s2[0]), sb = __bfloat1622float2(s2[1]);
        const float2 wa = __bfloat1622float2(w2[0]), wb = __bfloat1622float2(w2[1]);
        const float xn = __bfloat162float(prow[ch]);
        float acc = wa.x * sa.y;  // taps in order over the window [s1, s2, s3, x]
        acc = fmaf(wa.y, sb.x, acc);
        acc = fmaf(wb.x, sb.y, acc);
        acc = fmaf(wb.y, xn, acc);
        const float y = rbf(silu_fast(rbf(acc)));
        uint2 so;
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&so);
        o2[0] = __floats2bfloat162_rn(sa.y, sb.x);
        o2[1] = __floats2bfloat162_rn(sb.y, xn);
        *reinterpret_cast<uint2*>(sp) = so;
        (part == 0 ? qs : part == 1 ? ks : vs)[j] = y;
    }
    if (tid == 0) {  // gates: g fp32, beta rounded to bf16 (b's dtype)
        const float bv = __bfloat162float(prow[a.C + a.H * 128 + h]);        // b follows z
        const float av = __bfloat162float(prow[a.C + a.H * 128 + a.H + h]);  // a follows b
        const float x = av + __bfloat162float(a.dt_bias[h]);
        const float spl = x > 20.f ? x : log1pf(expf(x));
        gb[0] = -expf(__bfloat162float(a.A_log[h])) * spl;
        gb[1] = rbf(__fdividef(1.0f, 1.0f + __expf(-bv)));
    }
    __syncthreads();
    if (warp < 2) {  // q (warp 0) and k (warp 1) l2-normalised with bf16 roundings; q scaled by Dk^-1/2
        float* v = warp == 0 ? qs : ks;
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = v[lane + 32 * i];
        const float inv = l2norm_inv(x, GDN_BF16);
        const float sc = warp == 0 ? rsqrtf(128.f) : 1.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) v[lane + 32 * i] = round_to(x[i] * inv, GDN_BF16) * sc;
    }
    cp_async_wait_rec();
    __syncthreads();
    // 3. the recurrent rule for one token (gdn_recurrent_kernel's arithmetic)
    const float decay = expf(gb[0]);
    float4 part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kDecRegRows; ++r) {
        const float kr = ks[r0 + r];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) S[r][cc] *= decay;
        part.x += S[r][0] * kr, part.y += S[r][1] * kr, part.z += S[r][2] * kr, part.w += S[r][3] * kr;
    }
#pragma unroll
    for (int r = 0; r < kDecRows - kDecRegRows; ++r) {
        const float kr = ks[r0 + kDecRegRows + r];
        float4 x = srows[warp][r][lane];
        x.x *= decay, x.y *= decay, x.z *= decay, x.w *= decay;
        srows[warp][r][lane] = x;
        part.x += x.x * kr, part.y += x.y * kr, part.z += x.z * kr, part.w += x.w * kr;
    }
    *reinterpret_cast<float4*>(&red[warp][c0]) = part;
    __syncthreads();
    float kv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
        const float4 x = *reinterpret_cast<const float4*>(&red[w][c0]);
        kv[0] += x.x, kv[1] += x.y, kv[2] += x.z, kv[3] += x.w;
    }
    const float4 v4 = *reinterpret_cast<const float4*>(&vs[c0]);
    const float beta = gb[1];
    const float delta[4] = {(v4.x - kv[0]) * beta, (v4.y - kv[1]) * beta, (v4.z - kv[2]) * beta, (v4.w - kv[3]) * beta};
    float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kDecRegRows; ++r) {
        const float kr = ks[r0 + r], qr = qs[r0 + r];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) S[r][cc] += kr * delta[cc];
        op.x += S[r][0] * qr, op.y += S[r][1] * qr, op.z += S[r][2] * qr, op.w += S[r][3] * qr;
    }
#pragma unroll
    for (int r = 0; r < kDecRows - kDecRegRows; ++r) {
        const float kr = ks[r0 + kDecRegRows + r], qr = qs[r0 + kDecRegRows + r];
        float4 x = srows[warp][r][lane];
        x.x += kr * delta[0], x.y += kr * delta[1], x.z += kr * delta[2], x.w += kr * delta[3];
        srows[warp][r][lane] = x;
        op.x += x.x * qr, op.y += x.y * qr, op.z += x.z * qr, op.w += x.w * qr;
    }
    *reinterpret_cast<float4*>(&red2[warp][c0]) = op;
    // the new state leaves while the output is reduced
#pragma unroll
    for (int r = 0; r < kDecRegRows; ++r)
        *reinterpret_cast<float4*>(st + (int64_t)(r0 + r) * 128) = make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
#pragma unroll
    for (int r = 0; r < kDecRows - kDecRegRows; ++r)
        *reinterpret_cast<float4*>(st + (int64_t)(r0 + kDecRegRows + r) * 128) = srows[warp][r][lane];
    __syncthreads();
    if (warp == 0) {  // 4. o (bf16, the rule's output dtype) -> gated RMS norm with z
        float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(&red2[w][c0]);
            o[0] += x.x, o[1] += x.y, o[2] += x.z, o[3] += x.w;
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[i] = rbf(o[i]);
            ss = fmaf(o[i], o[i], ss);
        }
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss * (1.0f / 128.0f) + a.eps);
        const bf16* z = prow + a.C + h * 128 + c0;
        float res[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float n = rbf(o[i] * inv);
            const float wn = rbf(__bfloat162float(a.norm_w[c0 + i]) * n);
            res[i] = wn * silu_fast(__bfloat162float(z[i]));
        }
        bf16* orow = a.out + (int64_t)b * a.out_s + h * 128 + c0;
        *reinterpret_cast<__nv_bfloat162*>(orow) = __floats2bfloat162_rn(res[0], res[1]);
        *reinterpret_cast<__nv_bfloat162*>(orow + 2) = __floats2bfloat162_rn(res[2], res[3]);
    }
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

namespace {
int add_rms_norm_impl(const gdn_tensor* x, const float* partial, int nsplit, int64_t pN, int64_t pD,
                      const gdn_tensor* residual, const gdn_tensor* weight, float eps, gdn_tensor* out,
                      gdn_tensor* residual_out, void* stream) {
    using namespace gdn;
    int rc;
    int64_t N = pN, D = pD;
    if (!partial) {
        if ((rc = view("x", x, 2, nullptr))) return rc;
        N = x->shape[0];
        D = x->shape[1];
    } else if (nsplit < 1 || nsplit > 64 || (reinterpret_cast<uintptr_t>(partial) & 15) || pN < 0 || pD <= 0) {
        return bad("partial must be 16-byte aligned fp32 planes, 1 <= nsplit <= 64, rows >= 0, dim > 0");
    }
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
    AddNormArgs a{partial ? nullptr : reinterpret_cast<const bf16*>(x->data), partial ? 0 : x->stride[0], partial,
                  nsplit, residual ? reinterpret_cast<const bf16*>(residual->data) : nullptr,
                  residual ? residual->stride[0] : 0,
                  reinterpret_cast<const bf16*>(weight->data), reinterpret_cast<bf16*>(out->data), out->stride[0],
                  residual ? reinterpret_cast<bf16*>(residual_out->data) : nullptr,
                  residual ? residual_out->stride[0] : 0, (int)D, eps};
    return launched(launch_k(gdn_model_add_rms_norm_kernel, dim3((unsigned)N), dim3((unsigned)(D / 8)), 0,
                             reinterpret_cast<cudaStream_t>(stream), a),
                    "add_rms_norm launch");
}
}  // namespace

void gdn_model_set_programmatic_launch(int enable) { gdn::g_pdl.store(enable ? 1 : 0); }

int gdn_model_add_rms_norm(const gdn_tensor* x, const gdn_tensor* residual, const gdn_tensor* weight, float eps,
                           gdn_tensor* out, gdn_tensor* residual_out, void* stream) {
    return add_rms_norm_impl(x, nullptr, 0, 0, 0, residual, weight, eps, out, residual_out, stream);
}

int gdn_model_add_rms_norm_partials(const float* partial, int nsplit, int64_t rows, int64_t dim,
                                    const gdn_tensor* residual, const gdn_tensor* weight, float eps, gdn_tensor* out,
                                    gdn_tensor* residual_out, void* stream) {
    return add_rms_norm_impl(nullptr, partial, nsplit, rows, dim, residual, weight, eps, out, residual_out, stream);
}

int gdn_model_gdn_decode(const gdn_tensor* proj, gdn_tensor* conv_state, const gdn_tensor* conv_w,
                         const gdn_tensor* A_log, const gdn_tensor* dt_bias, float* state, const gdn_tensor* norm_w,
                         float eps, gdn_tensor* out, int prefetch_state, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("out", out, 2, nullptr))) return rc;
    const int64_t B = out->shape[0], HD = out->shape[1];
    if (HD % 128 || HD <= 0) return bad("out must be [B, H * 128]");
    const int64_t H = HD / 128, C = 3 * HD;
    const int64_t pshp[2] = {B, C + HD + 2 * H}, cshp[3] = {B, C, 4}, wshp[2] = {C, 4}, hshp[1] = {H}, nshp[1] = {128};
    if ((rc = view("proj", proj, 2, pshp)) || (rc = view("A_log", A_log, 1, hshp)) ||
        (rc = view("dt_bias", dt_bias, 1, hshp)) || (rc = view("norm_w", norm_w, 1, nshp)))
        return rc;
    // conv_state / conv_w: rows of 4 taps (8 bytes, read and written whole), channels packed
    for (const gdn_tensor* t : {static_cast<const gdn_tensor*>(conv_state), conv_w}) {
        const bool st = t == conv_state;
        const int nd = st ? 3 : 2;
        const int64_t* want = st ? cshp : wshp;
        if (!t || t->ndim != nd || t->dtype != GDN_BF16) return bad("%s must be a bf16 %d-D tensor", st ? "conv_state" : "conv_w", nd);
        for (int i = 0; i < nd; ++i)
            if (t->shape[i] != want[i]) return bad("%s has the wrong shape", st ? "conv_state" : "conv_w");
        if (t->stride[nd - 1] != 1 || t->stride[nd - 2] != 4 || (reinterpret_cast<uintptr_t>(t->data) & 7) ||
            (st && (t->stride[0] & 3)))
            return bad("%s must hold rows of 4 contiguous taps, 8-byte aligned", st ? "conv_state" : "conv_w");
    }
    if (!state || (reinterpret_cast<uintptr_t>(state) & 15)) return bad("state must be a 16-byte aligned fp32 buffer");
    if (!(eps >= 0.f)) return bad("eps must be >= 0");
    if (B * H > 0x7fffffffLL) return bad("B * H too large");
    if (B * H == 0) return GDN_OK;
    GdnDecodeArgs args{reinterpret_cast<const bf16*>(proj->data), proj->stride[0], reinterpret_cast<bf16*>(conv_state->data),
                       conv_state->stride[0], reinterpret_cast<const bf16*>(conv_w->data),
                       reinterpret_cast<const bf16*>(A_log->data), reinterpret_cast<const bf16*>(dt_bias->data), state,
                       reinterpret_cast<const bf16*>(norm_w->data), eps, reinterpret_cast<bf16*>(out->data),
                       out->stride[0], (int)H, (int)C, prefetch_state ? 1 : 0};
    return launched(launch_k(gdn_model_gdn_decode_kernel, dim3((unsigned)(B * H)), dim3(kDecThreads), 0,
                             reinterpret_cast<cudaStream_t>(stream), args),
                    "gdn decode launch");
}

int gdn_model_linear(const gdn_tensor* x, const gdn_tensor* w, gdn_tensor* out, float* partial, int ksplit,
                     int epilogue, void* stream) {
    using namespace gdn;
    int rc;
    if ((rc = view("x", x, 2, nullptr)) || (rc = view("w", w, 2, nullptr))) return rc;
    const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
    if (w->shape[1] != K) return bad("w must be [N, %lld], got width %lld", (long long)K, (long long)w->shape[1]);
    if (M < 1 || M > kGemmMaxM) return bad("x must have 1 to %d rows (a decode batch), got %lld", kGemmMaxM, (long long)M);
    if (K % 64 || K <= 0) return bad("K must be a positive multiple of 64, got %lld", (long long)K);
    if (N % 16 || N <= 0 || N / 16 > 0x7fffffffLL) return bad("N must be a positive multiple of 16, got %lld", (long long)N);
    if (epilogue != kStore && epilogue != kSiluMul && epilogue != kPartial) return bad("unknown epilogue %d", epilogue);
    const int kblocks = (int)(K / 64);
    if (epilogue == kPartial) {
        if (ksplit < 1 || ksplit > 64 || ksplit > kblocks) return bad("ksplit must be in [1, min(64, K/64)]");
        if (!partial || (reinterpret_cast<uintptr_t>(partial) & 15)) return bad("partial must be a 16-byte aligned fp32 buffer");
    } else {
        ksplit = 1;
        const int64_t oshp[2] = {M, epilogue == kSiluMul ? N / 2 : N};
        if ((rc = view("out", out, 2, oshp))) return rc;
    }
    const int per = (kblocks + ksplit - 1) / ksplit;
    if ((int64_t)(ksplit - 1) * per >= kblocks) return bad("ksplit %d leaves an empty K range", ksplit);
    if (N / 32 + 1 > 0x7fffffffLL) return bad("N too large");
    GemmArgs a{reinterpret_cast<const bf16*>(x->data), x->stride[0], reinterpret_cast<const bf16*>(w->data), w->stride[0],
               epilogue == kPartial ? nullptr : reinterpret_cast<bf16*>(out->data),
               epilogue == kPartial ? 0 : out->stride[0], partial, (int)M, (int)N, (int)K, ksplit, per};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = epilogue == kStore    ? launch_gemm<kStore>(a, st)
                    : epilogue == kSiluMul ? launch_gemm<kSiluMul>(a, st)
                                           : launch_gemm<kPartial>(a, st);
    return launched(e, "linear launch");
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
    return launched(launch_k(gdn_model_attn_prep_kernel, dim3((unsigned)T, (unsigned)B), dim3((unsigned)(32 * (Hq + 2 * Hkv))),
                             0, reinterpret_cast<cudaStream_t>(stream), a),
                    "attn_prep launch");
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
    return launched(launch_k(gdn_model_attention_kernel, dim3((unsigned)T, (unsigned)Hq, (unsigned)B),
                             dim3(kAttnWarps * 32), smem, reinterpret_cast<cudaStream_t>(stream), a),
                    "attention launch");
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
    return launched(launch_k(gdn_model_silu_mul_kernel, dim3((unsigned)((work + 255) / 256)), dim3(256), 0,
                             reinterpret_cast<cudaStream_t>(stream), a),
                    "silu_mul launch");
}

}  // extern "C"
