// Backward of the chunked gated delta rule, CUDA-core (FFMA) path in fp32.
//
// The reference (qwen3_5_transformers.py:110-187) is inference-only; the gradients
// here are those autograd takes through its torch forward.  Per 64-token chunk
// (Q = q^ Dk^-1/2, E_ij = e^(gc_i - gc_j), L = -(beta k^ k^T) E strictly lower,
// T = (I - L)^-1, u = T beta v, w = T beta e^gc k^, Kd = k^ e^(gc_last - gc),
// Aqk = (Q k^T) E incl. the diagonal, Qg = Q e^gc, v_new = u - w S_c):
//
//   dv_new = Kd dS_{c+1} + Aqk^T do_c           (reverse scan, with)
//   dS_c   = e^gc_last dS_{c+1} + Qg^T do_c - w^T dv_new
//   dQg = do S_c^T, dw = -dv_new S_c^T, dKd = v_new dS_{c+1}^T         (gdn_bwd_states)
//   d(beta v) = T^T dv_new, d(beta e^gc k^) = T^T dw  (back substitution: no T is formed)
//   dL = strict(d(beta v) u^T + d(beta e^gc k^) w^T)  (= T^T dT T^T, as u = T beta v, w = T beta e^gc k^)
//   dAqk = incl(do v_new^T)                                              (gdn_bwd_wy)
//   then the chain rule through E, beta, e^gc, Q = q^ Dk^-1/2 and the l2norm (gdn_bwd_grads).
//
// Launches: the forward's CUDA-core prep (u, w, Qg, Kd, Aqk, e^gc_last per chunk) and
// scan (recording S_c), then gdn_bwd_scan (one CTA per (b, h, 16 state columns), chunks
// in reverse), then gdn_bwd_states, gdn_bwd_wy and gdn_bwd_grads (one CTA per chunk each,
// all chunks in parallel).  With bf16 q/k/v and d_out every step runs on the tensor cores
// instead (gdn_chunk_tc.cu: the tensor-core prep also writes the u, w, Kd and Aqk tiles, its
// scan records S_c, then gdn_bwd_scan_tc, gdn_bwd_states_tc, gdn_bwd_wy_tc and
// gdn_bwd_grads_tc); the kernels in this file serve fp32 inputs.
#include "gdn_bwd.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

using bwd::chunk_gates;
using bwd::qk_load;
using bwd::qk_norm;

constexpr int kThreads = 256;
constexpr int kPad = 132;   // fp32 row stride of 128-wide shared tiles
constexpr int kPad64 = 68;  // fp32 row stride of 64-wide shared tiles
constexpr int kScanDv = 16; // gradient-state columns per reverse-scan CTA
constexpr int kWide = 512;  // threads of the WY and gradient kernels (16 warps: their shared memory allows one CTA
                            // per SM, so the warps come from the CTA)
constexpr int kRg = kWide / 16;     // row groups of the 64-row tiles: thread (ty, tx) owns rows ty + kRg r
constexpr int kRt = kChunk / kRg;   // rows per thread in those tiles

// Hint: bring [p, p + bytes) into L2 (16-byte aligned, a multiple of 16 bytes).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Row t of a [B,T,H,D] view into a 128-wide shared row (4 elements per lane), zero past T.
__device__ __forceinline__ void row_to_smem(const View4& v, int b, int64_t t, int64_t T, int h, int lane, float* dst) {
    const int64_t base = (int64_t)b * v.sb + t * v.st + (int64_t)h * v.sh;
#pragma unroll
    for (int e = 0; e < 4; ++e) dst[lane + 32 * e] = t < T ? load_elem(v.p, base + lane + 32 * e, v.dtype) : 0.f;
}

// ============================================================================ reverse scan
//   dv_new = Kd dS + Aqk^T do;  dS <- e^gc_last dS + Qg^T do - w^T dv_new   (chunks in reverse)
struct BwdScanSmem {
    float W[kChunk][kPad];
    float Qg[kChunk][kPad];
    float Kd[kChunk][kPad];
    float A[kChunk][kPad64];
    float dO[kChunk][kScanDv];
    float dVn[kChunk][kScanDv];
    float dS[kDk][kScanDv];
};

__global__ void __launch_bounds__(kThreads) gdn_bwd_scan(BwdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    BwdScanSmem& s = *reinterpret_cast<BwdScanSmem*>(smem_raw);
    const int tid = threadIdx.x;
    const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
    const int dv0 = blockIdx.y * kScanDv;
    const int64_t sbase = (int64_t)bh * kDk * kDv;
    for (int idx = tid; idx < kDk * kScanDv; idx += kThreads) {
        const int d = idx / kScanDv, cc = idx % kScanDv;
        s.dS[d][cc] = p.dhT ? p.dhT[sbase + (int64_t)d * kDv + dv0 + cc] : 0.f;
    }
    const int r = tid >> 2, cq = (tid & 3) * 4;   // dv_new: row r, 4 columns
    const int sd = tid >> 1, sc = (tid & 1) * 8;  // dS update: row sd, 8 columns
    for (int c = p.NC - 1; c >= 0; --c) {
        const int64_t ci = (int64_t)bh * p.NC + c;
        const float* fw = p.fws + ci * kWsChunkFloats;
        float* bw = p.bws + ci * kBwChunkFloats;
        __syncthreads();  // the previous chunk's readers are done; dS is final
        for (int idx = tid; idx < kChunk * kDk / 4; idx += kThreads) {  // asynchronous: all pieces in flight
            const int i = idx >> 5, d4 = (idx & 31) * 4;
            cp_async16_rec(&s.W[i][d4], fw + kWsW + i * kDk + d4);
            cp_async16_rec(&s.Qg[i][d4], fw + kWsQg + i * kDk + d4);
            cp_async16_rec(&s.Kd[i][d4], fw + kWsKd + i * kDk + d4);
        }
        for (int idx = tid; idx < kChunk * kChunk / 4; idx += kThreads) {
            const int i = idx >> 4, j4 = (idx & 15) * 4;
            cp_async16_rec(&s.A[i][j4], fw + kWsAqk + i * kChunk + j4);
        }
        cp_async_commit_rec();
        for (int idx = tid; idx < kChunk * kScanDv; idx += kThreads) {
            const int i = idx / kScanDv, cc = idx % kScanDv;
            const int64_t t = (int64_t)c * kChunk + i;
            s.dO[i][cc] = t < p.T ? load_elem(p.dout.p, (int64_t)b * p.dout.sb + t * p.dout.st +
                                                            (int64_t)h * p.dout.sh + dv0 + cc, p.dout.dtype)
                                  : 0.f;
        }
        for (int idx = tid; idx < kDk * kScanDv / 4; idx += kThreads) {  // dS_{c+1} for the chunk kernels
            const int d = idx / (kScanDv / 4), c4 = (idx % (kScanDv / 4)) * 4;
            st4(bw + kBwDSe + (int64_t)d * kDv + dv0 + c4, ld4(&s.dS[d][c4]));
        }
        const float gamma = fw[kWsGamma];
        cp_async_wait_rec();
        __syncthreads();
        {  // dv_new = Kd dS + Aqk^T do (Aqk is lower incl. the diagonal: rows j >= r)
            float a[4] = {0.f, 0.f, 0.f, 0.f};
            for (int d = 0; d < kDk; d += 4) {
                const float4 k4 = ld4(&s.Kd[r][d]);
                const float kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 s4 = ld4(&s.dS[d + e][cq]);
                    a[0] += kv[e] * s4.x;
                    a[1] += kv[e] * s4.y;
                    a[2] += kv[e] * s4.z;
                    a[3] += kv[e] * s4.w;
                }
            }
            for (int j = r; j < kChunk; ++j) {
                const float av = s.A[j][r];
                const float4 o4 = ld4(&s.dO[j][cq]);
                a[0] += av * o4.x;
                a[1] += av * o4.y;
                a[2] += av * o4.z;
                a[3] += av * o4.w;
            }
            const float4 v = make_float4(a[0], a[1], a[2], a[3]);
            st4(&s.dVn[r][cq], v);
            st4(bw + kBwDVn + r * kDv + dv0 + cq, v);
        }
        __syncthreads();
        {  // dS <- gamma dS + Qg^T do - w^T dv_new (row sd: own entries only)
            float a[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = 0.f;
            for (int j = 0; j < kChunk; ++j) {
                const float qv = s.Qg[j][sd], wv = s.W[j][sd];
                const float4 o0 = ld4(&s.dO[j][sc]), o1 = ld4(&s.dO[j][sc + 4]);
                const float4 n0 = ld4(&s.dVn[j][sc]), n1 = ld4(&s.dVn[j][sc + 4]);
                a[0] += qv * o0.x - wv * n0.x;
                a[1] += qv * o0.y - wv * n0.y;
                a[2] += qv * o0.z - wv * n0.z;
                a[3] += qv * o0.w - wv * n0.w;
                a[4] += qv * o1.x - wv * n1.x;
                a[5] += qv * o1.y - wv * n1.y;
                a[6] += qv * o1.z - wv * n1.z;
                a[7] += qv * o1.w - wv * n1.w;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) s.dS[sd][sc + e] = s.dS[sd][sc + e] * gamma + a[e];
        }
    }
    __syncthreads();
    if (p.dh0) {
        for (int idx = tid; idx < kDk * kScanDv; idx += kThreads) {
            const int d = idx / kScanDv, cc = idx % kScanDv;
            p.dh0[sbase + (int64_t)d * kDv + dv0 + cc] = s.dS[d][cc];
        }
    }
}

// ============================================================================ state products
//   v_new = u - w S_c, dQg = do S_c^T, dw = -dv_new S_c^T, dKd = v_new dS_{c+1}^T, <S_c, dS_{c+1}>
// S_c and dS_{c+1} pass through shared memory in 32-row slabs.  128-wide tiles map thread
// (ty, tx) to rows ty + 16 r and columns 4 tx .. 4 tx + 3 and 64 + 4 tx .. (conflict-free float4 rows);
// slab products map thread to row tid / 4 and slab columns tid % 4 + 4 e.
struct StatesSmem {
    float W[kChunk][kPad];   // w, then v_new
    float dO[kChunk][kPad];
    float dVn[kChunk][kPad];
    float S[32][kPad];       // slab of S_c
    float E[32][kPad];       // slab of dS_{c+1}
    float red[kThreads / 32];
};

__global__ void __launch_bounds__(kThreads) gdn_bwd_states(BwdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    StatesSmem& s = *reinterpret_cast<StatesSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* fw = p.fws + ci * kWsChunkFloats;
    float* bw = p.bws + ci * kBwChunkFloats;
    const int ty = tid >> 4, tx = tid & 15, c0 = 4 * tx, c1 = 64 + 4 * tx;
    const int ri = tid >> 2, cs = tid & 3;
    for (int i = warp; i < kChunk; i += kThreads / 32) row_to_smem(p.dout, b, t0 + i, p.T, h, lane, &s.dO[i][0]);
    for (int idx = tid; idx < kChunk * kDk / 4; idx += kThreads) {
        const int i = idx >> 5, d4 = (idx & 31) * 4;
        cp_async16_rec(&s.W[i][d4], fw + kWsW + i * kDk + d4);
        cp_async16_rec(&s.dVn[i][d4], bw + kBwDVn + i * kDv + d4);
    }
    cp_async_commit_rec();

    float acc[4][8];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
    float dgam = 0.f;
    for (int slab = 0; slab < 4; ++slab) {
        __syncthreads();
        for (int idx = tid; idx < 32 * kDv / 4; idx += kThreads) {
            const int rr = idx >> 5, d4 = (idx & 31) * 4;
            const int64_t row = 32 * slab + rr;
            cp_async16_rec(&s.S[rr][d4], bw + kBwS + row * kDv + d4);
            cp_async16_rec(&s.E[rr][d4], bw + kBwDSe + row * kDv + d4);
        }
        cp_async_commit_rec();
        cp_async_wait_rec();
        __syncthreads();
        for (int idx = tid; idx < 32 * kDv / 4; idx += kThreads) {  // <S_c, dS_{c+1}> over the slab
            const int rr = idx >> 5, d4 = (idx & 31) * 4;
            const float4 sv = ld4(&s.S[rr][d4]), ev = ld4(&s.E[rr][d4]);
            dgam += sv.x * ev.x + sv.y * ev.y + sv.z * ev.z + sv.w * ev.w;
        }
        // v_new partial: acc += w[:, slab] S[slab, :]
        for (int kk = 0; kk < 32; ++kk) {
            const float4 s0 = ld4(&s.S[kk][c0]), s1 = ld4(&s.S[kk][c1]);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float wv = s.W[ty + 16 * r][32 * slab + kk];
                acc[r][0] += wv * s0.x;
                acc[r][1] += wv * s0.y;
                acc[r][2] += wv * s0.z;
                acc[r][3] += wv * s0.w;
                acc[r][4] += wv * s1.x;
                acc[r][5] += wv * s1.y;
                acc[r][6] += wv * s1.z;
                acc[r][7] += wv * s1.w;
            }
        }
        // dQg[:, slab] = do S[slab]^T and dw[:, slab] = -dv_new S[slab]^T
        float q8[8], w8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) q8[e] = w8[e] = 0.f;
        for (int dv = 0; dv < kDv; dv += 4) {
            const float4 o4 = ld4(&s.dO[ri][dv]), n4 = ld4(&s.dVn[ri][dv]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 s4 = ld4(&s.S[cs + 4 * e][dv]);
                q8[e] += o4.x * s4.x + o4.y * s4.y + o4.z * s4.z + o4.w * s4.w;
                w8[e] += n4.x * s4.x + n4.y * s4.y + n4.z * s4.z + n4.w * s4.w;
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            bw[kBwDQg + ri * kDk + 32 * slab + cs + 4 * e] = q8[e];
            bw[kBwDW + ri * kDk + 32 * slab + cs + 4 * e] = -w8[e];
        }
    }
    __syncthreads();  // every reader of w is done: v_new replaces it
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int i = ty + 16 * r;
        const float4 u0 = ld4(fw + kWsU + i * kDv + c0), u1 = ld4(fw + kWsU + i * kDv + c1);
        const float4 v0 = make_float4(u0.x - acc[r][0], u0.y - acc[r][1], u0.z - acc[r][2], u0.w - acc[r][3]);
        const float4 v1 = make_float4(u1.x - acc[r][4], u1.y - acc[r][5], u1.z - acc[r][6], u1.w - acc[r][7]);
        st4(&s.W[i][c0], v0);
        st4(&s.W[i][c1], v1);
        st4(bw + kBwVn + i * kDv + c0, v0);
        st4(bw + kBwVn + i * kDv + c1, v1);
    }
    // dKd[:, slab] = v_new dS_{c+1}[slab]^T
    for (int slab = 0; slab < 4; ++slab) {
        __syncthreads();
        for (int idx = tid; idx < 32 * kDv / 4; idx += kThreads) {
            const int rr = idx >> 5, d4 = (idx & 31) * 4;
            cp_async16_rec(&s.E[rr][d4], bw + kBwDSe + (int64_t)(32 * slab + rr) * kDv + d4);
        }
        cp_async_commit_rec();
        cp_async_wait_rec();
        __syncthreads();
        float k8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) k8[e] = 0.f;
        for (int dv = 0; dv < kDv; dv += 4) {
            const float4 n4 = ld4(&s.W[ri][dv]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 e4 = ld4(&s.E[cs + 4 * e][dv]);
                k8[e] += n4.x * e4.x + n4.y * e4.y + n4.z * e4.z + n4.w * e4.w;
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) bw[kBwDKd + ri * kDk + 32 * slab + cs + 4 * e] = k8[e];
    }
    dgam = warp_sum(dgam);
    if (lane == 0) s.red[warp] = dgam;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) t += s.red[w];
        bw[kBwSmall] = t;
    }
}

// ============================================================================ WY backward
//   d(beta v) = T^T dv_new and d(beta e^gc k^) = T^T dw by back substitution on (I - L)^T (thread =
//   one of the 256 right-hand-side columns, as the forward's prep solves for u and w), then dv, the
//   beta / gc / k^ terms of those products, dL = strict(d(beta v) u^T + d(beta e^gc k^) w^T) and
//   dAqk = incl(do v_new^T).
struct WySmem {
    float K[kChunk][kPad];     // k^
    float Lt[kChunk][kPad64];  // Lt[j][i] = L_ij
    float Xv[kChunk][kPad];    // d(beta v)
    float Xk[kChunk][kPad];    // d(beta e^gc k^)
    float U[kChunk][kPad];     // u, then v_new
    float W[kChunk][kPad];     // w, then do
    float gc[kChunk], beta[kChunk], egc[kChunk], ekd[kChunk];
};

__global__ void __launch_bounds__(kWide) gdn_bwd_wy(BwdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    WySmem& s = *reinterpret_cast<WySmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* fw = p.fws + ci * kWsChunkFloats;
    float* bw = p.bws + ci * kBwChunkFloats;
    // Every global input of the kernel is requested at entry: u, w (for dL) and v_new (for dAqk) by
    // asynchronous copies, d_out rows into Xk; Xv and Xk hold v_new and d_out until dAqk is formed,
    // then the back substitution's results.
    for (int idx = tid; idx < kChunk * kDk / 4; idx += kWide) {
        const int i = idx >> 5, d4 = (idx & 31) * 4;
        cp_async16_rec(&s.U[i][d4], fw + kWsU + i * kDv + d4);
        cp_async16_rec(&s.W[i][d4], fw + kWsW + i * kDk + d4);
        cp_async16_rec(&s.Xv[i][d4], bw + kBwVn + i * kDv + d4);
    }
    cp_async_commit_rec();
    if (tid == 0) {  // the back substitution's right-hand sides (dv_new, dw) into L2 meanwhile
        prefetch_l2(bw + kBwDVn, kChunk * kDv * 4);
        prefetch_l2(bw + kBwDW, kChunk * kDk * 4);
    }
    const int ty = tid >> 4, tx = tid & 15;
    const int cols[2] = {4 * tx, 64 + 4 * tx};
    for (int i = warp; i < kChunk; i += kWide / 32) row_to_smem(p.dout, b, t0 + i, p.T, h, lane, &s.Xk[i][0]);
    {  // k rows: a warp's 4 rows loaded together, then normalised
        constexpr int kR = kChunk / (kWide / 32);
        float x[kR][4], r;
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) qk_load(p.k, b, t0 + warp + (kWide / 32) * rr, p.T, h, lane, x[rr]);
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) {
            const int i = warp + (kWide / 32) * rr;
            qk_norm(p.k, t0 + i, p.T, p.l2norm, x[rr], r);
#pragma unroll
            for (int e = 0; e < 4; ++e) s.K[i][lane + 32 * e] = x[rr][e];
        }
    }
    chunk_gates(p, b, h, t0, s.gc, s.beta, s.egc, s.ekd);  // ends with a barrier

    {  // L_ij = -(beta_i k_i.k_j) e^(gc_i - gc_j), i > j, stored transposed
        float kk[kRt][4];
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) kk[r][cc] = 0.f;
        for (int d = 0; d < kDk; d += 4) {
            float4 ki[kRt], kj[4];
#pragma unroll
            for (int r = 0; r < kRt; ++r) ki[r] = ld4(&s.K[ty + kRg * r][d]);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) kj[cc] = ld4(&s.K[tx + 16 * cc][d]);
#pragma unroll
            for (int r = 0; r < kRt; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    kk[r][cc] += ki[r].x * kj[cc].x + ki[r].y * kj[cc].y + ki[r].z * kj[cc].z + ki[r].w * kj[cc].w;
        }
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int i = ty + kRg * r, j = tx + 16 * cc;
                s.Lt[j][i] = (i > j) ? -(s.beta[i] * kk[r][cc]) * expf(s.gc[i] - s.gc[j]) : 0.f;
            }
    }
    cp_async_wait_rec();
    __syncthreads();  // Lt, v_new (Xv) and d_out (Xk) are in shared memory
    {  // dAqk = incl(do v_new^T)
        float a[kRt][4];
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.f;
        for (int d = 0; d < kDv; d += 4) {
            float4 oo[kRt], vv[4];
#pragma unroll
            for (int r = 0; r < kRt; ++r) oo[r] = ld4(&s.Xk[ty + kRg * r][d]);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) vv[cc] = ld4(&s.Xv[tx + 16 * cc][d]);
#pragma unroll
            for (int r = 0; r < kRt; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    a[r][cc] += oo[r].x * vv[cc].x + oo[r].y * vv[cc].y + oo[r].z * vv[cc].z + oo[r].w * vv[cc].w;
        }
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int i = ty + kRg * r, j = tx + 16 * cc;
                bw[kBwDA + i * kChunk + j] = (i >= j) ? a[r][cc] : 0.f;
            }
    }
    __syncthreads();  // v_new and d_out are read: the substitution writes Xv and Xk
    if (tid < kDv + kDk) {  // back substitution: x_i = rhs_i + sum_{m > i} L_mi x_m, i = 63 .. 0
        const int col = tid;
        const float* src = bw + (col < kDv ? kBwDVn + col : kBwDW + (col - kDv));
        float x[kChunk];
#pragma unroll
        for (int i = 0; i < kChunk; ++i) x[i] = src[i * kDv];
#pragma unroll
        for (int i = kChunk - 2; i >= 0; --i) {
            // four independent partial sums: the dependent chain is a quarter as long
            float a0 = x[i], a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int m4 = (i + 1) / 4; m4 < kChunk / 4; ++m4) {
                // Lt[i][m] = L_mi = 0 for m <= i, so the head of the first group adds 0 * x
                const float4 l = ld4(&s.Lt[i][4 * m4]);
                a0 += l.x * x[4 * m4];
                a1 += l.y * x[4 * m4 + 1];
                a2 += l.z * x[4 * m4 + 2];
                a3 += l.w * x[4 * m4 + 3];
            }
            x[i] = (a0 + a1) + (a2 + a3);
        }
        float* dst = col < kDv ? &s.Xv[0][col] : &s.Xk[0][col - kDv];
#pragma unroll
        for (int i = 0; i < kChunk; ++i) dst[i * kPad] = x[i];
    }
    __syncthreads();
    {  // dv = beta d(beta v); d beta, d gc and the k^ term of d(beta e^gc k^)
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
            const int i = ty + kRg * r;
            const int64_t t = t0 + i;
            const float bi = s.beta[i], be = s.beta[i] * s.egc[i];
            float sv = 0.f, sk = 0.f;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const int cc = cols[hlf];
                const float4 xv = ld4(&s.Xv[i][cc]), xk = ld4(&s.Xk[i][cc]), kv = ld4(&s.K[i][cc]);
                const float xva[4] = {xv.x, xv.y, xv.z, xv.w};
                {
                    const int64_t vb = (int64_t)b * p.v.sb + t * p.v.st + (int64_t)h * p.v.sh + cc;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float vv = t < p.T ? load_elem(p.v.p, vb + e, p.v.dtype) : 0.f;
                        sv += vv * xva[e];
                    }
                }
                if (t < p.T) {
                    const int64_t ob = (int64_t)b * p.dv.sb + t * p.dv.st + (int64_t)h * p.dv.sh + cc;
                    __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(p.dv.p) + ob;
                    if (p.dv.dtype == GDN_BF16 && (reinterpret_cast<uintptr_t>(o16) & 7) == 0) {  // one 8-byte store
                        const __nv_bfloat162 o01 = __floats2bfloat162_rn(bi * xva[0], bi * xva[1]);
                        const __nv_bfloat162 o23 = __floats2bfloat162_rn(bi * xva[2], bi * xva[3]);
                        *reinterpret_cast<uint2*>(o16) = make_uint2(*reinterpret_cast<const uint32_t*>(&o01),
                                                                    *reinterpret_cast<const uint32_t*>(&o23));
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) store_elem(p.dv.p, ob + e, p.dv.dtype, bi * xva[e]);
                    }
                }
                sk += kv.x * xk.x + kv.y * xk.y + kv.z * xk.z + kv.w * xk.w;
                st4(bw + kBwDKp + i * kDk + cc, make_float4(be * xk.x, be * xk.y, be * xk.z, be * xk.w));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                sv += __shfl_xor_sync(0xffffffffu, sv, o);
                sk += __shfl_xor_sync(0xffffffffu, sk, o);
            }
            if (tx == 0) {
                bw[kBwSmall + 64 + i] = sv + s.egc[i] * sk;  // dbeta: v . d(beta v) + e^gc k^ . d(beta e^gc k^)
                bw[kBwSmall + 128 + i] = be * sk;            // dgc:   (beta e^gc k^) . d(beta e^gc k^)
            }
        }
    }
    {  // dL = strict(d(beta v) u^T + d(beta e^gc k^) w^T)
        float a[kRt][4];
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) a[r][cc] = 0.f;
        for (int d = 0; d < kDk; d += 4) {
            float4 xv[kRt], xk[kRt], uu[4], ww[4];
#pragma unroll
            for (int r = 0; r < kRt; ++r) {
                xv[r] = ld4(&s.Xv[ty + kRg * r][d]);
                xk[r] = ld4(&s.Xk[ty + kRg * r][d]);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uu[cc] = ld4(&s.U[tx + 16 * cc][d]);
                ww[cc] = ld4(&s.W[tx + 16 * cc][d]);
            }
#pragma unroll
            for (int r = 0; r < kRt; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                    a[r][cc] += xv[r].x * uu[cc].x + xv[r].y * uu[cc].y + xv[r].z * uu[cc].z + xv[r].w * uu[cc].w +
                                xk[r].x * ww[cc].x + xk[r].y * ww[cc].y + xk[r].z * ww[cc].z + xk[r].w * ww[cc].w;
        }
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int i = ty + kRg * r, j = tx + 16 * cc;
                bw[kBwDL + i * kChunk + j] = (i > j) ? a[r][cc] : 0.f;
            }
    }
}

// ============================================================================ gradients
//   Aqk = (Q k^T) E, L = -(beta G) E (G = k^ k^T):  dP = dAqk E, dG = -beta_i E dL,
//   dbeta += (-G E) . dL, dgc_i += sum_j R_ij - sum_j R_ji with R = Aqk dAqk + L dL;
//   dQ = dP k^ + e^gc dQg, dk^ = dP^T Q + (dG + dG^T) k^ + e^(gc_last - gc) dKd + [beta e^gc d(...)];
//   dgc += Qg . dQg - Kd . dKd, dgc_last += sum Kd . dKd + e^gc_last <S_c, dS_{c+1}>;
//   dg = reverse cumsum of dgc in the chunk; dq = Dk^-1/2 dQ and dk^ through the l2norm.
struct GradSmem {
    float Q[kChunk][kPad];    // q^ Dk^-1/2
    float K[kChunk][kPad];    // k^
    float X[kChunk][kPad];    // dQg
    float Xd[kChunk][kPad];   // dKd
    float Kp[kChunk][kPad];   // dk^ through beta e^gc k^
    float P[kChunk][kPad64];  // dAqk -> dP
    float G[kChunk][kPad64];  // dL -> dG
    float gc[kChunk], beta[kChunk], egc[kChunk], ekd[kChunk], rq[kChunk], rk[kChunk];
    float dgc[kChunk], dbeta[kChunk];
    float colpart[kRg][kChunk];  // column sums of R per row group, summed in a fixed order
    float dglpart[kRg];          // dgc_last terms per row group
};

__global__ void __launch_bounds__(kWide) gdn_bwd_grads(BwdParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    GradSmem& s = *reinterpret_cast<GradSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* bw = p.bws + ci * kBwChunkFloats;
    const float scale = rsqrtf((float)kDk);
    // every record tile of the chunk is requested at entry (asynchronous copies) and waited for once
    for (int idx = tid; idx < kChunk * kChunk / 4; idx += kWide) {
        const int i = idx >> 4, j4 = (idx & 15) * 4;
        cp_async16_rec(&s.P[i][j4], bw + kBwDA + i * kChunk + j4);
        cp_async16_rec(&s.G[i][j4], bw + kBwDL + i * kChunk + j4);
    }
    for (int idx = tid; idx < kChunk * kDk / 4; idx += kWide) {
        const int i = idx >> 5, d4 = (idx & 31) * 4;
        cp_async16_rec(&s.X[i][d4], bw + kBwDQg + i * kDk + d4);
        cp_async16_rec(&s.Xd[i][d4], bw + kBwDKd + i * kDk + d4);
        cp_async16_rec(&s.Kp[i][d4], bw + kBwDKp + i * kDk + d4);
    }
    cp_async_commit_rec();
    {  // q and k rows: a warp's 4 rows of each loaded together, then normalised
        constexpr int kR = kChunk / (kWide / 32);
        float xq[kR][4], xk[kR][4], r;
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) {
            qk_load(p.q, b, t0 + warp + (kWide / 32) * rr, p.T, h, lane, xq[rr]);
            qk_load(p.k, b, t0 + warp + (kWide / 32) * rr, p.T, h, lane, xk[rr]);
        }
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) {
            const int i = warp + (kWide / 32) * rr;
            qk_norm(p.q, t0 + i, p.T, p.l2norm, xq[rr], r);
#pragma unroll
            for (int e = 0; e < 4; ++e) s.Q[i][lane + 32 * e] = xq[rr][e] * scale;
            if (lane == 0) s.rq[i] = r;
            qk_norm(p.k, t0 + i, p.T, p.l2norm, xk[rr], r);
#pragma unroll
            for (int e = 0; e < 4; ++e) s.K[i][lane + 32 * e] = xk[rr][e];
            if (lane == 0) s.rk[i] = r;
        }
    }
    if (tid < kChunk) {
        s.dbeta[tid] = bw[kBwSmall + 64 + tid];
        s.dgc[tid] = bw[kBwSmall + 128 + tid];
    }
    cp_async_wait_rec();  // the record tiles landed; chunk_gates' barriers publish them
    chunk_gates(p, b, h, t0, s.gc, s.beta, s.egc, s.ekd);  // ends with a barrier

    const int ty = tid >> 4, tx = tid & 15;
    {  // the 64 x 64 terms
        float kk[kRt][4], qk[kRt][4];
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) kk[r][cc] = qk[r][cc] = 0.f;
        for (int d = 0; d < kDk; d += 4) {
            float4 ki[kRt], qi[kRt], kj[4];
#pragma unroll
            for (int r = 0; r < kRt; ++r) {
                ki[r] = ld4(&s.K[ty + kRg * r][d]);
                qi[r] = ld4(&s.Q[ty + kRg * r][d]);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) kj[cc] = ld4(&s.K[tx + 16 * cc][d]);
#pragma unroll
            for (int r = 0; r < kRt; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    kk[r][cc] += ki[r].x * kj[cc].x + ki[r].y * kj[cc].y + ki[r].z * kj[cc].z + ki[r].w * kj[cc].w;
                    qk[r][cc] += qi[r].x * kj[cc].x + qi[r].y * kj[cc].y + qi[r].z * kj[cc].z + qi[r].w * kj[cc].w;
                }
        }
        __syncthreads();  // every thread has read the operands; P and G are rewritten in place below
        float rowR[kRt], rowB[kRt], colR[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < kRt; ++r) rowR[r] = rowB[r] = 0.f;
#pragma unroll
        for (int r = 0; r < kRt; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int i = ty + kRg * r, j = tx + 16 * cc;
                const float E = (i >= j) ? expf(s.gc[i] - s.gc[j]) : 0.f;
                const float LB = (i > j) ? -kk[r][cc] * E : 0.f;  // -G E; L = beta_i LB
                const float A = (i >= j) ? qk[r][cc] * E : 0.f;
                const float dA = s.P[i][j], dL = s.G[i][j];
                const float R = A * dA + s.beta[i] * LB * dL;
                rowR[r] += R;
                colR[cc] += R;
                rowB[r] += LB * dL;
                s.P[i][j] = dA * E;
                s.G[i][j] = (i > j) ? -s.beta[i] * E * dL : 0.f;
            }
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                rowR[r] += __shfl_xor_sync(0xffffffffu, rowR[r], o);
                rowB[r] += __shfl_xor_sync(0xffffffffu, rowB[r], o);
            }
            if (tx == 0) {
                atomicAdd(&s.dgc[ty + kRg * r], rowR[r]);
                atomicAdd(&s.dbeta[ty + kRg * r], rowB[r]);
            }
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) s.colpart[ty][tx + 16 * cc] = colR[cc];
    }
    __syncthreads();
    if (tid < kChunk) {  // every add to one address comes from one thread, in program order: deterministic
        float cs = 0.f;
        for (int y = 0; y < kRg; ++y) cs += s.colpart[y][tid];
        s.dgc[tid] -= cs;
    }
    __syncthreads();  // dgc is updated again below, by other threads
    const int cols[2] = {4 * tx, 64 + 4 * tx};
    float dq[kRt][8], dk[kRt][8];
#pragma unroll
    for (int r = 0; r < kRt; ++r)
#pragma unroll
        for (int e = 0; e < 8; ++e) dq[r][e] = dk[r][e] = 0.f;
    for (int j = 0; j < kChunk; ++j) {
        const float4 k0 = ld4(&s.K[j][cols[0]]), k1 = ld4(&s.K[j][cols[1]]);
        const float4 q0 = ld4(&s.Q[j][cols[0]]), q1 = ld4(&s.Q[j][cols[1]]);
        const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
            const int i = ty + kRg * r;
            const float pij = s.P[i][j], pji = s.P[j][i], gs = s.G[i][j] + s.G[j][i];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                dq[r][e] += pij * kv[e];
                dk[r][e] += pji * qv[e] + gs * kv[e];
            }
        }
    }
    {  // + e^gc dQg; dgc += Qg . dQg
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
            const int i = ty + kRg * r;
            const float eg = s.egc[i];
            float sq = 0.f;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const float4 x = ld4(&s.X[i][cols[hlf]]), qq = ld4(&s.Q[i][cols[hlf]]);
                dq[r][4 * hlf] += eg * x.x;
                dq[r][4 * hlf + 1] += eg * x.y;
                dq[r][4 * hlf + 2] += eg * x.z;
                dq[r][4 * hlf + 3] += eg * x.w;
                sq += qq.x * x.x + qq.y * x.y + qq.z * x.z + qq.w * x.w;
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (tx == 0) atomicAdd(&s.dgc[i], eg * sq);
        }
    }
    {  // + e^(gc_last - gc) dKd + the beta e^gc term; dgc -= Kd . dKd, dgc_last += sum Kd . dKd
        float dgl = 0.f;
#pragma unroll
        for (int r = 0; r < kRt; ++r) {
            const int i = ty + kRg * r;
            const float ek = s.ekd[i];
            float sk = 0.f;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const float4 x = ld4(&s.Xd[i][cols[hlf]]), kq = ld4(&s.K[i][cols[hlf]]);
                const float4 kp = ld4(&s.Kp[i][cols[hlf]]);
                dk[r][4 * hlf] += ek * x.x + kp.x;
                dk[r][4 * hlf + 1] += ek * x.y + kp.y;
                dk[r][4 * hlf + 2] += ek * x.z + kp.z;
                dk[r][4 * hlf + 3] += ek * x.w + kp.w;
                sk += kq.x * x.x + kq.y * x.y + kq.z * x.z + kq.w * x.w;
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
            if (tx == 0) atomicAdd(&s.dgc[i], -ek * sk);
            dgl += ek * sk;
        }
        if (tx == 0) s.dglpart[ty] = dgl;
    }
    __syncthreads();
    if (tid == 0) {
        float dgl = 0.f;
        for (int y = 0; y < kRg; ++y) dgl += s.dglpart[y];
        s.dgc[kChunk - 1] += dgl + s.egc[kChunk - 1] * bw[kBwSmall];
    }
    __syncthreads();
    // outputs: dq, dk through the l2norm (dx = r (dx^ - x^ (x^ . dx^)), x^ = x r), dg, dbeta
#pragma unroll
    for (int r = 0; r < kRt; ++r) {
        const int i = ty + kRg * r;
        const int64_t t = t0 + i;
        const bool in = t < p.T;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
            const View4& X = which == 0 ? p.q : p.k;
            const Out4& O = which == 0 ? p.dq : p.dk;
            const float rr = which == 0 ? s.rq[i] : s.rk[i];
            float g8[8], xh[8];
            float dot = 0.f;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const int64_t xb = (int64_t)b * X.sb + t * X.st + (int64_t)h * X.sh + cols[hlf];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    g8[4 * hlf + e] = which == 0 ? scale * dq[r][4 * hlf + e] : dk[r][4 * hlf + e];
                    xh[4 * hlf + e] = in ? load_elem(X.p, xb + e, X.dtype) * rr : 0.f;
                    dot += xh[4 * hlf + e] * g8[4 * hlf + e];
                }
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (in) {
#pragma unroll
                for (int hlf = 0; hlf < 2; ++hlf) {
                    const int64_t ob = (int64_t)b * O.sb + t * O.st + (int64_t)h * O.sh + cols[hlf];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float gv = g8[4 * hlf + e];
                        store_elem(O.p, ob + e, O.dtype, p.l2norm ? rr * (gv - xh[4 * hlf + e] * dot) : gv);
                    }
                }
            }
        }
    }
    if (warp == 0) {  // dg_t = sum_{i >= t} dgc_i: suffix scan over the chunk, two rows per lane
        const float a0 = s.dgc[2 * lane], a1 = s.dgc[2 * lane + 1];
        float x = a0 + a1;  // suffix sum from this pair on
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_down_sync(0xffffffffu, x, o);
            if (lane + o < 32) x += y;
        }
        const float dg[2] = {x, x - a0};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int i = 2 * lane + e;
            const int64_t t = t0 + i;
            if (t < p.T) {
                store_elem(p.dg.p, (int64_t)b * p.dg.sb + t * p.dg.st + (int64_t)h * p.dg.sh, p.dg.dtype, dg[e]);
                store_elem(p.dbeta.p, (int64_t)b * p.dbeta.sb + t * p.dbeta.st + (int64_t)h * p.dbeta.sh,
                           p.dbeta.dtype, s.dbeta[i]);
            }
        }
    }
}

}  // namespace

cudaError_t launch_chunk_bwd(const ChunkParams& fwd, const BwdParams& p, cudaStream_t stream) {
    static_assert(sizeof(BwdScanSmem) <= 227 * 1024 && sizeof(StatesSmem) <= 227 * 1024, "smem");
    static_assert(sizeof(WySmem) <= 227 * 1024 && sizeof(GradSmem) <= 227 * 1024, "smem");
    cudaError_t e;
    // forward recompute, the scan recording S_c into every chunk's backward record
    ChunkParams f = fwd;
    f.out = nullptr;
    f.hT = nullptr;
    f.states = p.bws + kBwS;
    f.states_stride = kBwChunkFloats;
    if (p.tc_records) {  // tensor-core prep (records M, Q', b, o0; u, w, Kd, Aqk tiles into fws) + scan
        f.ws = reinterpret_cast<float*>(p.tc_records);
        f.bwd_tiles = p.fws;
        if ((e = phase_event(0, stream)) != cudaSuccess) return e;
        if ((e = launch_chunk_tc_prep(f, stream)) != cudaSuccess) return e;
        if ((e = phase_event(1, stream)) != cudaSuccess) return e;
        if ((e = launch_chunk_tc_scan(f, stream)) != cudaSuccess) return e;
        if ((e = phase_event(2, stream)) != cudaSuccess) return e;
    } else {  // the CUDA-core prep and scan (phase events 0-2 inside)
        f.ws = p.fws;
        if ((e = launch_chunk_simt(f, stream)) != cudaSuccess) return e;
    }
    struct K {
        const void* fn;
        size_t smem;
    };
    const K ks[4] = {{(const void*)gdn_bwd_scan, sizeof(BwdScanSmem)},
                     {(const void*)gdn_bwd_states, sizeof(StatesSmem)},
                     {(const void*)gdn_bwd_wy, sizeof(WySmem)},
                     {(const void*)gdn_bwd_grads, sizeof(GradSmem)}};
    for (const K& k : ks)
        if ((e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem)) != cudaSuccess)
            return e;
    const unsigned nchunks = (unsigned)((int64_t)p.B * p.H * p.NC);
    if (p.tc_records) {
        if ((e = launch_bwd_scan_tc(p, stream)) != cudaSuccess) return e;
    } else {
        gdn_bwd_scan<<<dim3((unsigned)(p.B * p.H), kDv / kScanDv), kThreads, sizeof(BwdScanSmem), stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        note_launch();
    }
    if ((e = phase_event(3, stream)) != cudaSuccess) return e;
    if (p.tc_records) {  // bf16 mode: the state products on the tensor cores
        if ((e = launch_bwd_states_tc(p, stream)) != cudaSuccess) return e;
    } else {
        gdn_bwd_states<<<nchunks, kThreads, sizeof(StatesSmem), stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        note_launch();
    }
    if ((e = phase_event(4, stream)) != cudaSuccess) return e;
    if (p.tc_records) {  // bf16 mode: the WY products on the tensor cores
        if ((e = launch_bwd_wy_tc(p, stream)) != cudaSuccess) return e;
    } else {
        gdn_bwd_wy<<<nchunks, kWide, sizeof(WySmem), stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        note_launch();
    }
    if ((e = phase_event(5, stream)) != cudaSuccess) return e;
    if (p.tc_records) {  // bf16 mode: the chain rule's products on the tensor cores
        if ((e = launch_bwd_grads_tc(p, stream)) != cudaSuccess) return e;
    } else {
        gdn_bwd_grads<<<nchunks, kWide, sizeof(GradSmem), stream>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        note_launch();
    }
    return phase_event(6, stream);
}

}  // namespace gdn
