// Chunked gated delta rule on the sm_100a tensor cores (tcgen05 + TMEM).
//
// The reference's chunk loop (qwen3_5_transformers.py:170-180) is rewritten as
// an affine recurrence on the chunk-start state S_c (Dk x Dv, fp32):
//
//   S_{c+1} = M_c S_c + b_c          M_c = e^{gc_last} I - kd^T w,   b_c = kd^T u
//   o_c     = Q'_c S_c + o0_c        Q'_c = q e^{gc} Dk^-1/2 - Aqk w,  o0_c = Aqk u
//
// with u = T beta v, w = T beta e^{gc} k (T the unit-lower-triangular WY inverse,
// :154-160), kd = k e^{gc_last - gc} (:179) and Aqk the causal decayed q k^T
// (:172).  Everything that does not depend on S is computed for all chunks in
// parallel (gdn_prep_tc); the sequential part shrinks to one 128x128x128 and
// one 64x128x128 product per chunk (gdn_scan_tc).
//
// Precision.  Only q^, k^ (the l2-normalised inputs, bf16 exactly as the
// reference rounds them) and v are exact bf16 MMA operands.  Every other
// operand of the prep is a derived fp32 quantity and enters its MMA as a
// hi + lo pair of bf16 (two MMAs), so the prep is fp32-accurate.  The scan
// feeds M_c, Q'_c and S_c to the MMA in bf16 and keeps S, b and o0 in fp32.
//
// gdn_prep_tc: persistent, one CTA (16 warps) per SM walking the (batch, head,
// 64-token chunk) records; the next chunk's rows are prefetched with cp.async
// and each output image leaves with an asynchronous bulk copy.  Operands
// that share a B matrix are stacked into M=128 MMAs so every accumulator fills
// all 128 TMEM lanes.
//   1. rows of q, k, v -> l2norm (16-bit rounding as the reference) -> bf16
//      128B-swizzled tiles [k^; q^] and v in shared memory
//   2. [k^; q^] k^T on the tensor cores -> G_k (lanes 0-63) and G_q (64-127)
//   3. L = -(beta G_k e^(gc_i-gc_j)) strictly lower, Aqk = Dk^-1/2 G_q e^(gc_i-gc_j) causal
//   4. T = (I - L)^-1 in 16x16 blocks (diagonal blocks by substitution, then
//      the off-diagonal blocks by distance)
//   5. X = E_d T B_e, Y = E_d T B, W = Aqk T B, Z = Aqk T B_e  (64x64, fp32)
//   6. [X; Z] k^ -> P_X | Zk and [Y; W] v -> P_Y | o0  (M=128, N=128, K=64, hi+lo)
//   7. Q' = q^ e^gc Dk^-1/2 - Zk, o0 -> workspace; P_X, P_Y -> hi+lo B tiles
//   8. M' = k^T P_X, b = k^T P_Y (M=128, N=128, K=64, hi+lo)
//   9. M = e^gc_last I - M', b -> workspace
// gdn_scan_tc: one CTA per (batch, head, 32-column slice of Dv); warps 4-5
//   bulk-copy each chunk's workspace record (double-buffered, the M/Q half freed
//   as soon as the tensor core has read it, records pulled into L2 four chunks
//   ahead); warps 0-3 turn the state accumulator into the next state, one lane
//   issues the next chunk's state MMAs as soon as that state is in shared
//   memory (then the output MMAs, into alternating TMEM columns), and a chunk's
//   output rows are written while the next chunk's MMAs run.
#include <cuda_bf16.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_tc.cuh"

namespace gdn {
namespace {

using namespace tc;

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s; a healthy wait here takes microseconds

__device__ __forceinline__ void report(unsigned int* err, unsigned int bit) {
    if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// bf16 hi/lo split: x ~= hi + lo with |x - hi - lo| <= 2^-16 |x|.
__device__ __forceinline__ void split_bf16(float x, float& hi, float& lo) {
    hi = __bfloat162float(__float2bfloat16_rn(x));
    lo = x - hi;
}

// ============================================================================ prep

constexpr int kPrepThreads = 512;
constexpr uint32_t P_KQ = 0;           // bf16 [128 rows][128] swizzled: rows 0-63 k^, 64-127 q^ (atom columns 16 KiB apart)
constexpr uint32_t P_V = 32768;        // bf16 [64 rows][128] swizzled v (atom columns 8 KiB apart)
constexpr int kLd = 68;                // fp32 row stride of L and T (16-byte rows)
constexpr int kAqkLd = 65;             // Aqk is only accessed as scalars: odd stride
constexpr uint32_t P_L = 49152;        // fp32 [64][68]
constexpr uint32_t P_AQK = 66560;      // fp32 [64][65]
constexpr uint32_t P_T = 83200;        // fp32 [64][68]
constexpr uint32_t P_Y3 = 100608;      // fp32 [3][16][16], scratch of the blocked inverse
constexpr uint32_t P_SPLIT = 104448;   // [X;Z] and [Y;W] hi/lo A tiles (4 x 16 KiB), later PX/PY hi/lo B tiles
constexpr uint32_t P_MISC = 169984;
constexpr uint32_t P_RAW = 172032;     // raw bf16 rows [3][64][128] of the next chunk (cp.async prefetch, 48 KiB)
// Output staging in regions that are dead by then; each image leaves with one bulk copy.
constexpr uint32_t P_STG_Q = P_L;           // Q' image (16 KiB), written in step 7 (L/Aqk/T are dead)
constexpr uint32_t P_STG_O0 = P_L + 16384;  // o0 column tiles (32 KiB), step 7
constexpr uint32_t P_STG_M = P_KQ;          // M image (32 KiB), step 9 (k^/q^ are dead after step 8)
constexpr uint32_t P_STG_B = P_SPLIT;       // b column tiles (64 KiB), step 9 (P tiles are dead after step 8)
static_assert(P_STG_O0 + 32768 <= P_SPLIT, "step-7 staging must not overlap the P tiles");
constexpr uint32_t P_SMEM = P_RAW + 49152 + 1024;
constexpr uint32_t kPrepTmemCols = 256;

struct PrepMisc {
    float gc[64];
    float beta[64];
    float egc[64];
    float ekd[64];
    uint64_t bar;
    uint32_t tmem;
};

__device__ __forceinline__ void store_bf16x4(unsigned char* tile, uint32_t off, const float (&x)[4]) {
    uint2 u;
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    *reinterpret_cast<uint2*>(tile + off) = u;
}

// 8 consecutive values -> one 16-byte chunk of a swizzled bf16 tile (global or shared).
__device__ __forceinline__ void store_bf16x8(unsigned char* tile, uint32_t off, const float* x) {
    uint4 u;
    u.x = pack_bf16x2(x[0], x[1]);
    u.y = pack_bf16x2(x[2], x[3]);
    u.z = pack_bf16x2(x[4], x[5]);
    u.w = pack_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(tile + off) = u;
}

// hi/lo halves of 8 consecutive values into two swizzled bf16 tiles.
__device__ __forceinline__ void store_split8(unsigned char* hi_tile, unsigned char* lo_tile, uint32_t off,
                                             const float* x) {
    float h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) split_bf16(x[e], h[e], l[e]);
    store_bf16x8(hi_tile, off, h);
    store_bf16x8(lo_tile, off, l);
}

// fp32 row of 32 values in a [rows][32] block whose 16-byte chunks are swizzled by row % 8.
__device__ __forceinline__ uint32_t f32blk_offset(int row, int chunk4) {
    return (uint32_t)row * 128u + (uint32_t)((chunk4 ^ (row & 7)) * 16);
}

// Issue the row loads of `chunk` into the raw staging (q, k, v: [64 rows][128] bf16 each, rows
// past T zero-filled) and load its g / beta into registers of threads 0-63.
__device__ __forceinline__ void prep_prefetch(const ChunkParams& p, int64_t chunk, unsigned char* raw, int tid,
                                              float& g_next, float& b_next) {
    const int c = (int)(chunk % p.NC);
    const int bh = (int)(chunk / p.NC);
    const int b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    for (int idx = tid; idx < 3 * kChunk * 16; idx += kPrepThreads) {
        const int tsr = idx >> 10, r = (idx >> 4) & 63, j = idx & 15;
        const View4& vw = tsr == 0 ? p.q : (tsr == 1 ? p.k : p.v);
        const int64_t t = t0 + r;
        const bool valid = t < p.T;
        const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(vw.p);
        const void* src = valid ? static_cast<const void*>(base + (int64_t)b * vw.sb + t * vw.st + (int64_t)h * vw.sh + 8 * j)
                                : static_cast<const void*>(base);
        cp_async16(raw + tsr * 16384 + r * 256 + j * 16, src, valid ? 16u : 0u);
    }
    cp_async_commit();
    if (tid < kChunk) {
        const int64_t t = t0 + tid;
        g_next = b_next = 0.f;
        if (t < p.T) {
            g_next = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            b_next = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
    }
}

__global__ void __launch_bounds__(kPrepThreads, 1) gdn_prep_tc(ChunkParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    PrepMisc& ms = *reinterpret_cast<PrepMisc*>(sm + P_MISC);
    float(*sL)[kLd] = reinterpret_cast<float(*)[kLd]>(sm + P_L);
    float(*sA)[kAqkLd] = reinterpret_cast<float(*)[kAqkLd]>(sm + P_AQK);
    float(*sT)[kLd] = reinterpret_cast<float(*)[kLd]>(sm + P_T);
    float(*sY)[16][16] = reinterpret_cast<float(*)[16][16]>(sm + P_Y3);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quad = warp & 3, cq = warp >> 2;  // TMEM lane quadrant, column quarter
    const float scale = rsqrtf((float)kDk);
    const int64_t nchunks = (int64_t)p.B * p.H * p.NC;
    unsigned char* raw = sm + P_RAW;

    if (warp == 0) {
        tmem_alloc(&ms.tmem, kPrepTmemCols);
        tmem_relinquish();
    }
    if (tid == 32) {
        mbar_init(&ms.bar, 1);
        fence_mbar_init();
    }
    float g_next = 0.f, b_next = 0.f;  // g / beta of the chunk whose rows are in flight (threads 0-63)
    if ((int64_t)blockIdx.x < nchunks) prep_prefetch(p, blockIdx.x, raw, tid, g_next, b_next);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);
    bool ok = true;
    int it = 0;

    // Persistent: one CTA per SM walks the chunks, the next chunk's rows landing while this one computes.
    for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x, ++it) {
    const int c = (int)(chunk % p.NC);
    const int64_t t0 = (int64_t)c * kChunk;
    unsigned char* wrec = reinterpret_cast<unsigned char*>(p.ws) + chunk * kTcChunkBytes;
    const uint32_t ph = (uint32_t)it & 1u;  // parity of this chunk's first of three barrier phases

    // ---- 1. normalised rows -> swizzled bf16 tiles (qwen3_5_transformers.py:122-137).
    //      The rows were prefetched; the previous chunk's Q'/o0/M copies must have left L and KQ.
    cp_async_wait_all();
    if (tid == 32) bulk_wait_read_keep1();
    __syncthreads();
    {
        // 8 sums of squares (q and k of 4 rows) reduced together: independent shuffle chains.
        // The inverse norm uses rsqrtf: it is rounded to bf16 right away, so it differs from a
        // correctly rounded 1/sqrt only when it lies within ~2 fp32 ulp of a bf16 rounding boundary
        // (the reference's own CPU bf16 rsqrt is an estimate as well).
        constexpr int kRows = kChunk / (kPrepThreads / 32);
        float q[kRows][4], k[kRows][4], v[kRows][4], ss[2 * kRows];
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
            const int r = warp + 16 * rr;
            const uint2 qu = *reinterpret_cast<const uint2*>(raw + 0 * 16384 + r * 256 + 8 * lane);
            const uint2 ku = *reinterpret_cast<const uint2*>(raw + 1 * 16384 + r * 256 + 8 * lane);
            const uint2 vu = *reinterpret_cast<const uint2*>(raw + 2 * 16384 + r * 256 + 8 * lane);
            const __nv_bfloat162* qb = reinterpret_cast<const __nv_bfloat162*>(&qu);
            const __nv_bfloat162* kb = reinterpret_cast<const __nv_bfloat162*>(&ku);
            const __nv_bfloat162* vb = reinterpret_cast<const __nv_bfloat162*>(&vu);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                q[rr][2 * e] = __low2float(qb[e]);
                q[rr][2 * e + 1] = __high2float(qb[e]);
                k[rr][2 * e] = __low2float(kb[e]);
                k[rr][2 * e + 1] = __high2float(kb[e]);
                v[rr][2 * e] = __low2float(vb[e]);
                v[rr][2 * e + 1] = __high2float(vb[e]);
            }
            float sq = 0.f, sk = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {  // x*x rounded in bf16, summed in fp32 (qwen3_5_transformers.py:106)
                sq += round_to(q[rr][e] * q[rr][e], GDN_BF16);
                sk += round_to(k[rr][e] * k[rr][e], GDN_BF16);
            }
            ss[2 * rr] = sq;
            ss[2 * rr + 1] = sk;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int i = 0; i < 2 * kRows; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], o);
        }
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
            const int r = warp + 16 * rr;
            if (p.l2norm && t0 + r < p.T) {
                const float iq = round_to(rsqrtf(round_to(round_to(ss[2 * rr], GDN_BF16) + 1e-6f, GDN_BF16)), GDN_BF16);
                const float ik = round_to(rsqrtf(round_to(round_to(ss[2 * rr + 1], GDN_BF16) + 1e-6f, GDN_BF16)), GDN_BF16);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    q[rr][e] = round_to(q[rr][e] * iq, GDN_BF16);
                    k[rr][e] = round_to(k[rr][e] * ik, GDN_BF16);
                }
            }
            store_bf16x4(sm + P_KQ, sw128_offset(r, 4 * lane, 128), k[rr]);
            store_bf16x4(sm + P_KQ, sw128_offset(64 + r, 4 * lane, 128), q[rr]);
            store_bf16x4(sm + P_V, sw128_offset(r, 4 * lane, 64), v[rr]);
        }
    }
    if (tid < kChunk) {
        ms.gc[tid] = g_next;
        ms.beta[tid] = b_next;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the raw staging is consumed: pull in the chunk after this one
    if (chunk + gridDim.x < nchunks) prep_prefetch(p, chunk + gridDim.x, raw, tid, g_next, b_next);

    // ---- 2. [k^; q^] k^T -> TMEM cols [0,64): lanes 0-63 G_k = k^ k^T, lanes 64-127 G_q = q^ k^T
    if (tid == 0) {
        const uint32_t id = make_idesc_f16(128, 64, false, false, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint64_t d = make_sdesc(sbase + P_KQ + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128B);
            mma_f16(tm, d, d, id, ks > 0);  // B reads only rows 0-63 (k^) of the same tile
        }
        mma_commit(&ms.bar);
    }
    if (warp == 1) {  // inclusive scan of g over the chunk (:151), two values per lane
        const float g0 = ms.gc[2 * lane], g1 = ms.gc[2 * lane + 1];
        float x = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        ms.gc[2 * lane] = x - g1;
        ms.gc[2 * lane + 1] = x;
    }
    __syncthreads();
    if (tid < kChunk) {
        ms.egc[tid] = __expf(ms.gc[tid]);
        ms.ekd[tid] = __expf(ms.gc[kChunk - 1] - ms.gc[tid]);
    }
    ok = mbar_wait(&ms.bar, ph, kWaitNs);
    tc_fence_after();

    // ---- 3. L = -(beta_i G_k e^(gc_i-gc_j)) strictly lower (:152-153), Aqk = Dk^-1/2 G_q e^(gc_i-gc_j) causal (:172)
    if (!__syncthreads_or(!ok)) {
        float gv[16];
        tmem_ld16(tmem_addr(tm, 32 * quad, 16 * cq), gv);
        tmem_ld_wait();
        const int r = 32 * quad + lane, i = r & 63;
        const float gci = ms.gc[i];
        if (r < 64) {
            const float bi = ms.beta[i];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = 16 * cq + e;
                sL[i][j] = (j < i) ? -(bi * gv[e]) * __expf(gci - ms.gc[j]) : 0.f;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = 16 * cq + e;
                sA[i][j] = (j <= i) ? (scale * gv[e]) * __expf(gci - ms.gc[j]) : 0.f;
            }
        }
    } else {
        ok = false;
    }
    tc_fence_before();
    __syncthreads();

    // ---- 4. T = (I - L)^-1 in 16x16 blocks (the forward substitution of :154-158):
    //      diagonal blocks by substitution, then T_rc = T_rr sum_{k=c}^{r-1} L_rk T_kc by block distance.
    if (ok) {
        if (tid < 64) {
            const int blk = tid >> 4, j = tid & 15, o = 16 * blk;
            float x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
            for (int i = 1; i < 16; ++i) {
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int m = 0; m < i; m += 2) {
                    s0 += sL[o + i][o + m] * x[m];
                    if (m + 1 < i) s1 += sL[o + i][o + m + 1] * x[m + 1];
                }
                x[i] = (i == j) ? 1.f : s0 + s1;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) sT[o + i][o + j] = x[i];
        } else {  // zero the strictly upper blocks
            for (int idx = tid - 64; idx < 6 * 256; idx += kPrepThreads - 64) {
                const int blkid = idx >> 8, e = idx & 255;
                const int rb = blkid < 3 ? 0 : (blkid < 5 ? 1 : 2);
                const int cb = blkid < 3 ? blkid + 1 : (blkid < 5 ? blkid - 1 : 3);
                sT[16 * rb + (e >> 4)][16 * cb + (e & 15)] = 0.f;
            }
        }
    }
    __syncthreads();
    if (ok) {  // distance 1: Y_c = L_{c+1,c} T_cc
        for (int o = tid; o < 768; o += kPrepThreads) {
            const int cb = o >> 8, i = (o >> 4) & 15, j = o & 15;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int m = 0; m < 16; m += 2) {
                s0 += sL[16 * (cb + 1) + i][16 * cb + m] * sT[16 * cb + m][16 * cb + j];
                s1 += sL[16 * (cb + 1) + i][16 * cb + m + 1] * sT[16 * cb + m + 1][16 * cb + j];
            }
            sY[cb][i][j] = s0 + s1;
        }
    }
    __syncthreads();
    if (ok) {  // T_{c+1,c} = T_{c+1,c+1} Y_c
        for (int o = tid; o < 768; o += kPrepThreads) {
            const int cb = o >> 8, i = (o >> 4) & 15, j = o & 15, rb = 16 * (cb + 1);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int m = 0; m < 16; m += 2) {
                s0 += sT[rb + i][rb + m] * sY[cb][m][j];
                s1 += sT[rb + i][rb + m + 1] * sY[cb][m + 1][j];
            }
            sT[rb + i][16 * cb + j] = s0 + s1;
        }
    }
    __syncthreads();
    if (ok) {  // distance 2: Y_c = L_{c+2,c} T_cc + L_{c+2,c+1} T_{c+1,c}
        const int cb = tid >> 8, i = (tid >> 4) & 15, j = tid & 15, rb = 16 * (cb + 2);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            s0 += sL[rb + i][16 * cb + m] * sT[16 * cb + m][16 * cb + j];
            s1 += sL[rb + i][16 * (cb + 1) + m] * sT[16 * (cb + 1) + m][16 * cb + j];
        }
        sY[cb][i][j] = s0 + s1;
    }
    __syncthreads();
    if (ok) {  // T_{c+2,c} = T_{c+2,c+2} Y_c
        const int cb = tid >> 8, i = (tid >> 4) & 15, j = tid & 15, rb = 16 * (cb + 2);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int m = 0; m < 16; m += 2) {
            s0 += sT[rb + i][rb + m] * sY[cb][m][j];
            s1 += sT[rb + i][rb + m + 1] * sY[cb][m + 1][j];
        }
        sT[rb + i][16 * cb + j] = s0 + s1;
    }
    __syncthreads();
    if (ok && tid < 256) {  // distance 3: Y = sum_{k<3} L_{3,k} T_{k,0}
        const int i = tid >> 4, j = tid & 15;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            s0 += sL[48 + i][m] * sT[m][j];
            s1 += sL[48 + i][16 + m] * sT[16 + m][j];
            s2 += sL[48 + i][32 + m] * sT[32 + m][j];
        }
        sY[0][i][j] = s0 + s1 + s2;
    }
    __syncthreads();
    if (ok && tid < 256) {  // T_{3,0} = T_33 Y
        const int i = tid >> 4, j = tid & 15;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int m = 0; m < 16; m += 2) {
            s0 += sT[48 + i][48 + m] * sY[0][m][j];
            s1 += sT[48 + i][48 + m + 1] * sY[0][m + 1][j];
        }
        sT[48 + i][j] = s0 + s1;
    }
    __syncthreads();

    if (tid == 32) bulk_wait_read_all();  // the previous chunk's b copy has left P_SPLIT
    __syncthreads();

    // ---- 5. the four 64x64 coefficient matrices, hi/lo bf16 A tiles [X;Z] and [Y;W]
    //      X = E_d T B_e, Y = E_d T B, W = (Aqk T) B, Z = (Aqk T) B_e
    if (ok) {
        const int i = tid & 63, j0 = (tid >> 6) * 8;
        float at[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) at[e] = 0.f;
        for (int m = j0; m <= i; ++m) {  // (Aqk T)[i][j] = sum_{m=j..i} Aqk[i][m] T[m][j]
            const float a = sA[i][m];
            const float4 t0v = *reinterpret_cast<const float4*>(&sT[m][j0]);
            const float4 t1v = *reinterpret_cast<const float4*>(&sT[m][j0 + 4]);
            at[0] += a * t0v.x;
            at[1] += a * t0v.y;
            at[2] += a * t0v.z;
            at[3] += a * t0v.w;
            at[4] += a * t1v.x;
            at[5] += a * t1v.y;
            at[6] += a * t1v.z;
            at[7] += a * t1v.w;
        }
        const float4 ta = *reinterpret_cast<const float4*>(&sT[i][j0]);
        const float4 tb = *reinterpret_cast<const float4*>(&sT[i][j0 + 4]);
        const float ti[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
        const float ekdi = ms.ekd[i];
        float X[8], Y[8], W[8], Z[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int j = j0 + e;
            const float bj = ms.beta[j], bej = ms.beta[j] * ms.egc[j];
            X[e] = ekdi * ti[e] * bej;
            Y[e] = ekdi * ti[e] * bj;
            W[e] = at[e] * bj;
            Z[e] = at[e] * bej;
        }
        unsigned char* sp = sm + P_SPLIT;
        store_split8(sp + 0 * 16384, sp + 1 * 16384, sw128_offset(i, j0, 128), X);
        store_split8(sp + 0 * 16384, sp + 1 * 16384, sw128_offset(64 + i, j0, 128), Z);
        store_split8(sp + 2 * 16384, sp + 3 * 16384, sw128_offset(i, j0, 128), Y);
        store_split8(sp + 2 * 16384, sp + 3 * 16384, sw128_offset(64 + i, j0, 128), W);
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- 6. [X;Z] k^ -> cols [0,128) (P_X | Zk), [Y;W] v -> cols [128,256) (P_Y | o0); M=128, N=128, K=64, hi+lo
    if (ok && tid == 0) {
        tc_fence_after();
        const uint32_t id = make_idesc_f16(128, 128, false, true, true);
        const uint32_t sp = sbase + P_SPLIT;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t bt = r == 0 ? sbase + P_KQ : sbase + P_V;
            const uint32_t blbo = r == 0 ? 16384 : 8192;
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {  // hi, lo
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t ad = make_sdesc(sp + (2 * r + s2) * 16384 + ks * 32, 16, 1024, kSwizzle128B);
                    const uint64_t bd = make_sdesc(bt + ks * 2048, blbo, 1024, kSwizzle128B);
                    mma_f16(tm + 128 * r, ad, bd, id, (s2 | ks) != 0);
                }
            }
        }
        mma_commit(&ms.bar);
    }
    if (ok) ok = mbar_wait(&ms.bar, ph ^ 1u, kWaitNs);
    tc_fence_after();

    // ---- 7. rows 0-63: P_X, P_Y -> hi/lo B tiles; rows 64-127: Q' and o0 -> workspace
    if (!__syncthreads_or(!ok)) {
        const int r = 32 * quad + lane, i = r & 63;
        unsigned char* sp = sm + P_SPLIT;
        float v[32];
        tmem_ld32(tmem_addr(tm, 32 * quad, 32 * cq), v);
        tmem_ld_wait();
        if (r < 64) {  // P_X (MN-major B tile: rows = tokens)
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8)
                store_split8(sp, sp + 16384, sw128_offset(i, 32 * cq + 8 * q8, 64), v + 8 * q8);
        } else {  // Q' = q^ Dk^-1/2 e^gc - Zk (the q e^gc S of :175 and -Aqk w S of :176 combined)
            const float qs = scale * ms.egc[i];
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
                const int d = 32 * cq + 8 * q8;
                const uint4 qu = *reinterpret_cast<const uint4*>(sm + P_KQ + sw128_offset(64 + i, d, 128));
                const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(&qu);
                float o[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = qs * __bfloat162float(qb[e]) - v[8 * q8 + e];
                store_bf16x8(sm + P_STG_Q, sw128_offset(i, d, 64), o);
            }
        }
        tmem_ld32(tmem_addr(tm, 32 * quad, 128 + 32 * cq), v);
        tmem_ld_wait();
        if (r < 64) {  // P_Y
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8)
                store_split8(sp + 32768, sp + 49152, sw128_offset(i, 32 * cq + 8 * q8, 64), v + 8 * q8);
        } else {  // o0 = Aqk u, fp32 column tile cq
            unsigned char* blk = sm + P_STG_O0 + cq * (64 * 128);
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
                *reinterpret_cast<float4*>(blk + f32blk_offset(i, q4)) =
                    make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        }
    } else {
        ok = false;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (ok && tid == 32) {  // Q' and o0 leave while the tensor core works on step 8
        bulk_s2g(wrec + kTcQ, sm + P_STG_Q, 16384);
        bulk_s2g(wrec + kTcO0, sm + P_STG_O0, 32768);
        bulk_commit();
    }

    // ---- 8. M' = k^T P_X -> [0,128), b = k^T P_Y -> [128,256)  (M=128 over Dk, K = tokens)
    if (ok && tid == 0) {
        const uint32_t id = make_idesc_f16(128, 128, true, true, true);
        const uint32_t sp = sbase + P_SPLIT;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t ad = make_sdesc(sbase + P_KQ + ks * 2048, 16384, 1024, kSwizzle128B);
                    const uint64_t bd = make_sdesc(sp + (2 * r + s2) * 16384 + ks * 2048, 8192, 1024, kSwizzle128B);
                    mma_f16(tm + 128 * r, ad, bd, id, (s2 | ks) != 0);
                }
            }
        }
        mma_commit(&ms.bar);
    }
    if (ok) ok = mbar_wait(&ms.bar, ph, kWaitNs);
    tc_fence_after();

    // ---- 9. M = e^gc_last I - M' (bf16 image), b (fp32 column tiles)
    if (!__syncthreads_or(!ok)) {
        const int dk = 32 * quad + lane;
        const float gamma = ms.egc[kChunk - 1];
        float v[32];
        tmem_ld32(tmem_addr(tm, 32 * quad, 32 * cq), v);
        tmem_ld_wait();
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
            const int col = 32 * cq + 8 * q8;
            float m[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) m[e] = ((col + e) == dk ? gamma : 0.f) - v[8 * q8 + e];
            store_bf16x8(sm + P_STG_M, sw128_offset(dk, col, 128), m);
        }
        tmem_ld32(tmem_addr(tm, 32 * quad, 128 + 32 * cq), v);
        tmem_ld_wait();
        unsigned char* blk = sm + P_STG_B + cq * (128 * 128);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
            *reinterpret_cast<float4*>(blk + f32blk_offset(dk, q4)) =
                make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
    } else {
        ok = false;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 32 && ok) {  // two groups: M (KQ region) then b (P_SPLIT region)
        bulk_s2g(wrec + kTcM, sm + P_STG_M, 32768);
        bulk_commit();
        bulk_s2g(wrec + kTcB, sm + P_STG_B, 65536);
        bulk_commit();
    }
    if (!ok) break;
    }  // chunk loop
    if (tid == 32) bulk_wait_read_all();  // shared memory must outlive every copy that reads it
    cp_async_wait_all();                 // and every prefetch that writes it
    if (!ok && tid == 0) report(p.err, kErrTimeoutPrep);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, kPrepTmemCols);
}

// ============================================================================ scan

constexpr int kScanThreads = 192;          // warps 0-3: state/output epilogue (thread 0 issues the MMAs),
                                           // 4: M/Q bulk copies + L2 prefetch, 5: b/o0 bulk copies
constexpr int kScanPrefetch = 4;           // chunks ahead that the producer pulls into L2
constexpr int kScanIssuer = 16;            // warp 0 lane 16: issues the MMAs (lanes 16-31 own no output rows)
constexpr uint32_t kScanTmemCols = 128;    // cols [0,32) state accumulator, [32,64) / [64,96) output accumulators
constexpr uint32_t S_STAGE = 73728;        // M image 32K | Q image 16K | b slice 16K | o0 slice 8K
constexpr uint32_t S_OFF_Q = 32768, S_OFF_B = 49152, S_OFF_O0 = 65536;
constexpr uint32_t S_STILE = 2 * S_STAGE;  // state operand, two tiles by chunk parity: bf16 [128 dk][64] swizzled
                                           // (32 columns used); chunk c's MMAs read tile c % 2
constexpr uint32_t S_MISC = S_STILE + 2 * 16384;
constexpr uint32_t S_SMEM = S_MISC + 256 + 1024;

struct ScanMisc {
    uint64_t full_mq[2];   // M/Q images landed (tx)
    uint64_t full_bo[2];   // b/o0 slices landed (tx)
    uint64_t empty_mq[2];  // the MMAs that read M/Q completed (tcgen05.commit)
    uint64_t empty_bo[2];  // the epilogue read b and o0 (128 arrivals)
    uint64_t mma_s;        // state accumulator of this chunk ready
    uint64_t mma_o[2];     // output accumulator of chunk c ready, alternating by chunk parity
    uint32_t tmem;
    int abort;
};

// Named barrier over `nthreads` threads that also returns whether any of them passed `flag` != 0,
// so a failure seen by one thread ends the loop of all of them together.
__device__ __forceinline__ bool named_barrier_any(uint32_t id, uint32_t nthreads, bool flag) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)flag), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// o_c rows 16w..16w+15 of this CTA's 32 columns: o = Q'S (accumulator) + o0 (stage smem).
__device__ __forceinline__ void scan_store_output(const ChunkParams& p, const unsigned char* st, const float (&o)[32],
                                                  int c, int warp, int lane, int b, int h, int dv0) {
    if (lane >= 16) return;
    const int tok = 16 * warp + lane;
    const int64_t t = (int64_t)c * kChunk + tok;
    if (t >= p.T) return;
    float ov[32];
#pragma unroll
    for (int q4 = 0; q4 < 8; ++q4) {
        const float4 oo = *reinterpret_cast<const float4*>(st + S_OFF_O0 + f32blk_offset(tok, q4));
        ov[4 * q4] = o[4 * q4] + oo.x;
        ov[4 * q4 + 1] = o[4 * q4 + 1] + oo.y;
        ov[4 * q4 + 2] = o[4 * q4 + 2] + oo.z;
        ov[4 * q4 + 3] = o[4 * q4 + 3] + oo.w;
    }
    unsigned char* dst = reinterpret_cast<unsigned char*>(p.out) +
                         2 * ((int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + dv0);
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) store_bf16x8(dst, 16 * q8, ov + 8 * q8);
}

__global__ void __launch_bounds__(kScanThreads, 1) gdn_scan_tc(ChunkParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    ScanMisc& ms = *reinterpret_cast<ScanMisc*>(sm + S_MISC);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh % p.H;
    const int dvt = blockIdx.y & 3;  // 32-column slice of the state (and of b / o0)
    const bool summary = p.scan_mode == 1;
    const bool transition = summary && blockIdx.y < 4;  // state starts from I, b ignored
    const int dv0 = dvt * kTcDvTile;
    const unsigned char* wbase = reinterpret_cast<const unsigned char*>(p.ws) + (int64_t)bh * p.NC * kTcChunkBytes;

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ms.full_mq[s], 1);
            mbar_init(&ms.full_bo[s], 1);
            mbar_init(&ms.empty_mq[s], 1);
            mbar_init(&ms.empty_bo[s], 128);
        }
        mbar_init(&ms.mma_s, 1);
        mbar_init(&ms.mma_o[0], 1);
        mbar_init(&ms.mma_o[1], 1);
        ms.abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kScanTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);
    bool ok = true;

    if (warp >= 4) {
        // ---------------- producers: warp 4 streams the M/Q images, warp 5 the b/o0 slices
        if (lane == 0) {
            const bool mq = warp == 4;
            uint64_t* full = mq ? ms.full_mq : ms.full_bo;
            uint64_t* empty = mq ? ms.empty_mq : ms.empty_bo;
            const uint32_t bytes = mq ? 32768 + 16384 : 16384 + 8192;
            int issued = 0;
            for (int c = 0; c < p.NC; ++c) {
                const int s = c & 1;
                if (mq && c + kScanPrefetch < p.NC) {
                    const unsigned char* pre = wbase + (int64_t)(c + kScanPrefetch) * kTcChunkBytes;
                    bulk_prefetch_l2(pre + kTcM, 32768 + 16384);
                    bulk_prefetch_l2(pre + kTcB + dvt * 16384, 16384);
                    bulk_prefetch_l2(pre + kTcO0 + dvt * 8192, 8192);
                }
                if (c >= 2 && !mbar_wait(&empty[s], ((c >> 1) - 1) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                if (ms.abort) break;
                const unsigned char* rec = wbase + (int64_t)c * kTcChunkBytes;
                unsigned char* st = sm + s * S_STAGE;
                mbar_arrive_expect_tx(&full[s], bytes);
                if (mq) {
                    bulk_g2s(st, rec + kTcM, 32768, &full[s]);
                    bulk_g2s(st + S_OFF_Q, rec + kTcQ, 16384, &full[s]);
                } else {
                    bulk_g2s(st + S_OFF_B, rec + kTcB + dvt * 16384, 16384, &full[s]);
                    bulk_g2s(st + S_OFF_O0, rec + kTcO0 + dvt * 8192, 8192, &full[s]);
                }
                ++issued;
            }
            // leave no copy in flight: wait for the last record of each stage to land
            for (int c = (issued > 2 ? issued - 2 : 0); c < issued; ++c)
                if (!mbar_wait(&full[c & 1], (c >> 1) & 1, kWaitNs)) ok = false;
        }
    } else {
        // ---------------- thread = state row dk (TMEM lane); warp w also owns output rows 16w..16w+15
        const int dk = tid;
        float S[kTcDvTile];
        const int64_t srow = ((int64_t)bh * kDk + dk) * kDv + dv0;
#pragma unroll
        for (int q4 = 0; q4 < kTcDvTile / 4; ++q4) {
            float4 v = (p.h0 && !summary) ? *reinterpret_cast<const float4*>(p.h0 + srow + 4 * q4)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
            if (transition) {  // identity columns dv0 .. dv0+31
                v.x = (dk == dv0 + 4 * q4) ? 1.f : 0.f;
                v.y = (dk == dv0 + 4 * q4 + 1) ? 1.f : 0.f;
                v.z = (dk == dv0 + 4 * q4 + 2) ? 1.f : 0.f;
                v.w = (dk == dv0 + 4 * q4 + 3) ? 1.f : 0.f;
            }
            S[4 * q4] = v.x;
            S[4 * q4 + 1] = v.y;
            S[4 * q4 + 2] = v.z;
            S[4 * q4 + 3] = v.w;
        }
        unsigned char* stile = sm + S_STILE;
#pragma unroll
        for (int q8 = 0; q8 < kTcDvTile / 8; ++q8) store_bf16x8(stile, sw128_offset(dk, 8 * q8, 128), S + 8 * q8);
        fence_proxy_async_smem();

        // descriptors of stage 0 / k-step 0; the others differ only in the start address
        const uint32_t idS = make_idesc_f16(128, kTcDvTile, false, true, true);
        const uint32_t idO = make_idesc_f16(64, kTcDvTile, false, true, true);
        const uint64_t dM = make_sdesc(sbase, 16, 1024, kSwizzle128B);
        const uint64_t dQ = make_sdesc(sbase + S_OFF_Q, 16, 1024, kSwizzle128B);
        const uint64_t dS = make_sdesc(sbase + S_STILE, 16384, 1024, kSwizzle128B);

        for (int c = 0; c < p.NC; ++c) {
            const int s = c & 1;
            // every row of S_c is in the operand tile; leave together if any thread failed a wait
            if (named_barrier_any(1, 128, !ok)) {
                ok = false;
                break;
            }
            if (tid == kScanIssuer) {
                if (!mbar_wait(&ms.full_mq[s], (c >> 1) & 1, kWaitNs)) {
                    ms.abort = 1;  // no MMA this chunk: every thread's wait below gives up
                } else {
                    tc_fence_after();
                    const uint64_t so = (uint64_t)((s * S_STAGE) >> 4);
                    // state first: it is the only product on the sequential path
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16(tm + 0, dM + so + (uint64_t)((((ks >> 2) * 16384) + (ks & 3) * 32) >> 4),
                                dS + (uint64_t)((s * 16384 + ks * 2048) >> 4), idS, ks > 0);
                    mma_commit(&ms.mma_s);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        mma_f16(tm + kTcDvTile * (1 + s), dQ + so + (uint64_t)((((ks >> 2) * 8192) + (ks & 3) * 32) >> 4),
                                dS + (uint64_t)((s * 16384 + ks * 2048) >> 4), idO, ks > 0);
                    mma_commit(&ms.mma_o[s]);
                    mma_commit(&ms.empty_mq[s]);
                }
            }
            // previous chunk's output rows, overlapping this chunk's MMAs
            if (c > 0) {
                const int sp = (c - 1) & 1;
                if (!mbar_wait(&ms.mma_o[sp], ((c - 1) >> 1) & 1, kWaitNs)) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                float o[32];
                tmem_ld32(tmem_addr(tm, 32 * warp, kTcDvTile * (1 + sp)), o);
                tmem_ld_wait();
                if (!summary) scan_store_output(p, sm + sp * S_STAGE, o, c - 1, warp, lane, b, h, dv0);
                mbar_arrive(&ms.empty_bo[sp]);
            }
            if (!mbar_wait(&ms.mma_s, c & 1, kWaitNs) || !mbar_wait(&ms.full_bo[s], (c >> 1) & 1, kWaitNs)) {
                ok = false;
                continue;  // the barrier at the top of the loop ends every thread's loop
            }
            tc_fence_after();
            float d[32];
            tmem_ld32(tmem_addr(tm, 32 * warp, 0), d);
            tmem_ld_wait();
            const unsigned char* st = sm + s * S_STAGE;
            // S_{c+1} = M_c S_c + b_c
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
                float4 bb = *reinterpret_cast<const float4*>(st + S_OFF_B + f32blk_offset(dk, q4));
                if (transition) bb = make_float4(0.f, 0.f, 0.f, 0.f);
                S[4 * q4] = d[4 * q4] + bb.x;
                S[4 * q4 + 1] = d[4 * q4 + 1] + bb.y;
                S[4 * q4 + 2] = d[4 * q4 + 2] + bb.z;
                S[4 * q4 + 3] = d[4 * q4 + 3] + bb.w;
            }
            if (c + 1 < p.NC) {  // tile (c+1) % 2 was last read by chunk c-1's MMAs, all complete
#pragma unroll
                for (int q8 = 0; q8 < kTcDvTile / 8; ++q8)
                    store_bf16x8(stile + (s ^ 1) * 16384, sw128_offset(dk, 8 * q8, 128), S + 8 * q8);
                fence_proxy_async_smem();
            }
            tc_fence_before();
        }
        if (ok) {
            const int sp = (p.NC - 1) & 1;
            if (mbar_wait(&ms.mma_o[sp], ((p.NC - 1) >> 1) & 1, kWaitNs)) {
                tc_fence_after();
                float o[32];
                tmem_ld32(tmem_addr(tm, 32 * warp, kTcDvTile * (1 + sp)), o);
                tmem_ld_wait();
                if (!summary) scan_store_output(p, sm + sp * S_STAGE, o, p.NC - 1, warp, lane, b, h, dv0);
                mbar_arrive(&ms.empty_bo[sp]);
            } else {
                ok = false;
            }
            float* dst = summary ? (transition ? p.hT : p.hT2) : p.hT;
            if (ok && dst) {
#pragma unroll
                for (int q4 = 0; q4 < kTcDvTile / 4; ++q4)
                    *reinterpret_cast<float4*>(dst + srow + 4 * q4) =
                        make_float4(S[4 * q4], S[4 * q4 + 1], S[4 * q4 + 2], S[4 * q4 + 3]);
            }
        }
    }
    if (!ok) {
        ms.abort = 1;
        report(p.err, kErrTimeoutScan);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, kScanTmemCols);
}

}  // namespace

cudaError_t launch_chunk_tc_prep(const ChunkParams& p, cudaStream_t stream) {
    static_assert(P_SMEM <= 227 * 1024 && S_SMEM <= 227 * 1024, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(gdn_prep_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM);
    if (e != cudaSuccess) return e;
    const int64_t nchunks = (int64_t)p.B * p.H * p.NC;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const unsigned prep_grid = (unsigned)(nchunks < (int64_t)sms ? nchunks : (int64_t)sms);
    gdn_prep_tc<<<prep_grid, kPrepThreads, P_SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

cudaError_t launch_chunk_tc_scan(const ChunkParams& p, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(gdn_scan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S_SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)(p.B * p.H), (p.scan_mode == 1 ? 2 : 1) * (kDv / kTcDvTile));
    gdn_scan_tc<<<grid, kScanThreads, S_SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

cudaError_t launch_chunk_tc(const ChunkParams& p, cudaStream_t stream) {
    cudaError_t e;
    if ((e = phase_event(0, stream)) != cudaSuccess) return e;
    if ((e = launch_chunk_tc_prep(p, stream)) != cudaSuccess) return e;
    if ((e = phase_event(1, stream)) != cudaSuccess) return e;
    if ((e = launch_chunk_tc_scan(p, stream)) != cudaSuccess) return e;
    return phase_event(2, stream);
}

}  // namespace gdn
