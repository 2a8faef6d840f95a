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
// gdn_prep_tc: one CTA (16 warps) per (batch, head, 64-token chunk), two CTAs per
// SM (105 KB of shared memory each, one work region reused phase by phase), so
// one CTA's memory and barrier waits overlap the other's work; the bf16 images
// leave with asynchronous bulk copies, the fp32 tiles straight from TMEM.
// Operands that share a B matrix are stacked into M=128 MMAs so every
// accumulator fills all 128 TMEM lanes.
//   1. rows of q, k, v (three TMA boxes of the caller's view at entry) ->
//      l2norm (16-bit rounding as the reference) -> bf16 128B-swizzled tiles
//      [k^; q^] and v in shared memory
//   2. [k^; q^] k^T on the tensor cores -> G_k (lanes 0-63) and G_q (64-127)
//   3. L = -(beta G_k e^(gc_i-gc_j)) strictly lower, Aqk = Dk^-1/2 G_q e^(gc_i-gc_j) causal
//   4. T = (I - L)^-1 in 16x16 blocks (diagonal blocks by substitution, then
//      the off-diagonal blocks by distance)
//   5. Aqk T on the tensor cores (M=64, N=64, K=64, hi/lo operands); then
//      X = T B_e, Y = T B, W = Aqk T B, Z = Aqk T B_e  (64x64, fp32)
//   6. [X; Z] k^ -> w | Zk, then [Y; W] v -> u | o0  (M=128, N=128, K=64, hi+lo)
//   7. Q' = q^ e^gc Dk^-1/2 - Zk, o0 -> workspace; P_X = E_d w, P_Y = E_d u -> hi+lo
//      B tiles (E_d = diag e^(gc_last - gc))
//   8. M' = k^T P_X, b = k^T P_Y (M=128, N=128, K=64, hi+lo)
//   9. M = e^gc_last I - M', b -> workspace
// gdn_scan_tc: one CTA per (batch, head, 32-column slice of Dv); warps 4-5
//   bulk-copy each chunk's workspace record (double-buffered, the M/Q half freed
//   as soon as the tensor core has read it, records pulled into L2 four chunks
//   ahead); warps 0-3 turn the state accumulator into the next state and signal
//   warp 6, which issues the next chunk's state MMAs as soon as that state is in
//   shared memory (then the output MMAs, into alternating TMEM columns) from one
//   elected lane of a converged warp; a chunk's output rows are written after
//   the next state has been handed over, while the next chunk's MMAs run.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "gdn_bwd.cuh"
#include "gdn_common.cuh"
#include "gdn_internal.h"
#include "gdn_tc.cuh"

namespace gdn {
namespace {

using namespace tc;

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s; a healthy wait here takes microseconds

__device__ __forceinline__ void report(unsigned int* err, unsigned int bit) { report_device_error(err, bit); }

// The scans hand each chunk's state to their MMA-issue warp through a named barrier: the state warps arrive
// (bar.arrive), the MMA warp waits (bar.sync) and then stores the number of barrier steps it has passed in
// `synced`.  A state warp that has given up (a failed wait) still takes every arrival, so that the MMA warp's
// syncs are never short of one, but first waits here until the MMA warp has passed the previous step.  The
// barrier counts threads, not steps: without this wait a warp that skips its work could arrive twice while
// another has not arrived once, complete a step without the MMA warp and leave its last sync waiting for good.
// The MMA warp waits on nothing unbounded except that barrier, so the wait ends; it is bounded all the same.
__device__ __forceinline__ void wait_barrier_step(const int* synced, int step) {
    const long long t0 = clock64();
    while (*reinterpret_cast<const volatile int*>(synced) < step && clock64() - t0 < (long long)(kWaitNs * 2)) {
    }
}
__device__ __forceinline__ void mark_barrier_step(int* synced, int step, int lane) {
    if (lane == 0) *reinterpret_cast<volatile int*>(synced) = step;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// ============================================================================ prep

constexpr int kPrepThreads = 512;          // 16 warps; two CTAs share an SM (32 warps to hide latency)
constexpr int kPrepWarps = kPrepThreads / 32;
constexpr int kL2Rows = 2;                              // rows a warp normalises together
constexpr int kL2Batches = kChunk / (kL2Rows * kPrepWarps);
constexpr uint32_t P_KQ = 0;               // bf16 [128 rows][128] swizzled: rows 0-63 k^, 64-127 q^ (atom columns 16 KiB apart)
constexpr uint32_t P_V = 32768;            // bf16 [64 rows][128] swizzled v (atom columns 8 KiB apart)
constexpr uint32_t P_W = 49152;            // work region, reused phase by phase:
constexpr int kLd = 68;                    //   fp32 row stride of T (16-byte rows for float4 reads)
constexpr int kSLd = 65;                   //   odd stride of L (scalar access only)
constexpr uint32_t P_RAW = P_W;            //   step 1: raw q/k/v rows, [3][64][256 B] (48 KiB)
constexpr uint32_t P_AQK = P_W;            //   steps 3-5: Aqk as hi/lo bf16 A tiles [64][64] (2 x 8 KiB)
constexpr uint32_t P_L = P_W + 16384;      //   steps 3-4: L   fp32 [64][65]
constexpr uint32_t P_TT = P_W + 16384;     //   step 5: T as hi/lo bf16 B tiles [64][64] (2 x 8 KiB; L is dead)
constexpr uint32_t P_T = P_W + 33024;      //   steps 4-5: T   fp32 [64][68]
constexpr uint32_t P_Y3 = P_W + 50432;     //   step 4: fp32 [3][16][16] scratch of the blocked inverse
constexpr uint32_t P_ATILE = P_W;          //   step 6: [X;Z] then [Y;W] hi/lo A tiles (2 x 16 KiB)
constexpr uint32_t P_PX = P_W;             //   steps 7-8: P_X hi/lo B tiles (2 x 16 KiB)
constexpr uint32_t P_PYH = P_V;            //   steps 7-8: P_Y hi (v is dead after step 6)
constexpr uint32_t P_PYL = P_W + 32768;    //   steps 7-8: P_Y lo
constexpr uint32_t P_MISC = P_W + 53760;
constexpr uint32_t P_SMEM = P_MISC + 1088 + 1024;  // + alignment slack
constexpr uint32_t kPrepTmemCols = 256;
static_assert(P_Y3 + 3072 <= P_MISC, "work region");
static_assert(P_L + 64 * kSLd * 4 <= P_T && P_RAW + 3 * 64 * 256 <= P_MISC, "work region");
static_assert(P_PYL + 16384 <= P_MISC, "work region");

struct PrepMisc {
    float gc[64];
    float beta[64];
    float egc[64];
    float ekd[64];
    uint64_t bar;
    uint64_t bar_in;  // the q/k/v boxes landed (TMA)
    uint32_t tmem;
};

// Tensor maps of q, k and v for the prep's input boxes: 4-D over (D, H, T, B) of the caller's bf16 view, box
// (128, 1, 64, 1) = the 64 token rows of one (batch, head, chunk) as 256-byte rows.  `use` = 0: the maps could
// not be encoded (e.g. a stride of 0) and the rows are staged with per-thread cp.async copies instead.
struct PrepMaps {
    CUtensorMap m[3];
    int use;
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

// hi/lo halves of 8 consecutive values into two swizzled bf16 tiles: each pair is rounded to bf16 once (hi),
// the exact remainders x - hi are rounded again (lo).
__device__ __forceinline__ void store_split8(unsigned char* hi_tile, unsigned char* lo_tile, uint32_t off,
                                             const float* x) {
    uint4 hu, lu;
    uint32_t* hp = &hu.x;
    uint32_t* lp = &lu.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(x[2 * e], x[2 * e + 1]);
        const float2 hf = __bfloat1622float2(hb);
        const __nv_bfloat162 lb = __floats2bfloat162_rn(x[2 * e] - hf.x, x[2 * e + 1] - hf.y);
        hp[e] = *reinterpret_cast<const uint32_t*>(&hb);
        lp[e] = *reinterpret_cast<const uint32_t*>(&lb);
    }
    *reinterpret_cast<uint4*>(hi_tile + off) = hu;
    *reinterpret_cast<uint4*>(lo_tile + off) = lu;
}


// The backward tiles (u, w, Kd [64][128]; Aqk [64][64]) as the tensor-core prep writes them: chunk-major,
// element (row, col) at ((col / 4) * 64 + row) * 4 + col % 4, so the prep's stores from TMEM (a lane per
// row, four columns per store) write 512 contiguous bytes per warp.
__host__ __device__ constexpr int64_t cm_offset(int row, int col) { return ((int64_t)(col >> 2) * 64 + row) * 4 + (col & 3); }

// Row `row`, columns col0 .. col0+15 of a chunk-major backward tile.
__device__ __forceinline__ void store_cm16(float* tile, int row, int col0, const float* v) {
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<float4*>(tile + cm_offset(row, col0 + 4 * q4)) =
            make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
}

// Rows held one per lane (lane l: row l of a 32-row block, kN fp32 values in v) stored to global rows
// g + l * ld through the warp's staging tile [32][kN + 4]: each store instruction then writes whole
// 128-byte lines instead of 32 lines a 16-byte piece each.
// kRows < 32: only lanes 0 .. kRows-1 hold rows (an M=64 accumulator's lanes).
template <int kN, int kRows = 32>
__device__ __forceinline__ void store_rows_coalesced(float* stage, const float* v, float* g, int64_t ld, int lane) {
    constexpr int kS = kN + 4, kC = kN / 4;  // padded row stride; 16-byte pieces per row
    if (lane < kRows) {
#pragma unroll
        for (int q4 = 0; q4 < kC; ++q4)
            *reinterpret_cast<float4*>(stage + lane * kS + 4 * q4) =
                make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kRows * kC / 32; ++j) {
        const int idx = 32 * j + lane, row = idx / kC, piece = idx % kC;
        *reinterpret_cast<float4*>(g + row * ld + 4 * piece) = *reinterpret_cast<const float4*>(stage + row * kS + 4 * piece);
    }
    __syncwarp();  // the tile may be rewritten by the next call
}

__device__ __forceinline__ void load_bf16x4_smem(const unsigned char* src, float (&x)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    x[0] = __low2float(lo);
    x[1] = __high2float(lo);
    x[2] = __low2float(hi);
    x[3] = __high2float(hi);
}

// One M=128, N=128, K=64 product accumulated from the hi and lo halves of a K-major A tile
// (single atom column, 128 rows) against an MN-major B tile (rows = the 64 tokens).
__device__ __forceinline__ void mma_split_a(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_tile,
                                            uint32_t b_lbo, uint32_t idesc) {
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            mma_f16(d_tmem, make_sdesc((s2 ? a_lo : a_hi) + ks * 32, 16, 1024, kSwizzle128B),
                    make_sdesc(b_tile + ks * 2048, b_lbo, 1024, kSwizzle128B), idesc, (s2 | ks) != 0);
}

__global__ void __launch_bounds__(kPrepThreads, 2) gdn_prep_tc(ChunkParams p, const __grid_constant__ PrepMaps maps) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    PrepMisc& ms = *reinterpret_cast<PrepMisc*>(sm + P_MISC);
    float(*sL)[kSLd] = reinterpret_cast<float(*)[kSLd]>(sm + P_L);
    float(*sT)[kLd] = reinterpret_cast<float(*)[kLd]>(sm + P_T);
    float(*sY)[16][16] = reinterpret_cast<float(*)[16][16]>(sm + P_Y3);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quad = warp & 3, part = warp >> 2;  // TMEM lane quadrant, 16-column part of each 64
    // Chunks run latest first across all heads (block i -> chunk NC-1 - i/(B*H)), so the records the scan
    // reads first are the ones written last, still in L2 when the scan starts (a long sequence's records
    // do not all fit).  t0 is the chunk's first token, t_lim the end of its sequence.
    int b, h;
    int64_t chunk, t0, t_lim;  // record index, token range
    if (!p.cu_seqlens) {
        const int BH = p.B * p.H;
        const int c = p.NC - 1 - (int)(blockIdx.x / BH);
        const int bh = (int)(blockIdx.x % BH);
        chunk = (int64_t)bh * p.NC + c;
        b = bh / p.H;
        h = bh % p.H;
        t0 = (int64_t)c * kChunk;
        t_lim = p.T;
    } else {  // packed sequences: global chunk j (latest first), record j * H + h; the grid is a bound
        const int j = p.max_chunks - 1 - (int)(blockIdx.x / p.H);
        h = (int)(blockIdx.x % p.H);
        if (j >= p.chunk_base[p.N]) return;  // the whole CTA, before any barrier
        const int n = p.chunk_seq[j];
        b = 0;
        chunk = (int64_t)j * p.H + h;
        t0 = (int64_t)p.cu_seqlens[n] + (int64_t)(j - p.chunk_base[n]) * kChunk;
        t_lim = p.cu_seqlens[n + 1];
    }
    const float scale = rsqrtf((float)kDk);
    unsigned char* wrec = reinterpret_cast<unsigned char*>(p.ws) + chunk * kTcChunkBytes;

    // raw q/k/v rows of the chunk into the (still unused) work region [3][64 rows][256 B]: three TMA boxes
    // (rows past T read as zero), or without tensor maps 3 x 64 rows x 16 pieces of 16 bytes, 12 per thread,
    // all in flight at once (rows past the sequence's end zero-filled)
    if (tid == 32) {
        mbar_init(&ms.bar, 1);
        mbar_init(&ms.bar_in, 1);
        fence_mbar_init();
        if (maps.use) {
            mbar_arrive_expect_tx(&ms.bar_in, 3 * kChunk * 256);
#pragma unroll
            for (int tsr = 0; tsr < 3; ++tsr)
                tma_load_4d(sm + P_RAW + tsr * kChunk * 256, &maps.m[tsr], 0, h, (int)t0, b, &ms.bar_in);
        }
    }
    if (!maps.use) {
        for (int i = tid; i < 3 * kChunk * 16; i += kPrepThreads) {
            const int tsr = i >> 10, row = (i >> 4) & 63, piece = i & 15;
            const View4& V = tsr == 0 ? p.q : (tsr == 1 ? p.k : p.v);
            const int64_t t = t0 + row;
            const bool in = t < t_lim;
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(V.p) + (int64_t)b * V.sb +
                                       (in ? t : t0) * V.st + (int64_t)h * V.sh + 8 * piece;
            cp_async16(sm + P_RAW + (tsr * kChunk + row) * 256 + piece * 16, src, in ? 16u : 0u);
        }
        cp_async_commit();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kPrepTmemCols);
        tmem_relinquish();
    }
    if (tid < kChunk) {  // g, beta of the chunk (rows past the sequence's end are the zero padding)
        const int64_t t = t0 + tid;
        float gv = 0.f, bv = 0.f;
        if (t < t_lim) {
            gv = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            bv = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
        ms.gc[tid] = gv;
        ms.beta[tid] = bv;
    }

    bool in_ok = true;
    if (maps.use) {
        __syncthreads();  // the barrier is initialised before anyone waits on it
        in_ok = mbar_wait(&ms.bar_in, 0, kWaitNs);
        if (t0 + kChunk > t_lim) {  // a packed sequence's last chunk: the rows past its end belong to the next
            const int valid = (int)(t_lim - t0);
            for (int i = tid; i < 3 * kChunk * 16; i += kPrepThreads) {
                const int tsr = i >> 10, row = (i >> 4) & 63, piece = i & 15;
                if (row >= valid)
                    *reinterpret_cast<uint4*>(sm + P_RAW + (tsr * kChunk + row) * 256 + piece * 16) = make_uint4(0, 0, 0, 0);
            }
        }
    } else {
        cp_async_wait_all();
    }
    __syncthreads();
    // ---- 1. normalised rows -> swizzled bf16 tiles (qwen3_5_transformers.py:122-137).
    //      Each warp owns 4 rows of the staged copy, in batches of 2 whose 4 sums of squares are
    //      reduced together.  The inverse norm uses rsqrtf before its
    //      bf16 rounding: it differs from a correctly rounded 1/sqrt only within ~2 fp32 ulp of a bf16
    //      rounding boundary (the reference's own CPU bf16 rsqrt is an estimate as well).
#pragma unroll
    for (int batch = 0; batch < kL2Batches; ++batch) {
        constexpr int kRows = kL2Rows;
        float q[kRows][4], k[kRows][4], v[kRows][4], ss[2 * kRows];
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
            const int row = warp + kPrepWarps * (kRows * batch + rr);
            load_bf16x4_smem(sm + P_RAW + (0 * kChunk + row) * 256 + 8 * lane, q[rr]);
            load_bf16x4_smem(sm + P_RAW + (1 * kChunk + row) * 256 + 8 * lane, k[rr]);
            load_bf16x4_smem(sm + P_RAW + (2 * kChunk + row) * 256 + 8 * lane, v[rr]);
        }
#pragma unroll
        for (int rr = 0; rr < kRows; ++rr) {
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
            const int r = warp + kPrepWarps * (kRows * batch + rr);
            if (p.l2norm && t0 + r < t_lim) {
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
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);

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
        const float gc0 = x - g1, gcl = __shfl_sync(0xffffffffu, x, 31);  // gc_last: lane 31's sum
        ms.gc[2 * lane] = gc0;
        ms.gc[2 * lane + 1] = x;
        ms.egc[2 * lane] = __expf(gc0);
        ms.egc[2 * lane + 1] = __expf(x);
        ms.ekd[2 * lane] = __expf(gcl - gc0);
        ms.ekd[2 * lane + 1] = __expf(gcl - x);
    }
    bool ok = mbar_wait(&ms.bar, 0, kWaitNs) && in_ok;  // the barrier below publishes gc, e^gc and e^(gc_last - gc)
    tc_fence_after();

    // ---- 3. L = -(beta_i G_k e^(gc_i-gc_j)) strictly lower (:152-153), Aqk = Dk^-1/2 G_q e^(gc_i-gc_j) causal (:172)
    if (!__syncthreads_or(!ok)) {
        float gv[16];
        tmem_ld16(tmem_addr(tm, 32 * quad, 16 * part), gv);
        tmem_ld_wait();
        const int r = 32 * quad + lane, i = r & 63;
        const float gci = ms.gc[i];
        if (r < 64) {
            const float bi = ms.beta[i];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = 16 * part + e;
                sL[i][j] = (j < i) ? -(bi * gv[e]) * __expf(gci - ms.gc[j]) : 0.f;
            }
        } else {  // Aqk rows as the hi/lo bf16 A operand of step 5 (K-major, one atom column)
            float a[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = 16 * part + e;
                a[e] = (j <= i) ? (scale * gv[e]) * __expf(gci - ms.gc[j]) : 0.f;
            }
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8)
                store_split8(sm + P_AQK, sm + P_AQK + 8192, sw128_offset(i, 16 * part + 8 * q8, 64), a + 8 * q8);
            if (p.bwd_tiles) store_cm16(p.bwd_tiles + chunk * kWsChunkFloats + kWsAqk, i, 16 * part, a);
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
    // Off-diagonal blocks, each output a 1x4 register tile (row i, columns jg..jg+3): one L load and one
    // float4 T load per four FMAs.  sY holds 16x16 fp32 blocks.
    auto f4fma = [](float4& acc, float a, const float4 t) {
        acc.x += a * t.x;
        acc.y += a * t.y;
        acc.z += a * t.z;
        acc.w += a * t.w;
    };
    const int mi = (tid >> 2) & 15, mj = 4 * (tid & 3), mg = tid >> 6;  // row, column group, block of a thread
    if (ok && mg < 3) {  // distance 1: Y_c = L_{c+1,c} T_cc, c = mg
        const int ro = 16 * (mg + 1), co = 16 * mg;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m)
            f4fma(acc, sL[ro + mi][co + m], *reinterpret_cast<const float4*>(&sT[co + m][co + mj]));
        *reinterpret_cast<float4*>(&sY[mg][mi][mj]) = acc;
    }
    __syncthreads();
    if (ok && mg < 3) {  // T_{c+1,c} = T_{c+1,c+1} Y_c
        const int ro = 16 * (mg + 1), co = 16 * mg;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m)
            f4fma(acc, sT[ro + mi][ro + m], *reinterpret_cast<const float4*>(&sY[mg][m][mj]));
        *reinterpret_cast<float4*>(&sT[ro + mi][co + mj]) = acc;
    }
    __syncthreads();
    if (ok && mg < 2) {  // distance 2: Y_c = L_{c+2,c} T_cc + L_{c+2,c+1} T_{c+1,c}, c = mg
        const int ro = 16 * (mg + 2), co = 16 * mg;
        float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            f4fma(acc0, sL[ro + mi][co + m], *reinterpret_cast<const float4*>(&sT[co + m][co + mj]));
            f4fma(acc1, sL[ro + mi][co + 16 + m], *reinterpret_cast<const float4*>(&sT[co + 16 + m][co + mj]));
        }
        *reinterpret_cast<float4*>(&sY[mg][mi][mj]) =
            make_float4(acc0.x + acc1.x, acc0.y + acc1.y, acc0.z + acc1.z, acc0.w + acc1.w);
    }
    __syncthreads();
    if (ok && mg < 2) {  // T_{c+2,c} = T_{c+2,c+2} Y_c
        const int ro = 16 * (mg + 2), co = 16 * mg;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m)
            f4fma(acc, sT[ro + mi][ro + m], *reinterpret_cast<const float4*>(&sY[mg][m][mj]));
        *reinterpret_cast<float4*>(&sT[ro + mi][co + mj]) = acc;
    }
    __syncthreads();
    if (ok && mg < 3) {  // distance 3: the three terms L_{3,k} T_{k,0}, k = mg, summed in the next stage
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m)
            f4fma(acc, sL[48 + mi][16 * mg + m], *reinterpret_cast<const float4*>(&sT[16 * mg + m][mj]));
        *reinterpret_cast<float4*>(&sY[mg][mi][mj]) = acc;
    }
    __syncthreads();
    if (ok && mg == 0) {  // T_{3,0} = T_33 (Y_0 + Y_1 + Y_2)
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const float4 y0 = *reinterpret_cast<const float4*>(&sY[0][m][mj]);
            const float4 y1 = *reinterpret_cast<const float4*>(&sY[1][m][mj]);
            const float4 y2 = *reinterpret_cast<const float4*>(&sY[2][m][mj]);
            f4fma(acc, sT[48 + mi][48 + m],
                  make_float4(y0.x + y1.x + y2.x, y0.y + y1.y + y2.y, y0.z + y1.z + y2.z, y0.w + y1.w + y2.w));
        }
        *reinterpret_cast<float4*>(&sT[48 + mi][mj]) = acc;
    }
    __syncthreads();

    // ---- 5. (Aqk T) on the tensor core: T -> hi/lo B tiles over L (dead), then three M=64, N=64, K=64
    //      passes (hi.hi + hi.lo + lo.hi) into TMEM cols [0,64) (G is dead).  Rows of the M=64
    //      accumulator sit in lanes 0-15 of each 32-lane quadrant.
    if (ok) {
        const int m = tid >> 3, c0 = 8 * (tid & 7);
        float tv[8];
#pragma unroll
        for (int e4 = 0; e4 < 2; ++e4) {
            const float4 x = *reinterpret_cast<const float4*>(&sT[m][c0 + 4 * e4]);
            tv[4 * e4] = x.x;
            tv[4 * e4 + 1] = x.y;
            tv[4 * e4 + 2] = x.z;
            tv[4 * e4 + 3] = x.w;
        }
        store_split8(sm + P_TT, sm + P_TT + 8192, sw128_offset(m, c0, 64), tv);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (ok && tid == 0) {
        tc_fence_after();
        const uint32_t id = make_idesc_f16(64, 64, false, true, true);
        const uint32_t ah = sbase + P_AQK, al = ah + 8192, bh = sbase + P_TT, bl = bh + 8192;
        const uint32_t as[3] = {ah, ah, al}, bs[3] = {bh, bl, bh};
#pragma unroll
        for (int pass = 0; pass < 3; ++pass)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
                mma_f16(tm, make_sdesc(as[pass] + ks * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(bs[pass] + ks * 2048, 8192, 1024, kSwizzle128B), id, (pass | ks) != 0);
        mma_commit(&ms.bar);
    }
    if (ok) ok = mbar_wait(&ms.bar, 1, kWaitNs);  // second completion of the barrier
    ok = !__syncthreads_or(!ok);
    tc_fence_after();
    // Thread (quadrant, lane, part) holds 16 columns jc.. of one coefficient row ri: lanes 16-31 the row
    // of T (-> X, Y), lanes 0-15 the row of Aqk T (-> Z, W).
    const bool top = lane >= 16;
    const int ri = 16 * quad + (lane & 15), jc = 16 * part;
    float cv[16];
    if (ok) {
        tmem_ld16(tmem_addr(tm, 32 * quad, jc), cv);
        tmem_ld_wait();
        if (top) {
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
                const float4 x = *reinterpret_cast<const float4*>(&sT[ri][jc + 4 * e4]);
                cv[4 * e4] = x.x;
                cv[4 * e4 + 1] = x.y;
                cv[4 * e4 + 2] = x.z;
                cv[4 * e4 + 3] = x.w;
            }
        }
    }
    tc_fence_before();
    __syncthreads();  // the tiles of step 5 are read: the work region is free for the A tiles
    // ---- 6. the four 64x64 coefficient matrices X = T B_e, Y = T B, W = (Aqk T) B, Z = (Aqk T) B_e,
    //      in two M=128, N=128, K=64 rounds (hi+lo): [X;Z] k^ -> cols [0,128) (w | Zk), then
    //      [Y;W] v -> cols [128,256) (u | o0), the A tiles of the second round written over the first's.
    const uint32_t id6 = make_idesc_f16(128, 128, false, true, true);
    uint32_t ph = 1;
    for (int round = 0; round < 2 && ok; ++round) {
        float x[16];  // row ri (X or Y) or 64+ri (Z or W)
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int j = jc + e;
            const float bj = ms.beta[j];
            const float bb = round == 0 ? bj * ms.egc[j] : bj;
            x[e] = cv[e] * bb;
        }
        unsigned char* at_hi = sm + P_ATILE;
        unsigned char* at_lo = sm + P_ATILE + 16384;
#pragma unroll
        for (int q8 = 0; q8 < 2; ++q8)
            store_split8(at_hi, at_lo, sw128_offset(top ? ri : 64 + ri, jc + 8 * q8, 128), x + 8 * q8);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            mma_split_a(tm + 128 * round, sbase + P_ATILE, sbase + P_ATILE + 16384,
                        round == 0 ? sbase + P_KQ : sbase + P_V, round == 0 ? 16384 : 8192, id6);
            mma_commit(&ms.bar);
        }
        ++ph;
        ok = mbar_wait(&ms.bar, ph & 1, kWaitNs);  // the A tiles may be rewritten only after the MMAs read them
        ok = !__syncthreads_or(!ok);
    }
    tc_fence_after();

    // ---- 7. rows 0-63: P_X = E_d w, P_Y = E_d u -> hi/lo B tiles (and w, u, Kd in fp32 for the backward);
    //      rows 64-127: Q' (in place of q^) and o0 -> workspace
    float* const tiles = p.bwd_tiles ? p.bwd_tiles + chunk * kWsChunkFloats : nullptr;
    if (ok) {
        const int r = 32 * quad + lane, i = r & 63;
        const float ed = ms.ekd[i];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {  // this thread's 32 columns, 16 at a time
            float v[16];
            const int d0 = 32 * part + 16 * cc;
            tmem_ld16(tmem_addr(tm, 32 * quad, d0), v);
            tmem_ld_wait();
            if (r < 64) {  // P_X (MN-major B tile: rows = tokens)
                if (tiles) {
                    store_cm16(tiles + kWsW, i, d0, v);
                    float kd[16];  // Kd = k^ e^(gc_last - gc), from the k^ rows of KQ
#pragma unroll
                    for (int q8 = 0; q8 < 2; ++q8) {
                        const uint4 ku = *reinterpret_cast<const uint4*>(sm + P_KQ + sw128_offset(i, d0 + 8 * q8, 128));
                        const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(&ku);
#pragma unroll
                        for (int e = 0; e < 8; ++e) kd[8 * q8 + e] = __bfloat162float(kb[e]) * ed;
                    }
                    store_cm16(tiles + kWsKd, i, d0, kd);
                }
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] *= ed;
#pragma unroll
                for (int q8 = 0; q8 < 2; ++q8)
                    store_split8(sm + P_PX, sm + P_PX + 16384, sw128_offset(i, d0 + 8 * q8, 64), v + 8 * q8);
            } else {  // Q' = q^ Dk^-1/2 e^gc - Zk (the q e^gc S of :175 and -Aqk w S of :176 combined)
                const float qs = scale * ms.egc[i];
#pragma unroll
                for (int q8 = 0; q8 < 2; ++q8) {
                    const uint32_t off = sw128_offset(64 + i, d0 + 8 * q8, 128);
                    const uint4 qu = *reinterpret_cast<const uint4*>(sm + P_KQ + off);
                    const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(&qu);
                    float o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[e] = qs * __bfloat162float(qb[e]) - v[8 * q8 + e];
                    store_bf16x8(sm + P_KQ, off, o);  // rows 64-127 of KQ: the layout of the Q' image
                }
            }
        }
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            float v[16];
            const int d0 = 32 * part + 16 * cc;
            tmem_ld16(tmem_addr(tm, 32 * quad, 128 + d0), v);
            tmem_ld_wait();
            if (r < 64) {  // P_Y
                if (tiles) store_cm16(tiles + kWsU, i, d0, v);
#pragma unroll
                for (int e = 0; e < 16; ++e) v[e] *= ed;
#pragma unroll
                for (int q8 = 0; q8 < 2; ++q8)
                    store_split8(sm + P_PYH, sm + P_PYL, sw128_offset(i, d0 + 8 * q8, 64), v + 8 * q8);
            } else {  // o0 = Aqk u, fp32 column tile d0/32, straight to the workspace: the tile is stored
                      // chunk-major ([8 chunks of 4 columns][64 rows][4]), so each store of a warp (32 rows, one
                      // chunk) writes 512 contiguous bytes
                unsigned char* blk = wrec + kTcO0 + (d0 >> 5) * (64 * 128);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    *reinterpret_cast<float4*>(blk + (((d0 & 31) >> 2) + q4) * 1024 + i * 16) =
                        make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (ok && tid == 32) {  // the Q' image leaves while the tensor core works on step 8
        bulk_s2g(wrec + kTcQ, sm + P_KQ + 8192, 8192);
        bulk_s2g(wrec + kTcQ + 8192, sm + P_KQ + 16384 + 8192, 8192);
        bulk_commit();
    }

    // ---- 8. M' = k^T P_X -> [0,128), b = k^T P_Y -> [128,256)  (M=128 over Dk, K = tokens)
    if (ok && tid == 0) {
        const uint32_t id = make_idesc_f16(128, 128, true, true, true);
        const uint32_t btiles[4] = {sbase + P_PX, sbase + P_PX + 16384, sbase + P_PYH, sbase + P_PYL};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t ad = make_sdesc(sbase + P_KQ + ks * 2048, 16384, 1024, kSwizzle128B);
                    const uint64_t bd = make_sdesc(btiles[2 * r + s2] + ks * 2048, 8192, 1024, kSwizzle128B);
                    mma_f16(tm + 128 * r, ad, bd, id, (s2 | ks) != 0);
                }
            }
        }
        mma_commit(&ms.bar);
    }
    if (ok) ok = mbar_wait(&ms.bar, 0, kWaitNs);  // fifth completion of the barrier
    if (tid == 32) bulk_wait_read_all();       // KQ is rewritten below: the Q' copy must have read it
    tc_fence_after();

    // ---- 9. M = e^gc_last I - M' (bf16 image into KQ, then one bulk copy), b (fp32, straight to the record)
    if (!__syncthreads_or(!ok)) {
        const int dk = 32 * quad + lane;
        const float gamma = ms.egc[kChunk - 1];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            float v[16];
            const int c0 = 32 * part + 16 * cc;
            tmem_ld16(tmem_addr(tm, 32 * quad, c0), v);
            tmem_ld_wait();
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) {
                const int col = c0 + 8 * q8;
                float m[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) m[e] = ((col + e) == dk ? gamma : 0.f) - v[8 * q8 + e];
                store_bf16x8(sm + P_KQ, sw128_offset(dk, col, 128), m);
            }
        }
        // b straight from the accumulator to the record (chunk-major tiles: a warp's store is 512 contiguous
        // bytes), so only the M image is left for the bulk copy to drain before the CTA can leave
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            float v[16];
            const int c0 = 32 * part + 16 * cc;
            tmem_ld16(tmem_addr(tm, 32 * quad, 128 + c0), v);
            tmem_ld_wait();
            unsigned char* blk = wrec + kTcB + (c0 >> 5) * 16384;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
                *reinterpret_cast<float4*>(blk + ((((c0 & 31) >> 2) + q4) * 128 + dk) * 16) =
                    make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        }
    } else {
        ok = false;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 32) {
        if (ok) {
            bulk_s2g(wrec + kTcM, sm + P_KQ, 32768);
            bulk_commit();
        }
        bulk_wait_read_all();  // shared memory must outlive every copy that reads it
    }
    if (!ok && tid == 0) report(p.err, kErrTimeoutPrep);
    if (!in_ok) mbar_wait(&ms.bar_in, 0, kWaitNs);  // no box may land after the CTA has left
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kPrepTmemCols);
    }
    __syncthreads();
}

// ============================================================================ scan

constexpr int kScanThreads = 224;          // warps 0-3: state/output epilogue, 4: M/Q bulk copies + L2 prefetch,
                                           // 5: b/o0 bulk copies, 6: MMA issue
constexpr int kScanPrefetch = 4;           // chunks ahead that the producer pulls into L2
constexpr int kScanMmaWarp = 6;
constexpr uint32_t kScanBarS = 1;          // named barrier: epilogue (128) arrives with S_c stored, MMA warp waits
constexpr uint32_t kScanBarCount = 160;
// Shared-memory layout of a scan CTA that owns kW state columns (16 when the B*H*8 CTAs fit in one wave of
// SMs, else 32): per stage the M image 32K | Q image 16K | the b slice | the o0 slice (both contiguous in the
// chunk-major records), two stages, then the state operand tiles, the record staging and the barriers.
template <int kW>
struct ScanLayout {
    static constexpr int kSlices = kDv / kW;                                   // CTAs per head
    static constexpr uint32_t kTmemCols = kW == 16 ? 64 : 128;                 // state | two output accumulators
    static constexpr uint32_t kBBytes = 128 * kW * 4, kO0Bytes = 64 * kW * 4;  // a slice of b / of o0
    static constexpr uint32_t kOffQ = 32768, kOffB = 49152, kOffO0 = kOffB + kBBytes;
    static constexpr uint32_t kStage = (kOffO0 + kO0Bytes + 1023) / 1024 * 1024;
    static constexpr uint32_t kSTile = 2 * kStage;  // state operand, two tiles by chunk parity: bf16 [128 dk][64] swizzled
    static constexpr uint32_t kXpose = kSTile + 2 * 16384;  // per state warp: fp32 [32 rows][kW + 4] staging of S_c
    static constexpr uint32_t kMisc = kXpose + 4 * 32 * (kW + 4) * 4;
    static constexpr uint32_t kSmem = kMisc + 256 + 1024;
    static_assert(kTmemCols >= 3 * kW && kSmem <= 227 * 1024, "scan layout");
};

struct ScanMisc {
    uint64_t full_mq[2];   // M/Q images landed (tx)
    uint64_t full_bo[2];   // b/o0 slices landed (tx)
    uint64_t empty_mq[2];  // the MMAs that read M/Q completed (tcgen05.commit)
    uint64_t empty_bo[2];  // the epilogue read b and o0 (128 arrivals)
    uint64_t mma_s;        // state accumulator of this chunk ready
    uint64_t mma_o[2];     // output accumulator of chunk c ready, alternating by chunk parity
    uint32_t tmem;
    int abort;
    int synced;            // named-barrier steps the MMA warp has passed
};

__device__ __forceinline__ bool scan_aborted(const ScanMisc& ms) {
    return *reinterpret_cast<const volatile int*>(&ms.abort) != 0;
}

// o_c rows 16w..16w+15 of this CTA's columns: o = Q'S (accumulator) + o0 (stage smem).
template <int kW>
__device__ __forceinline__ void scan_store_output(const ChunkParams& p, const unsigned char* st, const float (&o)[kW],
                                                  int64_t t0, int64_t t_lim, int warp, int lane, int b, int h,
                                                  int dv0) {
    if (lane >= 16) return;
    const int tok = 16 * warp + lane;
    const int64_t t = t0 + tok;
    if (t >= t_lim) return;
    float ov[kW];
#pragma unroll
    for (int q4 = 0; q4 < kW / 4; ++q4) {
        const float4 oo = *reinterpret_cast<const float4*>(st + ScanLayout<kW>::kOffO0 + q4 * 1024 + tok * 16);  // chunk-major slice
        ov[4 * q4] = o[4 * q4] + oo.x;
        ov[4 * q4 + 1] = o[4 * q4 + 1] + oo.y;
        ov[4 * q4 + 2] = o[4 * q4 + 2] + oo.z;
        ov[4 * q4 + 3] = o[4 * q4 + 3] + oo.w;
    }
    unsigned char* dst = reinterpret_cast<unsigned char*>(p.out) +
                         2 * ((int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + dv0);
#pragma unroll
    for (int q8 = 0; q8 < kW / 8; ++q8) store_bf16x8(dst, 16 * q8, ov + 8 * q8);
}

// The chunk-to-chunk chain S_{c+1} = M_c S_c + b_c runs through three parties each
// chunk: the epilogue warps store S_c as a bf16 operand tile and arrive on a named
// barrier; the MMA warp (converged, one elected lane issuing) waits on it and issues
// the state product, then the output product; the epilogue waits for the state
// accumulator, adds b_c, stores S_{c+1} and arrives, and only then turns to chunk c's
// outputs, which overlap the next chunk's MMAs.  Every party takes every barrier
// step of every chunk, also after a failed wait (then it skips the work), so the
// named barrier can never be left short of arrivals.
template <int kW>
__global__ void __launch_bounds__(kScanThreads, 1) gdn_scan_tc(ChunkParams p) {
    using L = ScanLayout<kW>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    ScanMisc& ms = *reinterpret_cast<ScanMisc*>(sm + L::kMisc);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // (sequence, head) -- also the state's [Dk, Dv] block -- and the 32-column slice of the state (and of b /
    // o0).  Packed sequences: a 1-D grid over (rank, head, slice), longest sequence first, so the long chains
    // start before the short ones fill the remaining SMs.
    int bh, h, dvt;
    if (p.cu_seqlens) {
        const int x = blockIdx.x;
        h = (x / L::kSlices) % p.H;
        dvt = x % L::kSlices;
        bh = p.seq_order[x / (L::kSlices * p.H)] * p.H + h;
    } else {
        bh = blockIdx.x;
        h = bh % p.H;
        dvt = blockIdx.y % L::kSlices;
    }
    const bool summary = p.scan_mode == 1;
    const bool transition = summary && blockIdx.y < L::kSlices;  // state starts from I, b ignored
    const int dv0 = dvt * kW;
    // chunk c of this sequence: record rec0 + c * rec_step, tokens tbase + 64 c .. (below t_lim)
    int b = bh / p.H, NC = p.NC;
    int64_t rec0 = (int64_t)bh * p.NC, rec_step = 1, tbase = 0, t_lim = p.T;
    if (p.cu_seqlens) {
        const int n = bh / p.H;
        b = 0;
        NC = p.chunk_base[n + 1] - p.chunk_base[n];
        rec0 = (int64_t)p.chunk_base[n] * p.H + h;
        rec_step = p.H;
        tbase = p.cu_seqlens[n];
        t_lim = p.cu_seqlens[n + 1];
    }
    const unsigned char* wsb = reinterpret_cast<const unsigned char*>(p.ws);
    auto record = [&](int c) { return wsb + (rec0 + (int64_t)c * rec_step) * kTcChunkBytes; };

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
        ms.synced = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);
    bool ok = true;

    if (warp == kScanMmaWarp) {
        // ---------------- MMA issue: the whole warp runs the loop, one elected lane issues
        const uint32_t leader = elect_one();
        const uint32_t idS = make_idesc_f16(128, kW, false, true, true);
        const uint32_t idO = make_idesc_f16(64, kW, false, true, true);
        const uint64_t dM = make_sdesc(sbase, 16, 1024, kSwizzle128B);
        const uint64_t dQ = make_sdesc(sbase + L::kOffQ, 16, 1024, kSwizzle128B);
        const uint64_t dS = make_sdesc(sbase + L::kSTile, 16384, 1024, kSwizzle128B);
        for (int c = 0; c < NC; ++c) {
            const int s = c & 1;
            named_bar_sync(kScanBarS, kScanBarCount);  // S_c is in operand tile s
            mark_barrier_step(&ms.synced, c + 1, lane);
            bool go = ok && !scan_aborted(ms);
            if (go) go = mbar_wait(&ms.full_mq[s], (c >> 1) & 1, kWaitNs);
            if (!__all_sync(0xffffffffu, go)) {  // the warp decides together
                ok = false;  // no MMA from here on: the epilogue's waits give up at the abort flag
                ms.abort = 1;
                continue;
            }
            tc_fence_after();
            const uint64_t so = (uint64_t)((s * L::kStage) >> 4);
            // state first: it is the only product on the sequential path
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_f16_if(leader, tm + 0, dM + so + (uint64_t)((((ks >> 2) * 16384) + (ks & 3) * 32) >> 4),
                           dS + (uint64_t)((s * 16384 + ks * 2048) >> 4), idS, ks > 0);
            mma_commit_if(leader, &ms.mma_s);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_f16_if(leader, tm + kW * (1 + s),
                           dQ + so + (uint64_t)((((ks >> 2) * 8192) + (ks & 3) * 32) >> 4),
                           dS + (uint64_t)((s * 16384 + ks * 2048) >> 4), idO, ks > 0);
            mma_commit_if(leader, &ms.mma_o[s]);
            mma_commit_if(leader, &ms.empty_mq[s]);
            __syncwarp();
        }
    } else if (warp >= 4) {
        // ---------------- producers: warp 4 streams the M/Q images, warp 5 the b/o0 slices
        if (lane == 0) {
            const bool mq = warp == 4;
            uint64_t* full = mq ? ms.full_mq : ms.full_bo;
            uint64_t* empty = mq ? ms.empty_mq : ms.empty_bo;
            const uint32_t bytes = mq ? 32768 + 16384 : L::kBBytes + L::kO0Bytes;
            int issued = 0;
            for (int c = 0; c < NC; ++c) {
                const int s = c & 1;
                if (mq && c + kScanPrefetch < NC) {
                    const unsigned char* pre = record(c + kScanPrefetch);
                    bulk_prefetch_l2(pre + kTcM, 32768 + 16384);
                    bulk_prefetch_l2(pre + kTcB + dvt * L::kBBytes, L::kBBytes);
                    bulk_prefetch_l2(pre + kTcO0 + dvt * L::kO0Bytes, L::kO0Bytes);
                }
                if (scan_aborted(ms)) break;
                if (c >= 2 && !mbar_wait(&empty[s], ((c >> 1) - 1) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                const unsigned char* rec = record(c);
                unsigned char* st = sm + s * L::kStage;
                mbar_arrive_expect_tx(&full[s], bytes);
                if (mq) {
                    bulk_g2s(st, rec + kTcM, 32768, &full[s]);
                    bulk_g2s(st + L::kOffQ, rec + kTcQ, 16384, &full[s]);
                } else {
                    bulk_g2s(st + L::kOffB, rec + kTcB + dvt * L::kBBytes, L::kBBytes, &full[s]);
                    bulk_g2s(st + L::kOffO0, rec + kTcO0 + dvt * L::kO0Bytes, L::kO0Bytes, &full[s]);
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
        float S[kW];
        const int64_t srow = ((int64_t)bh * kDk + dk) * kDv + dv0;
#pragma unroll
        for (int q4 = 0; q4 < kW / 4; ++q4) {
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
        unsigned char* stile = sm + L::kSTile;
#pragma unroll
        for (int q8 = 0; q8 < kW / 8; ++q8) store_bf16x8(stile, sw128_offset(dk, 8 * q8, 128), S + 8 * q8);
        fence_proxy_async_smem();
        if (NC > 0) named_bar_arrive(kScanBarS, kScanBarCount);  // S_0 for chunk 0 (a sequence may be empty)

        for (int c = 0; c < NC; ++c) {
            const int s = c & 1;
            const unsigned char* st = sm + s * L::kStage;
            if (p.states)  // S_c (fp32) for the backward: the warp's 32 rows, this CTA's 32 columns
                store_rows_coalesced<kW>(
                    reinterpret_cast<float*>(sm + L::kXpose) + warp * 32 * (kW + 4), S,
                    p.states + (rec0 + (int64_t)c * rec_step) * p.states_stride + (int64_t)(32 * warp) * kDv + dv0,
                    kDv, lane);
            // ---- S_{c+1} = M_c S_c + b_c (the sequential path)
            if (ok && scan_aborted(ms)) ok = false;
            if (ok && (!mbar_wait(&ms.mma_s, c & 1, kWaitNs) || !mbar_wait(&ms.full_bo[s], (c >> 1) & 1, kWaitNs)))
                ok = false;
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: the warp loads or skips together
            if (ok) {
                tc_fence_after();
                float d[kW];
                if constexpr (kW == 16) tmem_ld16(tmem_addr(tm, 32 * warp, 0), d);
                else tmem_ld32(tmem_addr(tm, 32 * warp, 0), d);
                tmem_ld_wait();
#pragma unroll
                for (int q4 = 0; q4 < kW / 4; ++q4) {  // b slice chunk-major: row dk, 16 bytes apart
                    float4 bb = *reinterpret_cast<const float4*>(st + L::kOffB + (q4 * 128 + dk) * 16);
                    if (transition) bb = make_float4(0.f, 0.f, 0.f, 0.f);
                    S[4 * q4] = d[4 * q4] + bb.x;
                    S[4 * q4 + 1] = d[4 * q4 + 1] + bb.y;
                    S[4 * q4 + 2] = d[4 * q4 + 2] + bb.z;
                    S[4 * q4 + 3] = d[4 * q4 + 3] + bb.w;
                }
            }
            if (c + 1 < NC) {
                if (ok) {  // tile (c+1) % 2 was last read by chunk c-1's MMAs, complete before chunk c's state product
#pragma unroll
                    for (int q8 = 0; q8 < kW / 8; ++q8)
                        store_bf16x8(stile + (s ^ 1) * 16384, sw128_offset(dk, 8 * q8, 128), S + 8 * q8);
                    fence_proxy_async_smem();
                }
                tc_fence_before();
                if (!ok) wait_barrier_step(&ms.synced, c + 1);  // the MMA warp has passed step c
                named_bar_arrive(kScanBarS, kScanBarCount);
            }
            // ---- outputs of chunk c, overlapping chunk c+1's MMAs
            if (ok && !mbar_wait(&ms.mma_o[s], (c >> 1) & 1, kWaitNs)) ok = false;
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                tc_fence_after();
                float o[kW];
                if constexpr (kW == 16) tmem_ld16(tmem_addr(tm, 32 * warp, kW * (1 + s)), o);
                else tmem_ld32(tmem_addr(tm, 32 * warp, kW * (1 + s)), o);
                tmem_ld_wait();
                if (!summary && p.out)
                    scan_store_output<kW>(p, st, o, tbase + (int64_t)c * kChunk, t_lim, warp, lane, b, h, dv0);
                tc_fence_before();
            }
            if (!ok) ms.abort = 1;
            mbar_arrive(&ms.empty_bo[s]);
        }
        float* dst = summary ? (transition ? p.hT : p.hT2) : p.hT;
        if (ok && dst) {
#pragma unroll
            for (int q4 = 0; q4 < kW / 4; ++q4)
                *reinterpret_cast<float4*>(dst + srow + 4 * q4) =
                    make_float4(S[4 * q4], S[4 * q4 + 1], S[4 * q4 + 2], S[4 * q4 + 3]);
        }
    }
    if (!ok) {
        ms.abort = 1;
        report(p.err, kErrTimeoutScan);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, L::kTmemCols);
}

// ============================================================================ lean scan (many heads)
//
// gdn_scan_lean_tc: the scan for problems with more (batch, head) chains than SMs.  gdn_scan_tc holds an SM per
// chain (~160-200 KB of shared memory); with the records in DRAM rather than L2 a chain then waits on its record
// loads (~2.4 us a chunk at B=64, H=16), and one chain per SM leaves that latency exposed.  This kernel runs a
// chain in 112 KiB and 512 threads, so two share an SM.  One CTA per (batch, head, 32-column slice of Dv):
//   warps 0-7   chain: thread = state row dk = 32 (w % 4) + lane (its TMEM lane), columns 16 (w / 4) .. +15;
//               S_{c+1} = accumulator + b_c as the next bf16 operand tile, handed to the MMA warp through
//               named barrier 1; b read straight from the record into registers two chunks ahead
//   warps 8-11  outputs: thread = output row 16 (w - 8) + lane (lanes 0-15, the M=64 accumulator's rows), the
//               CTA's 32 columns; o_c = accumulator + o0_c (o0 read from the record one chunk ahead)
//   warp 12     M images into the stage freed by the state product of chunk c-2, and every record pulled into
//               L2 four chunks ahead
//   warp 13     MMAs (one elected lane of the converged warp): the state product M_c S_c, then the output
//               product Q'_c S_c
//   warp 14     Q' images into the stage freed by the output product of chunk c-2
//   warp 15     idle
// Shared memory: M images [2][32 KiB] | S_c operand tiles [2][8 KiB] (bf16 [128 dk][32], MN-major, 64B-swizzled) |
// Q' images [2][16 KiB], with the barriers in the 1 KiB alignment slack.  TMEM: state accumulator [0, 32),
// output accumulators [32, 64) and [64, 96) by chunk parity.

constexpr int kLeanW = 32;                      // state columns per CTA
constexpr int kLeanSlices = kDv / kLeanW;       // CTAs per (batch, head)
constexpr int kLeanThreads = 512;
constexpr uint32_t LN_M = 0;
constexpr uint32_t LN_S = 65536;
constexpr uint32_t LN_Q = 81920;
constexpr uint32_t LN_TILES = 114688;
constexpr uint32_t kLeanSmem = LN_TILES + 1024;  // + alignment slack, which also holds LeanMisc
constexpr uint32_t kLeanTmemCols = 128;
constexpr uint32_t kLeanBar = 1;                 // named barrier: chain warps (256) arrive with S_c stored, MMA warp waits
constexpr uint32_t kLeanBarCount = 288;
constexpr int kLnOut = 8, kLnProdM = 12, kLnMma = 13, kLnProdQ = 14;
constexpr int kLeanPrefetch = 4;                 // chunks ahead that the M producer pulls into L2
static_assert(kLeanSmem <= 227 * 1024, "lean scan shared memory");

struct LeanMisc {
    uint64_t full_m[2];  // M image of the stage landed (tx)
    uint64_t m_free[2];  // the state product that read the stage completed (tcgen05.commit)
    uint64_t full_q[2];  // Q' image of the stage landed (tx)
    uint64_t q_free[2];  // the output product that read the stage completed
    uint64_t mma_s;      // chunk c's state product completed
    uint64_t mma_o[2];   // output product of chunk c completed, by chunk parity
    uint64_t o_free[2];  // the output warps read output accumulator p (128 arrivals)
    uint64_t done;       // every product the MMA warp issued has completed
    uint32_t tmem;
    int abort;           // a party gave up: the others stop waiting and skip their work
    int synced;          // named-barrier steps the MMA warp has passed
};

// Byte offset of element (row, col), col < 32, in an MN-major 64B-swizzled tile of 16-bit elements: 64-byte
// rows, 8-row atoms of 512 bytes packed along the rows (SBO = 512); the 16-byte chunk c of row r is stored at
// chunk c ^ ((r / 2) % 4).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t col) {
    return row * 64u + ((((col >> 3) ^ (row >> 1)) & 3u) << 4) + (col & 7u) * 2u;
}

__device__ __forceinline__ bool lean_aborted(const LeanMisc& ms) {
    return *reinterpret_cast<const volatile int*>(&ms.abort) != 0;
}

// Bounded wait on an mbarrier phase that also gives up once another party has aborted.
__device__ __forceinline__ bool lean_wait(uint64_t* bar, uint32_t parity, const LeanMisc& ms) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    const long long budget = (long long)(kWaitNs * 2);
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (lean_aborted(ms) || clock64() - t0 > budget) return false;
    }
}

// 16 or 32 fp32 values of one row of a chunk-major record tile (element (row, col) at ((col / 4) * rows + row) * 4
// + col % 4): columns col0 .. col0+kN-1, 16-byte loads, each a 512- or 256-byte run across the warp.
template <int kRows, int kN>
__device__ __forceinline__ void load_cm(const unsigned char* tile, int row, int col0, float (&v)[kN]) {
#pragma unroll
    for (int q4 = 0; q4 < kN / 4; ++q4) {
        const float4 x = *reinterpret_cast<const float4*>(tile + ((int64_t)((col0 >> 2) + q4) * kRows + row) * 16);
        v[4 * q4] = x.x;
        v[4 * q4 + 1] = x.y;
        v[4 * q4 + 2] = x.z;
        v[4 * q4 + 3] = x.w;
    }
}

__global__ void __launch_bounds__(kLeanThreads, 2) gdn_scan_lean_tc(ChunkParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    unsigned char* sm = smem_raw + pad;
    LeanMisc& ms = *reinterpret_cast<LeanMisc*>(pad >= sizeof(LeanMisc) ? smem_raw : sm + LN_TILES);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = (int)(blockIdx.x / kLeanSlices), slice = (int)(blockIdx.x % kLeanSlices);
    const int b = bh / p.H, h = bh % p.H, NC = p.NC;
    const int dv0 = slice * kLeanW;  // first state column of the CTA
    const int64_t rec0 = (int64_t)bh * NC;
    const unsigned char* wsb = reinterpret_cast<const unsigned char*>(p.ws);
    auto record = [&](int c) { return wsb + (rec0 + c) * kTcChunkBytes; };

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ms.full_m[s], 1);
            mbar_init(&ms.m_free[s], 1);
            mbar_init(&ms.full_q[s], 1);
            mbar_init(&ms.q_free[s], 1);
            mbar_init(&ms.mma_o[s], 1);
            mbar_init(&ms.o_free[s], 128);
        }
        mbar_init(&ms.mma_s, 1);
        mbar_init(&ms.done, 1);
        ms.abort = 0;
        ms.synced = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kLeanTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);
    bool ok = true;

    if (warp == kLnMma) {
        // ---------------- MMAs: the whole warp runs the loop, one elected lane issues
        const uint32_t leader = elect_one();
        const uint32_t idS = make_idesc_f16(128, kLeanW, false, true, true);
        const uint32_t idO = make_idesc_f16(64, kLeanW, false, true, true);
        const uint64_t dM = make_sdesc(sbase + LN_M, 16, 1024, kSwizzle128B);
        const uint64_t dQ = make_sdesc(sbase + LN_Q, 16, 1024, kSwizzle128B);
        const uint64_t dS = make_sdesc(sbase + LN_S, 8192, 512, kSwizzle64B);
        for (int c = 0; c < NC; ++c) {
            const int s = c & 1;
            named_bar_sync(kLeanBar, kLeanBarCount);  // S_c is in operand tile s
            mark_barrier_step(&ms.synced, c + 1, lane);
            bool go = ok && !lean_aborted(ms);
            if (go) go = lean_wait(&ms.full_m[s], (c >> 1) & 1, ms);
            if (!__all_sync(0xffffffffu, go)) {
                ok = false;
                ms.abort = 1;
                continue;
            }
            tc_fence_after();
            // state first: it is the only product on the sequential path
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_f16_if(leader, tm + 0, dM + (uint64_t)(((s * 32768) + ((ks >> 2) * 16384) + (ks & 3) * 32) >> 4),
                           dS + (uint64_t)((s * 8192 + ks * 1024) >> 4), idS, ks > 0);
            mma_commit_if(leader, &ms.mma_s);
            mma_commit_if(leader, &ms.m_free[s]);
            go = lean_wait(&ms.full_q[s], (c >> 1) & 1, ms);
            if (go && c >= 2) go = lean_wait(&ms.o_free[s], ((c >> 1) - 1) & 1, ms);
            if (!__all_sync(0xffffffffu, go)) {
                ok = false;
                ms.abort = 1;
                continue;
            }
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_f16_if(leader, tm + 32 + 32 * s,
                           dQ + (uint64_t)(((s * 16384) + ((ks >> 2) * 8192) + (ks & 3) * 32) >> 4),
                           dS + (uint64_t)((s * 8192 + ks * 1024) >> 4), idO, ks > 0);
            mma_commit_if(leader, &ms.mma_o[s]);
            mma_commit_if(leader, &ms.q_free[s]);
            __syncwarp();
        }
        mma_commit_if(leader, &ms.done);  // arrives once every product issued above has completed
        __syncwarp();
        if (!mbar_wait(&ms.done, 0, kWaitNs)) ok = false;
    } else if (warp == kLnProdM || warp == kLnProdQ) {
        // ---------------- producers (lane 0): M and Q' images into the stage the chunk two back freed
        if (lane == 0) {
            const bool mq = warp == kLnProdM;
            int issued = 0;
            for (int j = 0; j < NC; ++j) {
                if (lean_aborted(ms)) break;
                const int st = j & 1;
                if (mq && j + kLeanPrefetch < NC) {  // the whole record of a later chunk into L2
                    const unsigned char* pre = record(j + kLeanPrefetch);
                    bulk_prefetch_l2(pre + kTcM, 32768 + 16384);
                    bulk_prefetch_l2(pre + kTcB + (int64_t)slice * 128 * kLeanW * 4, 128 * kLeanW * 4);
                    bulk_prefetch_l2(pre + kTcO0 + (int64_t)slice * 64 * kLeanW * 4, 64 * kLeanW * 4);
                }
                if (j >= 2 && !lean_wait(mq ? &ms.m_free[st] : &ms.q_free[st], ((j >> 1) - 1) & 1, ms)) {
                    ok = false;
                    break;
                }
                if (mq) {
                    mbar_arrive_expect_tx(&ms.full_m[st], 32768);
                    bulk_g2s(sm + LN_M + st * 32768, record(j) + kTcM, 32768, &ms.full_m[st]);
                } else {
                    mbar_arrive_expect_tx(&ms.full_q[st], 16384);
                    bulk_g2s(sm + LN_Q + st * 16384, record(j) + kTcQ, 16384, &ms.full_q[st]);
                }
                ++issued;
            }
            // no copy may land after the CTA has left
            for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
                if (!mbar_wait(mq ? &ms.full_m[j & 1] : &ms.full_q[j & 1], (j >> 1) & 1, kWaitNs)) ok = false;
        }
    } else if (warp < kLnOut) {
        // ---------------- chain: thread = state row dk (TMEM lane 32 (w % 4) + lane), columns 16 (w / 4) .. +15
        const int dk = 32 * (warp & 3) + lane, cb = 16 * (warp >> 2);
        const int64_t srow = ((int64_t)bh * kDk + dk) * kDv + dv0 + cb;
        {
            float s0[16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                const float4 v = p.h0 ? *reinterpret_cast<const float4*>(p.h0 + srow + 4 * q4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                s0[4 * q4] = v.x;
                s0[4 * q4 + 1] = v.y;
                s0[4 * q4 + 2] = v.z;
                s0[4 * q4 + 3] = v.w;
            }
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) store_bf16x8(sm + LN_S, sw64_offset(dk, cb + 8 * q8), s0 + 8 * q8);
            fence_proxy_async_smem();
        }
        if (NC > 0) named_bar_arrive(kLeanBar, kLeanBarCount);  // S_0 for chunk 0
        // b_c of this thread's row and columns lives in bA (c even) or bB (c odd), read two chunks ahead
        float bA[16], bB[16];
        if (NC > 0) load_cm<128, 16>(record(0) + kTcB, dk, dv0 + cb, bA);
        if (NC > 1) load_cm<128, 16>(record(1) + kTcB, dk, dv0 + cb, bB);
        auto chain_step = [&](int c, float (&bc)[16]) {
            // ---- S_{c+1} = M_c S_c + b_c (the sequential path)
            if (ok && lean_aborted(ms)) ok = false;
            if (ok) ok = lean_wait(&ms.mma_s, c & 1, ms);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective: the warp loads or skips together
            if (ok) {
                tc_fence_after();
                float d[16];
                tmem_ld16(tmem_addr(tm, 32 * (warp & 3), cb), d);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 16; ++e) d[e] += bc[e];
                if (c + 1 < NC) {  // tile (c+1) % 2 held S_{c-1}, whose products completed before chunk c's state
#pragma unroll
                    for (int q8 = 0; q8 < 2; ++q8)
                        store_bf16x8(sm + LN_S + ((c + 1) & 1) * 8192, sw64_offset(dk, cb + 8 * q8), d + 8 * q8);
                    fence_proxy_async_smem();
                } else if (p.hT) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4)
                        *reinterpret_cast<float4*>(p.hT + srow + 4 * q4) =
                            make_float4(d[4 * q4], d[4 * q4 + 1], d[4 * q4 + 2], d[4 * q4 + 3]);
                }
            }
            if (c + 1 < NC) {
                tc_fence_before();
                if (!ok) wait_barrier_step(&ms.synced, c + 1);  // the MMA warp has passed step c
                named_bar_arrive(kLeanBar, kLeanBarCount);  // every chunk, also after a failure
            }
            if (ok && c + 2 < NC) load_cm<128, 16>(record(c + 2) + kTcB, dk, dv0 + cb, bc);  // bc is free: b_{c+2}
            if (!ok) ms.abort = 1;
        };
        for (int c = 0; c < NC; c += 2) {
            chain_step(c, bA);
            if (c + 1 < NC) chain_step(c + 1, bB);
        }
    } else if (warp < kLnProdM) {
        // ---------------- outputs: thread = output row 16 q + lane (lanes 0-15), the CTA's 32 columns
        const int q = warp - kLnOut, tok = 16 * q + lane;
        float ov[32];
        if (NC > 0 && lane < 16) load_cm<64, 32>(record(0) + kTcO0, tok, dv0, ov);
        for (int c = 0; c < NC; ++c) {
            if (ok && lean_aborted(ms)) ok = false;
            if (ok) ok = lean_wait(&ms.mma_o[c & 1], (c >> 1) & 1, ms);
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                tc_fence_after();
                const int64_t t = (int64_t)c * kChunk + tok;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float o[16];
                    tmem_ld16(tmem_addr(tm, 32 * q, 32 + 32 * (c & 1) + 16 * half), o);
                    tmem_ld_wait();
                    if (lane < 16 && t < p.T && p.out) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) o[e] += ov[16 * half + e];
                        unsigned char* dst = reinterpret_cast<unsigned char*>(p.out) +
                                             2 * ((int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + dv0 +
                                                  16 * half);
                        store_bf16x8(dst, 0, o);
                        store_bf16x8(dst, 16, o + 8);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&ms.o_free[c & 1]);  // every chunk, also after a failure
            if (ok && c + 1 < NC && lane < 16) load_cm<64, 32>(record(c + 1) + kTcO0, tok, dv0, ov);
            if (!ok) ms.abort = 1;
        }
    }
    if (!ok) ms.abort = 1;
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kLeanTmemCols);
    }
    if (tid == 0 && lean_aborted(ms)) report(p.err, kErrTimeoutScan);
}

// ============================================================================ reverse scan (backward)
//
// dS_c = M_c^T dS_{c+1} + Q'_c^T do_c over the forward's records, chunks in reverse: the transposed affine
// map of the forward scan (the gradient of S_{c+1} = M_c S_c + b_c, o_c = Q'_c S_c + o0_c).  One CTA per
// (b, h, 64-column half of Dv).  Warps 0-3 keep the fp32 gradient state (thread = row dk, 64 columns),
// record dS_{c+1} for the chunk kernels and hand a bf16 copy to warp 6, which issues M^T dS (K = 128) and
// Q'^T do (K = 64) into one TMEM accumulator from one elected lane of a converged warp; both transposes
// are the forward's images read MN-major.  Warp 4 bulk-copies the M / Q' images (double-buffered, pulled
// into L2 four chunks ahead), warp 5 stages do as a swizzled bf16 tile with cp.async (double-buffered).
constexpr int kBsThreads = 224;
constexpr int kBsMmaWarp = 6;
constexpr uint32_t kBsBar = 2;              // named barrier: the state warps (128) arrive, the MMA warp waits
constexpr uint32_t kBsBarCount = 160;
constexpr int kBsCols = 16;                 // gradient-state columns per CTA (eight CTAs per head)
constexpr uint32_t kBsTmemCols = 32;        // the 128 x 16 fp32 accumulator (the smallest allocation)
constexpr uint32_t B_STAGE = 49152;         // M image 32 KiB | Q' image 16 KiB
constexpr uint32_t B_OFF_Q = 32768;
constexpr uint32_t B_DO = 2 * B_STAGE;      // do tiles: bf16 [64 t][64] swizzled (this CTA's columns used), by parity
constexpr uint32_t B_STILE = B_DO + 2 * 8192;  // dS operand tiles: bf16 [128 dk][64] swizzled (this CTA's columns used)
constexpr uint32_t B_XPOSE = B_STILE + 2 * 16384;  // per state warp: fp32 [32 rows][kBsCols + 4] staging of the dS records
constexpr uint32_t B_MISC = B_XPOSE + 4 * 32 * (kBsCols + 4) * 4;
constexpr uint32_t B_SMEM = B_MISC + 256 + 1024;

struct BsMisc {
    uint64_t full_mq[2], empty_mq[2], full_do[2], empty_do[2];
    uint64_t mma;
    uint32_t tmem;
    int abort;
    int synced;  // named-barrier steps the MMA warp has passed
};

__device__ __forceinline__ bool bs_aborted(const BsMisc& ms) { return *reinterpret_cast<const volatile int*>(&ms.abort) != 0; }

__global__ void __launch_bounds__(kBsThreads, 1) gdn_bwd_scan_tc(BwdParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    BsMisc& ms = *reinterpret_cast<BsMisc*>(sm + B_MISC);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
    const int dv0 = blockIdx.y * kBsCols;
    const int NC = p.NC;
    const unsigned char* recs = reinterpret_cast<const unsigned char*>(p.tc_records) + (int64_t)bh * NC * kTcChunkBytes;
    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ms.full_mq[s], 1);
            mbar_init(&ms.empty_mq[s], 1);
            mbar_init(&ms.full_do[s], 1);
            mbar_init(&ms.empty_do[s], 1);
        }
        mbar_init(&ms.mma, 1);
        ms.abort = 0;
        ms.synced = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kBsTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);
    bool ok = true;
    // iteration it handles chunk c = NC - 1 - it with buffers it % 2

    if (warp == kBsMmaWarp) {
        const uint32_t leader = elect_one();
        const uint32_t id = make_idesc_f16(128, kBsCols, true, true, true);
        for (int it = 0; it < NC; ++it) {
            const int s = it & 1;
            named_bar_sync(kBsBar, kBsBarCount);  // dS_{c+1} is in operand tile s
            mark_barrier_step(&ms.synced, it + 1, lane);
            bool go = ok && !bs_aborted(ms);
            if (go) go = mbar_wait(&ms.full_mq[s], (it >> 1) & 1, kWaitNs);
            if (go) go = mbar_wait(&ms.full_do[s], (it >> 1) & 1, kWaitNs);
            if (!__all_sync(0xffffffffu, go)) {
                ok = false;
                ms.abort = 1;
                continue;
            }
            tc_fence_after();
            const uint32_t mimg = sbase + s * B_STAGE, qimg = mimg + B_OFF_Q;
            const uint32_t stile = sbase + B_STILE + s * 16384, dtile = sbase + B_DO + s * 8192;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)  // M^T dS: the M image (rows dk, 2 atom columns of k) read MN-major
                mma_f16_if(leader, tm, make_sdesc(mimg + ks * 2048, 16384, 1024, kSwizzle128B),
                           make_sdesc(stile + ks * 2048, 16384, 1024, kSwizzle128B), id, ks > 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)  // + Q'^T do: the Q' image (rows t, 2 atom columns of k) read MN-major
                mma_f16_if(leader, tm, make_sdesc(qimg + ks * 2048, 8192, 1024, kSwizzle128B),
                           make_sdesc(dtile + ks * 2048, 8192, 1024, kSwizzle128B), id, true);
            mma_commit_if(leader, &ms.mma);
            mma_commit_if(leader, &ms.empty_mq[s]);
            mma_commit_if(leader, &ms.empty_do[s]);
            __syncwarp();
        }
    } else if (warp == 4) {
        if (lane == 0) {  // M / Q' images of the chunk's record
            int issued = 0;
            for (int it = 0; it < NC; ++it) {
                const int s = it & 1, c = NC - 1 - it;
                if (c >= kScanPrefetch) bulk_prefetch_l2(recs + (int64_t)(c - kScanPrefetch) * kTcChunkBytes, 49152);
                if (bs_aborted(ms)) break;
                if (it >= 2 && !mbar_wait(&ms.empty_mq[s], ((it >> 1) - 1) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                const unsigned char* rec = recs + (int64_t)c * kTcChunkBytes;
                mbar_arrive_expect_tx(&ms.full_mq[s], 49152);
                bulk_g2s(sm + s * B_STAGE, rec + kTcM, 32768, &ms.full_mq[s]);
                bulk_g2s(sm + s * B_STAGE + B_OFF_Q, rec + kTcQ, 16384, &ms.full_mq[s]);
                ++issued;
            }
            // leave no copy in flight: wait for the last image of each stage to land
            for (int it = (issued > 2 ? issued - 2 : 0); it < issued; ++it)
                if (!mbar_wait(&ms.full_mq[it & 1], (it >> 1) & 1, kWaitNs)) ok = false;
        }
    } else if (warp == 5) {  // do tiles: rows t of the chunk, this CTA's columns, zero past T
        for (int it = 0; it < NC; ++it) {
            const int s = it & 1, c = NC - 1 - it;
            bool go = !bs_aborted(ms);
            if (go && it >= 2) go = mbar_wait(&ms.empty_do[s], ((it >> 1) - 1) & 1, kWaitNs);
            if (!__all_sync(0xffffffffu, go)) {
                ok = false;
                break;
            }
            unsigned char* tile = sm + B_DO + s * 8192;
            for (int piece = lane; piece < kChunk * (kBsCols / 8); piece += 32) {
                const int row = piece / (kBsCols / 8), c8 = piece % (kBsCols / 8);
                const int64_t t = (int64_t)c * kChunk + row;
                const bool in = t < p.T;
                const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.dout.p) + (int64_t)b * p.dout.sb +
                                           (in ? t : 0) * p.dout.st + (int64_t)h * p.dout.sh + dv0 + 8 * c8;
                cp_async16(tile + sw128_offset(row, 8 * c8, 64), src, in ? 16u : 0u);
            }
            cp_async_commit();
            cp_async_wait_all();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ms.full_do[s]);
        }
    } else {  // warps 0-3: thread = row dk of the gradient state, this CTA's columns
        const int dk = tid;
        float S[kBsCols];
        const int64_t srow = ((int64_t)bh * kDk + dk) * kDv + dv0;
#pragma unroll
        for (int q4 = 0; q4 < kBsCols / 4; ++q4) {
            const float4 v = p.dhT ? *reinterpret_cast<const float4*>(p.dhT + srow + 4 * q4) : make_float4(0.f, 0.f, 0.f, 0.f);
            S[4 * q4] = v.x;
            S[4 * q4 + 1] = v.y;
            S[4 * q4 + 2] = v.z;
            S[4 * q4 + 3] = v.w;
        }
        for (int it = 0; it < NC; ++it) {
            const int s = it & 1, c = NC - 1 - it;
            if (ok) {  // tile s was last read by the MMAs of iteration it - 2, complete before iteration it - 1's
#pragma unroll
                for (int q8 = 0; q8 < kBsCols / 8; ++q8)
                    store_bf16x8(sm + B_STILE + s * 16384, sw128_offset(dk, 8 * q8, 128), S + 8 * q8);
                fence_proxy_async_smem();
            }
            tc_fence_before();
            if (!ok) wait_barrier_step(&ms.synced, it);  // the MMA warp has passed step it - 1
            named_bar_arrive(kBsBar, kBsBarCount);
            // dS_{c+1} (fp32) for the chunk kernels, while the MMAs run: the warp's 32 rows, this CTA's columns
            store_rows_coalesced<kBsCols>(reinterpret_cast<float*>(sm + B_XPOSE) + warp * 32 * (kBsCols + 4), S,
                                     p.bws + ((int64_t)bh * NC + c) * kBwChunkFloats + kBwDSe +
                                         (int64_t)(32 * warp) * kDv + dv0,
                                     kDv, lane);
            if (ok && bs_aborted(ms)) ok = false;
            if (ok && !mbar_wait(&ms.mma, it & 1, kWaitNs)) ok = false;
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
            if (ok) {
                tc_fence_after();
                tmem_ld16(tmem_addr(tm, 32 * warp, 0), S);
                tmem_ld_wait();
                tc_fence_before();
            }
            if (!ok) ms.abort = 1;
        }
        if (ok && p.dh0) {
#pragma unroll
            for (int q4 = 0; q4 < kBsCols / 4; ++q4)
                *reinterpret_cast<float4*>(p.dh0 + srow + 4 * q4) = make_float4(S[4 * q4], S[4 * q4 + 1], S[4 * q4 + 2], S[4 * q4 + 3]);
        }
    }
    if (!ok) {
        ms.abort = 1;
        report(p.err, kErrTimeoutScan);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, kBsTmemCols);
}

// ============================================================================ backward: state products
//
// Per chunk, on the tensor cores, the products of the backward that involve the chunk-start state S_c and
// the end-state gradient dS' = dS_{c+1} (both fp32, entered as hi/lo bf16 pairs):
//   (1) dv_new = Kd dS' + Aqk^T do          (M=64; Aqk^T is Aqk's rows read MN-major, do exact bf16)
//   (2) v_new = u - w S                      (M=64)
//   (3) [dQg; -dw] = [do; dv_new] S^T        (M=128)
//   (4) dKd = v_new dS'^T                    (M=64)
// S and dS' are staged once as swizzled bf16 [128 dk][128 dv] tiles: an MN-major B operand for (1)/(2)
// (K = dk) and a K-major B operand for (3)/(4) (N = dk, K = dv).  Three MMA passes (hi.hi, hi.lo, lo.hi)
// per fp32 x fp32 product keep them fp32-accurate.  One CTA of 256 threads per chunk.
constexpr int kBtThreads = 256;
constexpr uint32_t T_DS = 0;          // dS' hi | lo (32 KiB each): bf16 [128 dk][128 dv], atom columns of 16 KiB
constexpr uint32_t T_S = 65536;       // S hi | lo, same layout
constexpr uint32_t T_DOB = 131072;    // do as the B operand of (1): bf16 [64 t][128 dv], atom columns of 8 KiB;
                                      // then v_new hi for (4)
constexpr uint32_t T_A = 147456;      // A operands (80 KiB): (1)-(2) Kd hi|lo +0/+16K, Aqk hi|lo +32K/+40K, w hi|lo
                                      // +48K/+64K; (3) [do; dv_new] hi|lo +0/+32K; (4) v_new lo +64K
constexpr uint32_t T_MISC = T_A + 81920;
constexpr uint32_t T_SMEM = T_MISC + 256 + 1024;
constexpr uint32_t kBtTmemCols = 512;  // (1) [0,128)  (2) [128,256)  (3) [256,384)  (4) [384,512)

struct BtMisc {
    uint64_t bar;
    uint32_t tmem;
    float red[kBtThreads / 32];
};

__global__ void __launch_bounds__(kBtThreads, 1) gdn_bwd_states_tc(BwdParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    BtMisc& ms = *reinterpret_cast<BtMisc*>(sm + T_MISC);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* fw = p.fws + ci * kWsChunkFloats;
    float* bw = p.bws + ci * kBwChunkFloats;
    if (tid == 0) {
        mbar_init(&ms.bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kBtTmemCols);
        tmem_relinquish();
    }
    // ---- staging: S and dS' (and <S, dS'>), Kd, Aqk, w as hi/lo tiles; do as an exact bf16 tile
    // Loads are issued in batches (16 float4 per thread in flight) before any conversion: a store to shared
    // memory between two global loads would otherwise serialise them.
    float dgam = 0.f;
    for (int base = tid; base < kDk * kDv / 8; base += 4 * kBtThreads) {  // S and dS': 8 groups of 8 per thread
        float4 v[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int idx = base + u * kBtThreads, r = idx >> 4, c8 = (idx & 15) * 8;
            v[u][0] = *reinterpret_cast<const float4*>(bw + kBwS + r * kDv + c8);
            v[u][1] = *reinterpret_cast<const float4*>(bw + kBwS + r * kDv + c8 + 4);
            v[u][2] = *reinterpret_cast<const float4*>(bw + kBwDSe + r * kDv + c8);
            v[u][3] = *reinterpret_cast<const float4*>(bw + kBwDSe + r * kDv + c8 + 4);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int idx = base + u * kBtThreads, r = idx >> 4, c8 = (idx & 15) * 8;
            const uint32_t off = sw128_offset(r, c8, 128);
            const float sx[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w, v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
            const float ex[8] = {v[u][2].x, v[u][2].y, v[u][2].z, v[u][2].w, v[u][3].x, v[u][3].y, v[u][3].z, v[u][3].w};
            store_split8(sm + T_S, sm + T_S + 32768, off, sx);
            store_split8(sm + T_DS, sm + T_DS + 32768, off, ex);
#pragma unroll
            for (int e = 0; e < 8; ++e) dgam += sx[e] * ex[e];
        }
    }
    {  // Kd and w: 4 groups each per thread; Aqk (rows j, columns t: the MN-major A^T): 2 groups
        float4 v[4][4], a[2][2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // chunk-major tiles: consecutive threads take consecutive rows
            const int idx = tid + u * kBtThreads, r = idx & 63, c8 = (idx >> 6) * 8;
            v[u][0] = *reinterpret_cast<const float4*>(fw + kWsKd + cm_offset(r, c8));
            v[u][1] = *reinterpret_cast<const float4*>(fw + kWsKd + cm_offset(r, c8 + 4));
            v[u][2] = *reinterpret_cast<const float4*>(fw + kWsW + cm_offset(r, c8));
            v[u][3] = *reinterpret_cast<const float4*>(fw + kWsW + cm_offset(r, c8 + 4));
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = tid + u * kBtThreads, r = idx & 63, c8 = (idx >> 6) * 8;
            a[u][0] = *reinterpret_cast<const float4*>(fw + kWsAqk + cm_offset(r, c8));
            a[u][1] = *reinterpret_cast<const float4*>(fw + kWsAqk + cm_offset(r, c8 + 4));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int idx = tid + u * kBtThreads, r = idx & 63, c8 = (idx >> 6) * 8;
            const uint32_t off = sw128_offset(r, c8, 64);
            const float kx[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w, v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
            const float wx[8] = {v[u][2].x, v[u][2].y, v[u][2].z, v[u][2].w, v[u][3].x, v[u][3].y, v[u][3].z, v[u][3].w};
            store_split8(sm + T_A, sm + T_A + 16384, off, kx);
            store_split8(sm + T_A + 49152, sm + T_A + 65536, off, wx);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = tid + u * kBtThreads, r = idx & 63, c8 = (idx >> 6) * 8;
            const float ax[8] = {a[u][0].x, a[u][0].y, a[u][0].z, a[u][0].w, a[u][1].x, a[u][1].y, a[u][1].z, a[u][1].w};
            store_split8(sm + T_A + 32768, sm + T_A + 40960, sw128_offset(r, c8, 64), ax);
        }
    }
    for (int idx = tid; idx < kChunk * kDv / 8; idx += kBtThreads) {  // do rows t (zero past T)
        const int r = idx >> 4, c8 = (idx & 15) * 8;
        const int64_t t = t0 + r;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (t < p.T)
            u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.dout.p) + (int64_t)b * p.dout.sb +
                                                t * p.dout.st + (int64_t)h * p.dout.sh + c8);
        *reinterpret_cast<uint4*>(sm + T_DOB + sw128_offset(r, c8, 64)) = u;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem, sb = smem_u32(sm);
    // pass p: (A hi, B hi), (A hi, B lo), (A lo, B hi)
    const uint32_t pa[3] = {0u, 0u, 1u}, pb[3] = {0u, 1u, 0u};
    if (tid == 0) {
        const uint32_t id_kmn = make_idesc_f16(64, 128, false, true, true);  // A K-major, B MN-major
        const uint32_t id_mnmn = make_idesc_f16(64, 128, true, true, true);  // A MN-major, B MN-major
        // (1) Kd dS' + Aqk^T do -> [0,128)
        bool acc = false;
        for (int ps = 0; ps < 3; ++ps)
            for (int ks = 0; ks < 8; ++ks, acc = true)
                mma_f16(tm, make_sdesc(sb + T_A + pa[ps] * 16384 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + T_DS + pb[ps] * 32768 + ks * 2048, 16384, 1024, kSwizzle128B), id_kmn, acc);
        for (int ps = 0; ps < 2; ++ps)
            for (int ks = 0; ks < 4; ++ks)
                mma_f16(tm, make_sdesc(sb + T_A + 32768 + ps * 8192 + ks * 2048, 8192, 1024, kSwizzle128B),
                        make_sdesc(sb + T_DOB + ks * 2048, 8192, 1024, kSwizzle128B), id_mnmn, true);
        // (2) w S -> [128,256)
        acc = false;
        for (int ps = 0; ps < 3; ++ps)
            for (int ks = 0; ks < 8; ++ks, acc = true)
                mma_f16(tm + 128, make_sdesc(sb + T_A + 49152 + pa[ps] * 16384 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + T_S + pb[ps] * 32768 + ks * 2048, 16384, 1024, kSwizzle128B), id_kmn, acc);
        mma_commit(&ms.bar);
    }
    bool ok = mbar_wait(&ms.bar, 0, kWaitNs);
    ok = !__syncthreads_or(!ok);
    tc_fence_after();
    // ---- dv_new, v_new from the accumulators (M=64: rows 16 q + l in lanes 32 q + l, l < 16); warps w and
    //      w + 4 share a quadrant and split the 128 columns
    const int q = warp & 3, chalf = warp >> 2, row = 16 * q + (lane & 15);
    const bool rl = lane < 16;
    if (ok) {
        for (int part = 0; part < 2; ++part) {
            float d[32];
            const int col0 = 64 * chalf + 32 * part;
            tmem_ld32(tmem_addr(tm, 32 * q, col0), d);  // dv_new (its record is written at the end)
            tmem_ld_wait();
            if (rl) {
#pragma unroll
                for (int q8 = 0; q8 < 4; ++q8)  // rows 64.. of the (3) A tile
                    store_split8(sm + T_A, sm + T_A + 32768, sw128_offset(64 + row, col0 + 8 * q8, 128), d + 8 * q8);
            }
            tmem_ld32(tmem_addr(tm, 32 * q, 128 + col0), d);  // w S
            tmem_ld_wait();
            if (rl) {
                float vn[32];
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                    const float4 u = *reinterpret_cast<const float4*>(fw + kWsU + cm_offset(row, col0 + 4 * q4));
                    vn[4 * q4] = u.x - d[4 * q4];
                    vn[4 * q4 + 1] = u.y - d[4 * q4 + 1];
                    vn[4 * q4 + 2] = u.z - d[4 * q4 + 2];
                    vn[4 * q4 + 3] = u.w - d[4 * q4 + 3];
                }
#pragma unroll
                for (int q8 = 0; q8 < 4; ++q8)  // the (4) A tile: hi in place of do's B tile, lo after the w tiles
                    store_split8(sm + T_DOB, sm + T_A + 65536, sw128_offset(row, col0 + 8 * q8, 64), vn + 8 * q8);
            }
        }
    }
    for (int idx = tid; idx < kChunk * kDv / 8; idx += kBtThreads) {  // rows 0..63 of the (3) A tile: do, lo = 0
        const int r = idx >> 4, c8 = (idx & 15) * 8;
        const int64_t t = t0 + r;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (t < p.T)
            u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.dout.p) + (int64_t)b * p.dout.sb +
                                                t * p.dout.st + (int64_t)h * p.dout.sh + c8);
        const uint32_t off = sw128_offset(r, c8, 128);
        *reinterpret_cast<uint4*>(sm + T_A + off) = u;
        *reinterpret_cast<uint4*>(sm + T_A + 32768 + off) = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (ok && tid == 0) {
        const uint32_t id_kk128 = make_idesc_f16(128, 128, false, false, true);
        const uint32_t id_kk64 = make_idesc_f16(64, 128, false, false, true);
        // (3) [do; dv_new] S^T -> [256,384): A K-major [128][128] (atom columns of 16 KiB), B = S K-major
        bool acc = false;
        for (int ps = 0; ps < 3; ++ps)
            for (int ks = 0; ks < 8; ++ks, acc = true)
                mma_f16(tm + 256, make_sdesc(sb + T_A + pa[ps] * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + T_S + pb[ps] * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        id_kk128, acc);
        // (4) v_new dS'^T -> [384,512): A K-major [64][128] (atom columns of 8 KiB), B = dS' K-major
        const uint32_t vh = sb + T_DOB, vl = sb + T_A + 65536;
        acc = false;
        for (int ps = 0; ps < 3; ++ps)
            for (int ks = 0; ks < 8; ++ks, acc = true)
                mma_f16(tm + 384, make_sdesc((pa[ps] ? vl : vh) + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + T_DS + pb[ps] * 32768 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        id_kk64, acc);
        mma_commit(&ms.bar);
    }
    if (ok) ok = mbar_wait(&ms.bar, 1, kWaitNs);
    ok = !__syncthreads_or(!ok);
    tc_fence_after();
    if (ok) {
        // The records, each warp's 32 (M=128) or 16 (M=64) rows x 32 columns at a time through its staging tile in
        // the S operand region (read by the MMAs just completed): (3) row 32 q + lane, (1) (2) (4) row 16 q + lane.
        // dQg and dKd are read only by the chain-rule kernel (a lane per row): stored chunk-major straight from
        // the accumulator rows; dw, dv_new and v_new row-major.
        float* stage = reinterpret_cast<float*>(sm + T_S) + warp * 32 * 36;
        for (int part = 0; part < 2; ++part) {
            float d[32];
            const int col0 = 64 * chalf + 32 * part;
            tmem_ld32(tmem_addr(tm, 32 * q, 256 + col0), d);  // (3): rows 0-63 dQg, 64-127 -dw
            tmem_ld_wait();
            if (q < 2) {
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4)
                    *reinterpret_cast<float4*>(bw + kBwDQg + cm_offset(32 * q + lane, col0 + 4 * q4)) =
                        make_float4(d[4 * q4], d[4 * q4 + 1], d[4 * q4 + 2], d[4 * q4 + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) d[e] = -d[e];
                store_rows_coalesced<32>(stage, d, bw + kBwDW + (32 * (q & 1)) * kDk + col0, kDk, lane);
            }
            tmem_ld32(tmem_addr(tm, 32 * q, 384 + col0), d);  // (4) dKd, M=64
            tmem_ld_wait();
            if (rl) {
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4)
                    *reinterpret_cast<float4*>(bw + kBwDKd + cm_offset(row, col0 + 4 * q4)) =
                        make_float4(d[4 * q4], d[4 * q4 + 1], d[4 * q4 + 2], d[4 * q4 + 3]);
            }
            tmem_ld32(tmem_addr(tm, 32 * q, col0), d);  // (1) dv_new, M=64
            tmem_ld_wait();
            store_rows_coalesced<32, 16>(stage, d, bw + kBwDVn + (16 * q) * kDv + col0, kDv, lane);
            tmem_ld32(tmem_addr(tm, 32 * q, 128 + col0), d);  // (2) w S, M=64: v_new = u - w S
            tmem_ld_wait();
            if (rl) {
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                    const float4 u = *reinterpret_cast<const float4*>(fw + kWsU + cm_offset(row, col0 + 4 * q4));
                    d[4 * q4] = u.x - d[4 * q4];
                    d[4 * q4 + 1] = u.y - d[4 * q4 + 1];
                    d[4 * q4 + 2] = u.z - d[4 * q4 + 2];
                    d[4 * q4 + 3] = u.w - d[4 * q4 + 3];
                }
            }
            store_rows_coalesced<32, 16>(stage, d, bw + kBwVn + (16 * q) * kDv + col0, kDv, lane);
        }
    }
    dgam = warp_sum(dgam);
    if (lane == 0) ms.red[warp] = dgam;
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < kBtThreads / 32; ++w) t += ms.red[w];
        bw[kBwSmall] = t;
        if (!ok) report(p.err, kErrTimeoutPrep);
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kBtTmemCols);
    }
}

// ============================================================================ backward WY terms
// gdn_bwd_wy_tc: the WY part of the chunk's backward in bf16 mode, one CTA (16 warps) per chunk; the
// CUDA-core gdn_bwd_wy with its three products on the tensor cores (M=64 accumulators: row 16 q + l in
// lane 32 q + l, l < 16):
//   1. G = k^ k^T (exact bf16 operands) and dAqk = incl(do v_new^T) (v_new as hi/lo)   -> cols [0,64), [64,128)
//   2. L^T from G; dAqk -> its record
//   3. X = [d(beta v) | d(beta e^gc k^)] = (I - L)^-T [dv_new | dw] by back substitution (warps 0-7, one
//      column each), written as hi/lo A tiles; warps 8-15 meanwhile stage [u | w] as hi/lo B tiles
//   4. row-wise: dv = beta d(beta v), dKp = beta e^gc d(beta e^gc k^), the dbeta and dgc parts
//   5. dL = strict(X [u | w]^T) (K=256, three hi/lo passes)                               -> cols [128,192)
constexpr int kWtThreads = 512;
constexpr uint32_t kWtTmemCols = 256;
constexpr uint32_t W_K = 0;          // k^ bf16 [64][128], K-major (atom columns 8 KiB apart)
constexpr uint32_t W_DO = 16384;     // do bf16 [64][128], K-major; with W_VN the output staging after step 1
constexpr uint32_t W_VN = 32768;     // v_new hi | lo bf16 [64][128] (16 KiB each)
constexpr uint32_t W_LT = 65536;     // fp32 L^T [64][68]
constexpr uint32_t W_XA = 82944;     // X hi | lo bf16 [64][256] (32 KiB each), K-major (atom columns 8 KiB apart)
constexpr uint32_t W_UW = 148480;    // [u | w] hi | lo, same layout
constexpr uint32_t W_MISC = 214016;
struct WtMisc {
    float gc[64], beta[64], egc[64], ekd[64];
    uint64_t bar;
    uint32_t tmem;
};
constexpr uint32_t W_SMEM = W_MISC + (uint32_t)sizeof(WtMisc) + 1024;
static_assert(W_XA % 1024 == 0 && W_UW % 1024 == 0 && W_LT + 64 * 68 * 4 <= W_XA, "tile alignment");
static_assert(16 * 32 * 20 * 4 <= W_LT - W_DO, "output staging");

__global__ void __launch_bounds__(kWtThreads, 1) gdn_bwd_wy_tc(BwdParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    WtMisc& ms = *reinterpret_cast<WtMisc*>(sm + W_MISC);
    float(*Lt)[68] = reinterpret_cast<float(*)[68]>(sm + W_LT);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* fw = p.fws + ci * kWsChunkFloats;
    float* bw = p.bws + ci * kBwChunkFloats;
    const __nv_bfloat16* dout = reinterpret_cast<const __nv_bfloat16*>(p.dout.p);
    const __nv_bfloat16* vin = reinterpret_cast<const __nv_bfloat16*>(p.v.p);

    if (tid == 0) {  // the substitution's right-hand sides into L2 meanwhile
        bulk_prefetch_l2(bw + kBwDVn, kChunk * kDv * 4);
        bulk_prefetch_l2(bw + kBwDW, kChunk * kDk * 4);
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kWtTmemCols);
        tmem_relinquish();
    }
    if (tid == 32) {
        mbar_init(&ms.bar, 1);
        fence_mbar_init();
    }
    // do rows (bf16) and v_new (fp32 -> hi/lo): two 8-column pieces each a thread
    {
        uint4 du[2];
        float4 vv[2][2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = tid + u * kWtThreads, r = idx >> 4, c8 = (idx & 15) * 8;
            const int64_t t = t0 + r;
            du[u] = t < p.T ? *reinterpret_cast<const uint4*>(dout + (int64_t)b * p.dout.sb + t * p.dout.st +
                                                              (int64_t)h * p.dout.sh + c8)
                            : make_uint4(0u, 0u, 0u, 0u);
            vv[u][0] = *reinterpret_cast<const float4*>(bw + kBwVn + r * kDv + c8);
            vv[u][1] = *reinterpret_cast<const float4*>(bw + kBwVn + r * kDv + c8 + 4);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = tid + u * kWtThreads, r = idx >> 4, c8 = (idx & 15) * 8;
            const uint32_t off = sw128_offset(r, c8, 64);
            *reinterpret_cast<uint4*>(sm + W_DO + off) = du[u];
            const float x[8] = {vv[u][0].x, vv[u][0].y, vv[u][0].z, vv[u][0].w,
                                vv[u][1].x, vv[u][1].y, vv[u][1].z, vv[u][1].w};
            store_split8(sm + W_VN, sm + W_VN + 16384, off, x);
        }
    }
    // this thread's v entries for step 4 (rows ty + 32 r, columns 4 tx and 64 + 4 tx), requested now
    const int ty = tid >> 4, tx = tid & 15;
    const int cols[2] = {4 * tx, 64 + 4 * tx};
    uint2 vraw[2][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int64_t t = t0 + ty + 32 * r;
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf)
            vraw[r][hlf] = t < p.T ? *reinterpret_cast<const uint2*>(vin + (int64_t)b * p.v.sb + t * p.v.st +
                                                                      (int64_t)h * p.v.sh + cols[hlf])
                                   : make_uint2(0u, 0u);
    }
    {  // k^ rows (a warp's 4 rows, 4 columns a lane), normalised as the forward does
        float x[4][4], r;
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) bwd::row4_bf16(p.k, b, t0 + warp + 16 * rr, p.T, h, lane, x[rr]);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int i = warp + 16 * rr;
            bwd::qk_norm(p.k, t0 + i, p.T, p.l2norm, x[rr], r);
            store_bf16x4(sm + W_K, sw128_offset(i, 4 * lane, 64), x[rr]);
        }
    }
    bwd::chunk_gates(p, b, h, t0, ms.gc, ms.beta, ms.egc, ms.ekd, true);  // its barriers publish the tiles
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem, sb = smem_u32(sm);

    // ---- 1. G = k^ k^T -> [0,64); dAqk = do v_new^T -> [64,128)
    if (tid == 0) {
        const uint32_t id = make_idesc_f16(64, 64, false, false, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint64_t d = make_sdesc(sb + W_K + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B);
            mma_f16(tm, d, d, id, ks > 0);
        }
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                mma_f16(tm + 64, make_sdesc(sb + W_DO + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + W_VN + s2 * 16384 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        id, (s2 | ks) != 0);
        mma_commit(&ms.bar);
    }
    bool ok = mbar_wait(&ms.bar, 0, kWaitNs);
    tc_fence_after();
    ok = !__syncthreads_or(!ok);

    // ---- 2. L^T; the dAqk record (through the warp's staging tile over do / v_new, read by the MMAs)
    const int q = warp & 3, cg = warp >> 2, row = 16 * q + (lane & 15), j0 = 16 * cg;
    float* stage = reinterpret_cast<float*>(sm + W_DO) + warp * 32 * 20;
    if (ok) {
        float gv[16];
        tmem_ld16(tmem_addr(tm, 32 * q, j0), gv);
        tmem_ld_wait();
        if (lane < 16) {
            const float bi = ms.beta[row], gci = ms.gc[row];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = j0 + e;
                Lt[j][row] = (row > j) ? -(bi * gv[e]) * expf(gci - ms.gc[j]) : 0.f;
            }
        }
        tmem_ld16(tmem_addr(tm, 32 * q, 64 + j0), gv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) gv[e] = (row >= j0 + e) ? gv[e] : 0.f;
        store_rows_coalesced<16, 16>(stage, gv, bw + kBwDA + (16 * q) * kChunk + j0, kChunk, lane);
    }
    __syncthreads();  // L^T is complete

    // ---- 3. back substitution (warps 0-7) | [u | w] hi/lo B tiles (warps 8-15)
    if (tid < kDv + kDk) {  // x_i = rhs_i + sum_{m > i} L_mi x_m, i = 63 .. 0, for column tid
        const int col = tid;
        const float* src = bw + (col < kDv ? kBwDVn + col : kBwDW + (col - kDv));
        float x[kChunk];
#pragma unroll
        for (int i = 0; i < kChunk; ++i) x[i] = src[i * kDv];
#pragma unroll
        for (int i = kChunk - 2; i >= 0; --i) {
            float a0 = x[i], a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int m4 = (i + 1) / 4; m4 < kChunk / 4; ++m4) {
                const float4 l = *reinterpret_cast<const float4*>(&Lt[i][4 * m4]);  // L_mi = 0 for m <= i
                a0 += l.x * x[4 * m4];
                a1 += l.y * x[4 * m4 + 1];
                a2 += l.z * x[4 * m4 + 2];
                a3 += l.w * x[4 * m4 + 3];
            }
            x[i] = (a0 + a1) + (a2 + a3);
        }
        __nv_bfloat16* xh = reinterpret_cast<__nv_bfloat16*>(sm + W_XA);
        __nv_bfloat16* xl = reinterpret_cast<__nv_bfloat16*>(sm + W_XA + 32768);
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
            const uint32_t off = sw128_offset(i, col, 64) >> 1;
            const __nv_bfloat16 hb = __float2bfloat16_rn(x[i]);
            xh[off] = hb;
            xl[off] = __float2bfloat16_rn(x[i] - __bfloat162float(hb));
        }
    } else {  // [u | w] rows j: 64 x 256 in 8-column pieces, 8 a thread
        const int t2 = tid - (kDv + kDk);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int idx = t2 + 256 * u, r = idx & 63, c8 = (idx >> 6) * 8;  // chunk-major tiles: rows consecutive
            const float* tile = fw + (c8 < kDv ? kWsU : kWsW);
            const float4 a = *reinterpret_cast<const float4*>(tile + cm_offset(r, c8 & 127)),
                         bq = *reinterpret_cast<const float4*>(tile + cm_offset(r, (c8 & 127) + 4));
            const float x[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
            store_split8(sm + W_UW, sm + W_UW + 32768, sw128_offset(r, c8, 64), x);
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- 5 (issued first). dL = X [u | w]^T -> [128,192): passes (hi, hi), (hi, lo), (lo, hi)
    if (ok && tid == 0) {
        const uint32_t id = make_idesc_f16(64, 64, false, false, true);
        const uint32_t pa[3] = {0u, 0u, 1u}, pb[3] = {0u, 1u, 0u};
#pragma unroll
        for (int ps = 0; ps < 3; ++ps)
#pragma unroll
            for (int ks = 0; ks < 16; ++ks)
                mma_f16(tm + 128,
                        make_sdesc(sb + W_XA + pa[ps] * 32768 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        make_sdesc(sb + W_UW + pb[ps] * 32768 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024, kSwizzle128B),
                        id, (ps | ks) != 0);
        mma_commit(&ms.bar);
    }

    // ---- 4. row-wise terms (rows ty + 32 r, columns cols[hlf] .. + 3), X read back as hi + lo
    if (ok) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int i = ty + 32 * r;
            const int64_t t = t0 + i;
            const float bi = ms.beta[i], be = ms.beta[i] * ms.egc[i];
            float sv = 0.f, sk = 0.f;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const int cc = cols[hlf];
                float xv[4], xk[4], kv[4];
                {
                    const uint32_t ov = sw128_offset(i, cc, 64), ok2 = sw128_offset(i, kDv + cc, 64);
                    float hi[4], lo[4];
                    load_bf16x4_smem(sm + W_XA + ov, hi);
                    load_bf16x4_smem(sm + W_XA + 32768 + ov, lo);
#pragma unroll
                    for (int e = 0; e < 4; ++e) xv[e] = hi[e] + lo[e];
                    load_bf16x4_smem(sm + W_XA + ok2, hi);
                    load_bf16x4_smem(sm + W_XA + 32768 + ok2, lo);
#pragma unroll
                    for (int e = 0; e < 4; ++e) xk[e] = hi[e] + lo[e];
                    load_bf16x4_smem(sm + W_K + sw128_offset(i, cc, 64), kv);
                }
                const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vraw[r][hlf].x));
                const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vraw[r][hlf].y));
                sv += v01.x * xv[0] + v01.y * xv[1] + v23.x * xv[2] + v23.y * xv[3];
                if (t < p.T) {
                    const int64_t ob = (int64_t)b * p.dv.sb + t * p.dv.st + (int64_t)h * p.dv.sh + cc;
                    __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(p.dv.p) + ob;
                    if (p.dv.dtype == GDN_BF16 && (reinterpret_cast<uintptr_t>(o16) & 7) == 0) {
                        *reinterpret_cast<uint2*>(o16) = make_uint2(pack_bf16x2(bi * xv[0], bi * xv[1]),
                                                                    pack_bf16x2(bi * xv[2], bi * xv[3]));
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) store_elem(p.dv.p, ob + e, p.dv.dtype, bi * xv[e]);
                    }
                }
                sk += kv[0] * xk[0] + kv[1] * xk[1] + kv[2] * xk[2] + kv[3] * xk[3];
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                sv += __shfl_xor_sync(0xffffffffu, sv, o);
                sk += __shfl_xor_sync(0xffffffffu, sk, o);
            }
            if (tx == 0) {
                bw[kBwSmall + 64 + i] = sv + ms.egc[i] * sk;  // dbeta: v . d(beta v) + e^gc k^ . d(beta e^gc k^)
                bw[kBwSmall + 128 + i] = be * sk;             // dgc:   (beta e^gc k^) . d(beta e^gc k^)
            }
        }
    }
    if (ok) {  // dKp = beta e^gc d(beta e^gc k^), chunk-major (read by the chain-rule kernel a lane per row)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int idx = tid + u * kWtThreads, r = idx & 63, col = 4 * (idx >> 6);
            const uint32_t off = sw128_offset(r, kDv + col, 64);
            float hi[4], lo[4];
            load_bf16x4_smem(sm + W_XA + off, hi);
            load_bf16x4_smem(sm + W_XA + 32768 + off, lo);
            const float be = ms.beta[r] * ms.egc[r];
            *reinterpret_cast<float4*>(bw + kBwDKp + cm_offset(r, col)) =
                make_float4(be * (hi[0] + lo[0]), be * (hi[1] + lo[1]), be * (hi[2] + lo[2]), be * (hi[3] + lo[3]));
        }
    }
    if (ok) ok = mbar_wait(&ms.bar, 1, kWaitNs);
    tc_fence_after();
    ok = !__syncthreads_or(!ok);
    if (ok) {  // the dL record (strictly lower)
        float gv[16];
        tmem_ld16(tmem_addr(tm, 32 * q, 128 + j0), gv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) gv[e] = (row > j0 + e) ? gv[e] : 0.f;
        store_rows_coalesced<16, 16>(stage, gv, bw + kBwDL + (16 * q) * kChunk + j0, kChunk, lane);
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && !ok) report(p.err, kErrTimeoutPrep);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, kWtTmemCols);
    }
}

// ============================================================================ backward gradients
// gdn_bwd_grads_tc: the chain rule of one chunk in bf16 mode, one CTA (16 warps) per chunk, with the products
// of the CUDA-core gdn_bwd_grads on the tensor cores:
//   1. [k^; q^] k^T (M=128, N=64, K=Dk, exact bf16 operands) -> lanes 0-63 G = k^ k^T, 64-127 q^ k^T
//   2. the 64x64 terms: dP = dAqk E, dG = -beta_i E dL (strictly lower), R = Aqk . dAqk + L . dL
//      (dgc_i += sum_j R_ij - sum_j R_ji), dbeta_i += sum_j (-G E)_ij dL_ij
//   3. [dP; dG + dG^T] k^ + [0; Dk^-1/2 dP^T] q^ (M=128, N=128, K=64 tokens, hi/lo A operands): lanes 0-63
//      the dQ rows without e^gc dQg, lanes 64-127 the dk^ rows without e^(gc_last-gc) dKd + dKp
//   4. per row: the remaining terms, dgc's Qg . dQg and Kd . dKd terms, the l2norm's derivative, the outputs
// dAqk, dL, dKp and the dbeta / dgc parts come from gdn_bwd_wy, dQg, dKd and <S_c, dS_{c+1}> from
// gdn_bwd_states_tc.
constexpr int kGtThreads = 512;
constexpr uint32_t kGtTmemCols = 256;  // cols [0,64): step 1, [64,192): step 3
constexpr int kGLd = 68;               // fp32 row stride of the 64x64 tiles
constexpr uint32_t G_KQ = 0;           // bf16 [128 rows][128] swizzled: rows 0-63 k^, 64-127 q^ (atom columns 16 KiB apart)
constexpr uint32_t G_A1 = 32768;       // [dP; dG + dG^T] hi | lo: K-major A tiles, 128 rows x 64 tokens (16 KiB each)
constexpr uint32_t G_A2 = 65536;       // [0; Dk^-1/2 dP^T] hi | lo
constexpr uint32_t G_P = 98304;        // fp32 dAqk, then dP
constexpr uint32_t G_L = G_P + 64 * kGLd * 4;  // fp32 dL, then dG
constexpr uint32_t G_R = G_L + 64 * kGLd * 4;  // fp32 R [64][65]
constexpr uint32_t G_MISC = G_R + 64 * 65 * 4;
struct GtMisc {
    float gc[64], beta[64], egc[64], ekd[64], rq[64], rk[64];
    float dgc[64], dbeta[64], colr[64], kdot[64];
    float rowb[4][64];     // sum_j (-G E) dL over each 16-column part
    float dot[4][128][2];  // per 32-column part and row: (q^ . dQg | k^ . dKd, x^ . g)
    uint64_t bar;
    uint32_t tmem;
};
constexpr uint32_t G_SMEM = G_MISC + (uint32_t)sizeof(GtMisc) + 1024;  // + alignment slack
static_assert(G_MISC % 8 == 0, "barrier alignment");

// As mma_split_a, adding to the accumulator from the first pass on.
__device__ __forceinline__ void mma_split_a_acc(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_tile,
                                                uint32_t b_lbo, uint32_t idesc) {
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
            mma_f16(d_tmem, make_sdesc((s2 ? a_lo : a_hi) + ks * 32, 16, 1024, kSwizzle128B),
                    make_sdesc(b_tile + ks * 2048, b_lbo, 1024, kSwizzle128B), idesc, true);
}

__global__ void __launch_bounds__(kGtThreads, 1) gdn_bwd_grads_tc(BwdParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    GtMisc& ms = *reinterpret_cast<GtMisc*>(sm + G_MISC);
    float(*sP)[kGLd] = reinterpret_cast<float(*)[kGLd]>(sm + G_P);
    float(*sL)[kGLd] = reinterpret_cast<float(*)[kGLd]>(sm + G_L);
    float(*sR)[65] = reinterpret_cast<float(*)[65]>(sm + G_R);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quad = warp & 3, part = warp >> 2;  // TMEM lane quadrant, column part
    const int64_t ci = blockIdx.x;
    const int c = (int)(ci % p.NC), bh = (int)(ci / p.NC), b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float* bw = p.bws + ci * kBwChunkFloats;
    const float scale = rsqrtf((float)kDk);

    // dAqk and dL by asynchronous copies; the dbeta / dgc parts; TMEM and the barrier
    for (int idx = tid; idx < kChunk * kChunk / 4; idx += kGtThreads) {
        const int i = idx >> 4, j4 = (idx & 15) * 4;
        cp_async16_rec(&sP[i][j4], bw + kBwDA + i * kChunk + j4);
        cp_async16_rec(&sL[i][j4], bw + kBwDL + i * kChunk + j4);
    }
    cp_async_commit_rec();
    // the dbeta / dgc parts, g and beta: loaded into registers now, stored after the q/k rows are requested
    float sdb = 0.f, sdg = 0.f, gv0 = 0.f, bv0 = 0.f;
    if (tid < kChunk) {
        sdb = bw[kBwSmall + 64 + tid];
        sdg = bw[kBwSmall + 128 + tid];
        const int64_t t = t0 + tid;
        if (t < p.T) {
            gv0 = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            bv0 = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
    }
    if (warp == 0) {
        tmem_alloc(&ms.tmem, kGtTmemCols);
        tmem_relinquish();
    }
    if (tid == 32) {
        mbar_init(&ms.bar, 1);
        fence_mbar_init();
    }
    if (tid == 64) {  // step 4's records (dQg; dKd and dKp, adjacent) into L2 while steps 1-3 run
        bulk_prefetch_l2(bw + kBwDQg, kChunk * kDk * 4);
        bulk_prefetch_l2(bw + kBwDKd, 2 * kChunk * kDk * 4);
    }
    {  // q^, k^ rows (a warp's 4 rows of each, 4 columns a lane), normalised as the forward does -> the bf16 tile
        constexpr int kR = kChunk / (kGtThreads / 32);
        float xq[kR][4], xk[kR][4];
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) {
            const int64_t t = t0 + warp + (kGtThreads / 32) * rr;
            bwd::row4_bf16(p.q, b, t, p.T, h, lane, xq[rr]);
            bwd::row4_bf16(p.k, b, t, p.T, h, lane, xk[rr]);
        }
#pragma unroll
        for (int rr = 0; rr < kR; ++rr) {
            const int i = warp + (kGtThreads / 32) * rr;
            float r;
            bwd::qk_norm(p.q, t0 + i, p.T, p.l2norm, xq[rr], r);
            if (lane == 0) ms.rq[i] = r;
            store_bf16x4(sm + G_KQ, sw128_offset(64 + i, 4 * lane, 128), xq[rr]);
            bwd::qk_norm(p.k, t0 + i, p.T, p.l2norm, xk[rr], r);
            if (lane == 0) ms.rk[i] = r;
            store_bf16x4(sm + G_KQ, sw128_offset(i, 4 * lane, 128), xk[rr]);
        }
    }
    if (tid < kChunk) {
        ms.dbeta[tid] = sdb;
        ms.dgc[tid] = sdg;
        ms.gc[tid] = gv0;
        ms.beta[tid] = bv0;
    }
    cp_async_wait_rec();
    __syncthreads();
    if (warp == 1) {  // inclusive scan of g over the chunk, two values a lane, as the tensor-core prep forms it
        const float g0 = ms.gc[2 * lane], g1 = ms.gc[2 * lane + 1];
        float x = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        const float gc0 = x - g1, gcl = __shfl_sync(0xffffffffu, x, 31);
        ms.gc[2 * lane] = gc0;
        ms.gc[2 * lane + 1] = x;
        ms.egc[2 * lane] = expf(gc0);
        ms.egc[2 * lane + 1] = expf(x);
        ms.ekd[2 * lane] = expf(gcl - gc0);
        ms.ekd[2 * lane + 1] = expf(gcl - x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = ms.tmem;
    const uint32_t sbase = smem_u32(sm);

    // ---- 1. [k^; q^] k^T -> cols [0,64)
    if (tid == 0) {
        const uint32_t id = make_idesc_f16(128, 64, false, false, true);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint64_t d = make_sdesc(sbase + G_KQ + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024, kSwizzle128B);
            mma_f16(tm, d, d, id, ks > 0);  // B reads only rows 0-63 (k^) of the same tile
        }
        mma_commit(&ms.bar);
    }
    bool ok = mbar_wait(&ms.bar, 0, kWaitNs);
    tc_fence_after();
    ok = !__syncthreads_or(!ok);

    // ---- 2. the 64x64 terms: thread (quadrant, lane, part) holds row r of step 1, columns j0 .. j0+15
    const int r = 32 * quad + lane, i = r & 63, j0 = 16 * part;
    float ra[16];  // Aqk . dAqk of this thread's entries (rows 64-127)
    if (ok) {
        float gv[16];
        tmem_ld16(tmem_addr(tm, 32 * quad, j0), gv);
        tmem_ld_wait();
        const float gci = ms.gc[i];
        if (r < 64) {  // L = -(beta_i G) E strictly lower
            const float bi = ms.beta[i];
            float rb = 0.f;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = j0 + e;
                const float dl = sL[i][j];
                float dg = 0.f, rl = 0.f;
                if (j < i) {
                    const float E = expf(gci - ms.gc[j]);
                    const float lb = -gv[e] * E;
                    rl = bi * lb * dl;
                    rb += lb * dl;
                    dg = -bi * E * dl;
                }
                sL[i][j] = dg;
                sR[i][j] = rl;
            }
            ms.rowb[part][i] = rb;
        } else {  // Aqk = Dk^-1/2 (q^ k^T) E incl. the diagonal
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int j = j0 + e;
                const float da = sP[i][j];
                float dp = 0.f, rv = 0.f;
                if (j <= i) {
                    const float E = expf(gci - ms.gc[j]);
                    rv = (scale * gv[e]) * E * da;
                    dp = da * E;
                }
                sP[i][j] = dp;
                ra[e] = rv;
            }
        }
    }
    __syncthreads();  // dP, dG and R_L are in shared memory
    if (ok) {
        if (r >= 64) {  // R += Aqk . dAqk; dP row i -> A1 row i; Dk^-1/2 (column i of dP) -> A2 row 64 + i
            float a[16], t[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                sR[i][j0 + e] += ra[e];
                a[e] = sP[i][j0 + e];
                t[e] = scale * sP[j0 + e][i];
            }
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) {
                store_split8(sm + G_A1, sm + G_A1 + 16384, sw128_offset(i, j0 + 8 * q8, 128), a + 8 * q8);
                store_split8(sm + G_A2, sm + G_A2 + 16384, sw128_offset(64 + i, j0 + 8 * q8, 128), t + 8 * q8);
            }
        } else {  // (dG + dG^T) row i -> A1 row 64 + i; A2 row i is zero
            float a[16], z[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                a[e] = sL[i][j0 + e] + sL[j0 + e][i];
                z[e] = 0.f;
            }
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) {
                store_split8(sm + G_A1, sm + G_A1 + 16384, sw128_offset(64 + i, j0 + 8 * q8, 128), a + 8 * q8);
                store_split8(sm + G_A2, sm + G_A2 + 16384, sw128_offset(i, j0 + 8 * q8, 128), z + 8 * q8);
            }
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- 3. [dP; dG + dG^T] k^ + [0; Dk^-1/2 dP^T] q^ -> cols [64,192); the sums of R meanwhile
    if (ok && tid == 0) {
        const uint32_t id = make_idesc_f16(128, 128, false, true, true);
        mma_split_a(tm + 64, sbase + G_A1, sbase + G_A1 + 16384, sbase + G_KQ, 16384, id);
        mma_split_a_acc(tm + 64, sbase + G_A2, sbase + G_A2 + 16384, sbase + G_KQ + 8192, 16384, id);
        mma_commit(&ms.bar);
    }
    if (tid < kChunk) {  // row sums of R and of (-G E) dL, in a fixed order
        float s = 0.f;
        for (int j = 0; j < kChunk; ++j) s += sR[tid][j];
        ms.dgc[tid] += s;
        ms.dbeta[tid] += ((ms.rowb[0][tid] + ms.rowb[1][tid]) + ms.rowb[2][tid]) + ms.rowb[3][tid];
    } else if (tid < 2 * kChunk) {  // column sums of R
        const int j = tid - kChunk;
        float s = 0.f;
        for (int ii = 0; ii < kChunk; ++ii) s += sR[ii][j];
        ms.colr[j] = s;
    }
    if (ok) ok = mbar_wait(&ms.bar, 1, kWaitNs);
    tc_fence_after();
    ok = !__syncthreads_or(!ok);

    // ---- 4. row r of step 3 (r < 64: dq row i, else dk row i), columns cb .. cb+31
    const int cb = 32 * part;
    const bool qrow = r < 64;
    const int64_t t = t0 + i;
    const bool in = t < p.T;
    const float rr = qrow ? ms.rq[i] : ms.rk[i];
    float gq[32], xh[32];
    float d1 = 0.f, d2 = 0.f;
    if (ok) {
        const View4& X = qrow ? p.q : p.k;
        const __nv_bfloat16* xrow = reinterpret_cast<const __nv_bfloat16*>(X.p) + (int64_t)b * X.sb +
                                    (in ? t : t0) * X.st + (int64_t)h * X.sh + cb;
        uint4 raw[4];
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) raw[q8] = in ? reinterpret_cast<const uint4*>(xrow)[q8] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int c0 = cb + 16 * hf;
            float4 x1[4], x2[4];  // dQg | dKd, and dKp
            const float* src1 = bw + (qrow ? kBwDQg : kBwDKd);  // chunk-major records: a warp reads 512-byte runs
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                x1[q4] = *reinterpret_cast<const float4*>(src1 + cm_offset(i, c0 + 4 * q4));
                x2[q4] = qrow ? make_float4(0.f, 0.f, 0.f, 0.f)
                              : *reinterpret_cast<const float4*>(bw + kBwDKp + cm_offset(i, c0 + 4 * q4));
            }
            float v[16];
            tmem_ld16(tmem_addr(tm, 32 * quad, 64 + c0), v);
            tmem_ld_wait();
            const float ex = qrow ? ms.egc[i] : ms.ekd[i];
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) {
                const uint4 hu = *reinterpret_cast<const uint4*>(sm + G_KQ + sw128_offset(qrow ? 64 + i : i, c0 + 8 * q8, 128));
                const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&hu);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int k = 8 * q8 + e;
                    const float4 a1 = x1[k >> 2], a2 = x2[k >> 2];
                    const float y1 = (k & 3) == 0 ? a1.x : (k & 3) == 1 ? a1.y : (k & 3) == 2 ? a1.z : a1.w;
                    const float y2 = (k & 3) == 0 ? a2.x : (k & 3) == 1 ? a2.y : (k & 3) == 2 ? a2.z : a2.w;
                    const float g = v[k] + ex * y1 + y2;
                    gq[16 * hf + k] = qrow ? scale * g : g;
                    d1 += __bfloat162float(hb[e]) * y1;
                }
            }
        }
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
            const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&raw[q8]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                xh[8 * q8 + e] = __bfloat162float(xb[e]) * rr;
                d2 += xh[8 * q8 + e] * gq[8 * q8 + e];
            }
        }
        ms.dot[part][r][0] = d1;
        ms.dot[part][r][1] = d2;
    }
    __syncthreads();
    if (ok && in) {  // dx = r (dx^ - x^ (x^ . dx^)) with the l2norm, dx^ otherwise
        const float dot = ((ms.dot[0][r][1] + ms.dot[1][r][1]) + ms.dot[2][r][1]) + ms.dot[3][r][1];
        const Out4& O = qrow ? p.dq : p.dk;
        const int64_t ob = (int64_t)b * O.sb + t * O.st + (int64_t)h * O.sh + cb;
        float o[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = p.l2norm ? rr * (gq[e] - xh[e] * dot) : gq[e];
        __nv_bfloat16* ob16 = reinterpret_cast<__nv_bfloat16*>(O.p) + ob;
        if (O.dtype == GDN_BF16 && (reinterpret_cast<uintptr_t>(ob16) & 15) == 0) {  // four 16-byte stores
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8)
                reinterpret_cast<uint4*>(ob16)[q8] =
                    make_uint4(pack_bf16x2(o[8 * q8], o[8 * q8 + 1]), pack_bf16x2(o[8 * q8 + 2], o[8 * q8 + 3]),
                               pack_bf16x2(o[8 * q8 + 4], o[8 * q8 + 5]), pack_bf16x2(o[8 * q8 + 6], o[8 * q8 + 7]));
        } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) store_elem(O.p, ob + e, O.dtype, o[e]);
        }
    }
    if (tid < kChunk) {  // dgc_i: - sum_j R_ji + e^gc Dk^-1/2 (q^ . dQg) - e^(gc_last-gc) (k^ . dKd)
        const float dq1 = ((ms.dot[0][tid][0] + ms.dot[1][tid][0]) + ms.dot[2][tid][0]) + ms.dot[3][tid][0];
        const float dk1 = ((ms.dot[0][64 + tid][0] + ms.dot[1][64 + tid][0]) + ms.dot[2][64 + tid][0]) +
                          ms.dot[3][64 + tid][0];
        ms.kdot[tid] = ms.ekd[tid] * dk1;
        ms.dgc[tid] += -ms.colr[tid] + ms.egc[tid] * scale * dq1 - ms.kdot[tid];
    }
    __syncthreads();
    if (tid == 0) {  // dgc_last += sum_i Kd . dKd + e^gc_last <S_c, dS_{c+1}>
        float dgl = 0.f;
        for (int ii = 0; ii < kChunk; ++ii) dgl += ms.kdot[ii];
        ms.dgc[kChunk - 1] += dgl + ms.egc[kChunk - 1] * bw[kBwSmall];
        if (!ok) report(p.err, kErrTimeoutPrep);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {  // dg_t = sum_{i >= t} dgc_i: suffix scan over the chunk, two rows per lane
        const float a0 = ms.dgc[2 * lane], a1 = ms.dgc[2 * lane + 1];
        float x = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_down_sync(0xffffffffu, x, o);
            if (lane + o < 32) x += y;
        }
        const float dg[2] = {x, x - a0};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int ii = 2 * lane + e;
            const int64_t tt = t0 + ii;
            if (ok && tt < p.T) {
                store_elem(p.dg.p, (int64_t)b * p.dg.sb + tt * p.dg.st + (int64_t)h * p.dg.sh, p.dg.dtype, dg[e]);
                store_elem(p.dbeta.p, (int64_t)b * p.dbeta.sb + tt * p.dbeta.st + (int64_t)h * p.dbeta.sh,
                           p.dbeta.dtype, ms.dbeta[ii]);
            }
        }
        tc_fence_after();
        tmem_dealloc(tm, kGtTmemCols);
    }
}

// Packed sequences: chunk_base[n] = sum_{m<n} ceil(T_m / 64) and chunk_seq[j] = the sequence of global
// chunk j, from the device's cu_seqlens, so the host never reads the offsets.  One CTA: each thread
// counts the chunks of a contiguous run of sequences, a block scan turns the counts into bases, and
// each thread writes its run.  Offsets that do not start at 0, decrease, or end at T set
// kErrBadSeqlens and leave zero chunks (every base 0), so the prep and scan do nothing.
constexpr int kOrderMax = 2048;

__global__ void __launch_bounds__(256) gdn_varlen_tables(ChunkParams p, int* chunk_base, int* chunk_seq) {
    __shared__ int part[256];
    __shared__ int ncs[kOrderMax];
    __shared__ int bad;
    const int tid = threadIdx.x, N = p.N;
    if (tid == 0) bad = 0;
    __syncthreads();
    for (int n = tid; n <= N; n += 256) {
        const int v = p.cu_seqlens[n];
        if ((n == 0 && v != 0) || (n == N && (int64_t)v != p.T) || (n < N && p.cu_seqlens[n + 1] < v)) bad = 1;
    }
    __syncthreads();
    const int per = (N + 255) / 256;
    const int n0 = min(N, tid * per), n1 = min(N, n0 + per);
    int local = 0;
    if (!bad)
        for (int n = n0; n < n1; ++n) local += (p.cu_seqlens[n + 1] - p.cu_seqlens[n] + kChunk - 1) / kChunk;
    part[tid] = local;
    __syncthreads();
    for (int o = 1; o < 256; o <<= 1) {  // inclusive block scan
        const int v = tid >= o ? part[tid - o] : 0;
        __syncthreads();
        part[tid] += v;
        __syncthreads();
    }
    const bool ok = !bad && part[255] <= p.max_chunks;
    int base = ok ? part[tid] - local : 0;
    for (int n = n0; n < n1; ++n) {
        chunk_base[n] = base;
        const int nc = ok ? (p.cu_seqlens[n + 1] - p.cu_seqlens[n] + kChunk - 1) / kChunk : 0;
        for (int c = 0; c < nc; ++c) chunk_seq[base + c] = n;
        base += nc;
    }
    if (tid == 0) {
        chunk_base[N] = ok ? part[255] : 0;
        if (!ok) report(p.err, kErrBadSeqlens);
    }
    // Sequences by chunk count, longest first (stable): rank = #{m : nc_m > nc_n, or equal with m < n}.  The
    // O(N^2) ranking serves up to kOrderMax sequences; beyond that the natural order is kept.
    int* order = const_cast<int*>(p.seq_order);
    if (N <= kOrderMax) {
        for (int n = tid; n < N; n += 256) ncs[n] = ok ? (p.cu_seqlens[n + 1] - p.cu_seqlens[n] + kChunk - 1) / kChunk : 0;
        __syncthreads();
        for (int n = tid; n < N; n += 256) {
            const int v = ncs[n];
            int rank = 0;
            for (int m = 0; m < N; ++m) rank += (ncs[m] > v) | ((ncs[m] == v) & (m < n));
            order[rank] = n;
        }
    } else {
        for (int n = tid; n < N; n += 256) order[n] = n;
    }
}

}  // namespace

namespace {
// One bounded wait that must run out: an mbarrier nobody arrives on, waited on with the same
// mbar_wait the chunk kernels use.  When the limit passes the kernel reports kErrWaitSelftest
// and returns, as a chunk kernel whose wait gave up would.
__global__ void __launch_bounds__(32) gdn_selftest_wait(unsigned int* err, uint64_t timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    const bool ok = mbar_wait(&bar, 0, timeout_ns);
    if (!ok && threadIdx.x == 0) report(err, kErrWaitSelftest);
}
}  // namespace

cudaError_t launch_selftest_wait(unsigned int* err, uint64_t timeout_ns, cudaStream_t stream) {
    gdn_selftest_wait<<<1, 32, 0, stream>>>(err, timeout_ns);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

cudaError_t launch_varlen_tables(const ChunkParams& p, cudaStream_t stream) {
    gdn_varlen_tables<<<1, 256, 0, stream>>>(p, const_cast<int*>(p.chunk_base), const_cast<int*>(p.chunk_seq));
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

// cudaFuncSetAttribute once per (kernel, device): the per-call host path stays short and free of
// calls that stream capture might refuse.
template <typename Kernel>
cudaError_t smem_attr_once(Kernel kernel, int bytes, std::atomic<uint64_t>& done_mask) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_release);
    return e;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            f = nullptr;
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// The prep's box map of a bf16 [B, T, H, 128] view (strides in elements, all multiples of 8: the tensor-core
// path's condition).  A dimension of extent 1 gets a nominal stride (its coordinate is always 0).
bool encode_rows_map(CUtensorMap* m, const View4& v, int64_t B, int64_t T, int64_t H) {
    const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc || B <= 0 || T <= 0 || H <= 0) return false;
    const cuuint64_t sh = H > 1 ? (cuuint64_t)v.sh * 2 : 256;
    const cuuint64_t st = T > 1 ? (cuuint64_t)v.st * 2 : sh * (cuuint64_t)H;
    const cuuint64_t sb = B > 1 ? (cuuint64_t)v.sb * 2 : st * (cuuint64_t)T;
    const cuuint64_t dims[4] = {(cuuint64_t)kDk, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[3] = {sh, st, sb};
    const cuuint32_t box[4] = {(cuuint32_t)kDk, 1, (cuuint32_t)kChunk, 1}, estr[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v.p), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_chunk_tc_prep(const ChunkParams& p, cudaStream_t stream) {
    static_assert(P_SMEM <= 227 * 1024, "shared memory budget");
    static_assert(sizeof(PrepMisc) <= 1088, "misc region");
    static std::atomic<uint64_t> attr_done{0};
    cudaError_t e = smem_attr_once(gdn_prep_tc, (int)P_SMEM, attr_done);
    if (e != cudaSuccess) return e;
    const int64_t nchunks = p.cu_seqlens ? (int64_t)p.max_chunks * p.H : (int64_t)p.B * p.H * p.NC;
    PrepMaps maps{};
    // the maps are 4-D over (D, H, T, B) with a 32-bit token coordinate
    maps.use = p.T <= 0x7fffffffLL && encode_rows_map(&maps.m[0], p.q, p.B, p.T, p.H) &&
               encode_rows_map(&maps.m[1], p.k, p.B, p.T, p.H) && encode_rows_map(&maps.m[2], p.v, p.B, p.T, p.H);
    gdn_prep_tc<<<(unsigned)nchunks, kPrepThreads, P_SMEM, stream>>>(p, maps);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

namespace {
template <int kW>
cudaError_t launch_scan_w(const ChunkParams& p, cudaStream_t stream) {
    using L = ScanLayout<kW>;
    static std::atomic<uint64_t> attr_done{0};
    cudaError_t e = smem_attr_once(gdn_scan_tc<kW>, (int)L::kSmem, attr_done);
    if (e != cudaSuccess) return e;
    const dim3 grid = p.cu_seqlens ? dim3((unsigned)(p.N * p.H * L::kSlices), 1)
                                   : dim3((unsigned)(p.B * p.H), (p.scan_mode == 1 ? 2 : 1) * L::kSlices);
    gdn_scan_tc<kW><<<grid, kScanThreads, L::kSmem, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}
}  // namespace

cudaError_t launch_scan_lean(const ChunkParams& p, cudaStream_t stream) {
    static std::atomic<uint64_t> attr_done{0};
    cudaError_t e = smem_attr_once(gdn_scan_lean_tc, (int)kLeanSmem, attr_done);
    if (e != cudaSuccess) return e;
    gdn_scan_lean_tc<<<(unsigned)((int64_t)p.B * p.H * kLeanSlices), kLeanThreads, kLeanSmem, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

// The scan is a chain of dependent chunk steps per CTA: 16-column slices shorten each step, but double the
// CTAs; they are used while all of them fit in one wave (one CTA per SM).  Beyond that the lean scan runs two
// 32-column chains per SM (the 32-column gdn_scan_tc for packed batches, shard summaries and the backward's
// recompute).
cudaError_t launch_chunk_tc_scan(const ChunkParams& p, cudaStream_t stream) {
    static std::atomic<int> nsm_cache[64];  // SM count per device, filled on first use (any host thread)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    int nsm = nsm_cache[dev].load(std::memory_order_relaxed);
    if (!nsm) {
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 1;
        nsm_cache[dev].store(nsm, std::memory_order_relaxed);
    }
    const int64_t rows = p.cu_seqlens ? (int64_t)p.N * p.H : (int64_t)p.B * p.H * (p.scan_mode == 1 ? 2 : 1);
    if (rows * ScanLayout<16>::kSlices <= nsm) return launch_scan_w<16>(p, stream);
    // more chains than one wave of one-per-SM CTAs: two chains per SM (fixed-length forward)
    if (!p.cu_seqlens && p.scan_mode == 0 && !p.states) return launch_scan_lean(p, stream);
    return launch_scan_w<32>(p, stream);
}

cudaError_t launch_bwd_states_tc(const BwdParams& p, cudaStream_t stream) {
    static_assert(T_SMEM <= 227 * 1024, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(gdn_bwd_states_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)T_SMEM);
    if (e != cudaSuccess) return e;
    gdn_bwd_states_tc<<<(unsigned)((int64_t)p.B * p.H * p.NC), kBtThreads, T_SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

cudaError_t launch_bwd_wy_tc(const BwdParams& p, cudaStream_t stream) {
    static_assert(W_SMEM <= 227 * 1024, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(gdn_bwd_wy_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)W_SMEM);
    if (e != cudaSuccess) return e;
    gdn_bwd_wy_tc<<<(unsigned)((int64_t)p.B * p.H * p.NC), kWtThreads, W_SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

cudaError_t launch_bwd_grads_tc(const BwdParams& p, cudaStream_t stream) {
    static_assert(G_SMEM <= 227 * 1024, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(gdn_bwd_grads_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G_SMEM);
    if (e != cudaSuccess) return e;
    gdn_bwd_grads_tc<<<(unsigned)((int64_t)p.B * p.H * p.NC), kGtThreads, G_SMEM, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

cudaError_t launch_bwd_scan_tc(const BwdParams& p, cudaStream_t stream) {
    static_assert(B_SMEM <= 227 * 1024, "shared memory budget");
    cudaError_t e = cudaFuncSetAttribute(gdn_bwd_scan_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)B_SMEM);
    if (e != cudaSuccess) return e;
    gdn_bwd_scan_tc<<<dim3((unsigned)(p.B * p.H), kDv / kBsCols), kBsThreads, B_SMEM, stream>>>(p);
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
