// Token-recurrent gated delta rule (the decode step), HBM-bound.
//
// Follows torch_recurrent_gated_delta_rule (qwen3_5_transformers.py:190-229):
//   S *= e^g;  kv = S^T k;  delta = beta (v - kv);  S += k delta^T;  o = S^T q
// State columns never interact (column j of kv, delta, S and o only involves column j of S), so the
// 128 x 128 fp32 state of a head is split by columns over four 128-thread CTAs: lane l owns column
// 32 s + l of the CTA's slice s, warp w rows 32w .. 32w+31, held in registers for all T tokens (read from
// HBM once and written once per call; the reference streams it five times per token).  Every state load
// and store of a warp is one contiguous 128-byte row piece.  Small CTAs (16 KB of state each, eight per
// SM) make a decode batch more than one wave of CTAs: CTAs that finish early write their states while the
// next ones read theirs, so the step streams like a copy instead of reading everything, then writing
// everything.  q and k are normalised once per head (redundantly in each of its four CTAs: 512 bytes).
// A single decode token over more heads than one wave of those CTAs holds runs gdn_recurrent_pair_kernel:
// one CTA per pair of slices, the second slice's state landing in shared memory (cp.async) while the first
// computes from registers, so every state load is in flight from the start and the CTAs fit one wave.
#include <atomic>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kRecCols = 32;                 // state columns per CTA (one per lane)
constexpr int kRecSlices = kDv / kRecCols;   // CTAs per head
constexpr int kRecWarps = 4;
constexpr int kRecThreads = 32 * kRecWarps;
constexpr int kRecRows = kDk / kRecWarps;    // state rows per warp (32)

// One token on a CTA's 32 state columns (lane = column; warp w holds rows 32w .. 32w+31 of S): S *= e^g,
// kv = S^T k (each warp's partial over its rows, k broadcast from shared memory four rows per load, then the
// four partials in warp order), delta = beta (v - kv), S += k delta^T and o = S^T q (summed the same way and
// returned to warp 0).  qs / ks hold the token's normalised q (scaled) and k, written before a block barrier
// the caller took.  Two block barriers.
__device__ __forceinline__ float rec_token(float (&S)[kRecRows], const float* qs, const float* ks, float decay,
                                           float beta, float vv, float (*red)[kRecCols], float (*red2)[kRecCols],
                                           int warp, int lane) {
    const int r0 = kRecRows * warp;
    float part = 0.f;
#pragma unroll
    for (int r = 0; r < kRecRows; r += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&ks[r0 + r]);
        const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            S[r + i] *= decay;
            part += S[r + i] * kk[i];
        }
    }
    red[warp][lane] = part;
    __syncthreads();
    float kv = 0.f;
#pragma unroll
    for (int w = 0; w < kRecWarps; ++w) kv += red[w][lane];
    const float delta = (vv - kv) * beta;
    float op = 0.f;
#pragma unroll
    for (int r = 0; r < kRecRows; r += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(&ks[r0 + r]);
        const float4 q4 = *reinterpret_cast<const float4*>(&qs[r0 + r]);
        const float kk[4] = {k4.x, k4.y, k4.z, k4.w}, qq[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            S[r + i] += kk[i] * delta;
            op += S[r + i] * qq[i];
        }
    }
    red2[warp][lane] = op;  // its own array: no barrier between the kv and o reductions
    __syncthreads();
    float o = 0.f;
    if (warp == 0) {
#pragma unroll
        for (int w = 0; w < kRecWarps; ++w) o += red2[w][lane];
    }
    return o;
}

__global__ void __launch_bounds__(kRecThreads, 8) gdn_recurrent_kernel(RecurrentParams p) {
    __shared__ __align__(16) float qs[kDk];
    __shared__ __align__(16) float ks[kDk];
    __shared__ float vs[kRecCols];
    __shared__ float gb[2];
    __shared__ float red[kRecWarps][kRecCols];   // kv partials
    __shared__ float red2[kRecWarps][kRecCols];  // o partials (their own array: no barrier between the two)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x / kRecSlices, slice = blockIdx.x % kRecSlices;
    const int b = bh / p.H, h = bh % p.H;
    const int r0 = kRecRows * warp, col = kRecCols * slice + lane;
    const float scale = rsqrtf((float)kDk);
    const int64_t sbase = (int64_t)bh * kDk * kDv + col;

    // this token's small inputs first (they gate the arithmetic), then the whole state slice in flight
    float x[4] = {0.f, 0.f, 0.f, 0.f}, vg = 0.f;
    auto load_token = [&](int64_t t) {
        if (warp < 2) {  // q (warp 0) and k (warp 1)
            const View4& vw = warp == 0 ? p.q : p.k;
            const int64_t base = (int64_t)b * vw.sb + t * vw.st + (int64_t)h * vw.sh;
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = load_elem(vw.p, base + lane + 32 * i, vw.dtype);
        } else if (warp == 2) {
            vg = load_elem(p.v.p, (int64_t)b * p.v.sb + t * p.v.st + (int64_t)h * p.v.sh + col, p.v.dtype);
        } else if (lane < 2) {
            const View3& vw = lane == 0 ? p.g : p.beta;
            vg = load_elem(vw.p, (int64_t)b * vw.sb + t * vw.st + (int64_t)h * vw.sh, vw.dtype);
        }
    };
    load_token(0);
    float S[kRecRows];
#pragma unroll
    for (int r = 0; r < kRecRows; ++r) S[r] = p.h0 ? p.h0[sbase + (int64_t)(r0 + r) * kDv] : 0.f;

    for (int64_t t = 0; t < p.T; ++t) {
        if (warp < 2) {  // normalised as the reference does
            if (p.l2norm) {
                const float inv = l2norm_inv(x, warp == 0 ? p.q.dtype : p.k.dtype);
#pragma unroll
                for (int i = 0; i < 4; ++i) x[i] = round_to(x[i] * inv, warp == 0 ? p.q.dtype : p.k.dtype);
            }
            float* dst = warp == 0 ? qs : ks;
            const float sc = warp == 0 ? scale : 1.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = x[i] * sc;
        } else if (warp == 2) {
            vs[lane] = vg;
        } else if (lane < 2) {
            gb[lane] = vg;
        }
        __syncthreads();
        if (t + 1 < p.T) load_token(t + 1);  // the next token's inputs arrive during this token's arithmetic

        const float o = rec_token(S, qs, ks, expf(gb[0]), gb[1], vs[lane], red, red2, warp, lane);
        if (warp == 0)
            store_elem(p.out, (int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + col, p.out_dtype, o);
        // No barrier before the next token: its writes of qs/ks/vs/gb come before its first barrier, and
        // every read of them (and of red) for this token came before rec_token's second barrier; red2, which
        // warp 0 is still reading, is rewritten only after the next token's second barrier.
    }

    if (p.hT) {
#pragma unroll
        for (int r = 0; r < kRecRows; ++r) p.hT[sbase + (int64_t)(r0 + r) * kDv] = S[r];
    }
}

// One decode token (T = 1) on two 32-column slices of a head (slices 2 pair and 2 pair + 1), one after the other
// with the same normalised q and k.  The second slice's 16 KB of state is copied into shared memory (cp.async,
// 16-byte pieces of its 128-byte row pieces) while the first slice's loads into registers are in flight and its
// token is computed; then it is read into the same registers.  Half as many CTAs as gdn_recurrent_kernel: a
// decode batch that takes that kernel more than one wave of CTAs fits one here, with every state load issued at
// the start.  The arithmetic of each slice is rec_token's, so the results are bit-identical to that kernel's.
__global__ void __launch_bounds__(kRecThreads, 8) gdn_recurrent_pair_kernel(RecurrentParams p) {
    __shared__ __align__(16) float qs[kDk];
    __shared__ __align__(16) float ks[kDk];
    __shared__ float vs[2][kRecCols];
    __shared__ float gb[2];
    __shared__ float red[kRecWarps][kRecCols];
    __shared__ float red2[kRecWarps][kRecCols];
    __shared__ __align__(16) float second[kDk][kRecCols];  // the second slice's state, rows dk

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x / 2, pair = blockIdx.x % 2;
    const int b = bh / p.H, h = bh % p.H;
    const int r0 = kRecRows * warp;
    const int col0 = 2 * kRecCols * pair + lane, col1 = col0 + kRecCols;  // this lane's column in each slice
    const int64_t head = (int64_t)bh * kDk * kDv;
    const float scale = rsqrtf((float)kDk);

    // the token's inputs, then both slices' states in flight
    float x[4] = {0.f, 0.f, 0.f, 0.f}, v0 = 0.f, v1 = 0.f, gv = 0.f;
    if (warp < 2) {  // q (warp 0) and k (warp 1)
        const View4& vw = warp == 0 ? p.q : p.k;
        const int64_t base = (int64_t)b * vw.sb + (int64_t)h * vw.sh;
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = load_elem(vw.p, base + lane + 32 * i, vw.dtype);
    } else if (warp == 2) {
        const int64_t base = (int64_t)b * p.v.sb + (int64_t)h * p.v.sh;
        v0 = load_elem(p.v.p, base + col0, p.v.dtype);
        v1 = load_elem(p.v.p, base + col1, p.v.dtype);
    } else if (lane < 2) {
        const View3& vw = lane == 0 ? p.g : p.beta;
        gv = load_elem(vw.p, (int64_t)b * vw.sb + (int64_t)h * vw.sh, vw.dtype);
    }
    if (p.h0) {  // 128 rows x 8 pieces of 16 bytes, 8 per thread
        for (int i = tid; i < kDk * 8; i += kRecThreads) {
            const int row = i >> 3, piece = i & 7;
            cp_async16_rec(&second[row][4 * piece],
                           p.h0 + head + (int64_t)row * kDv + 2 * kRecCols * pair + kRecCols + 4 * piece);
        }
        cp_async_commit_rec();
    }
    float S[kRecRows];
#pragma unroll
    for (int r = 0; r < kRecRows; ++r) S[r] = p.h0 ? p.h0[head + (int64_t)(r0 + r) * kDv + col0] : 0.f;

    if (warp < 2) {  // normalised as the reference does
        if (p.l2norm) {
            const float inv = l2norm_inv(x, warp == 0 ? p.q.dtype : p.k.dtype);
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = round_to(x[i] * inv, warp == 0 ? p.q.dtype : p.k.dtype);
        }
        float* dst = warp == 0 ? qs : ks;
        const float sc = warp == 0 ? scale : 1.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = x[i] * sc;
    } else if (warp == 2) {
        vs[0][lane] = v0;
        vs[1][lane] = v1;
    } else if (lane < 2) {
        gb[lane] = gv;
    }
    __syncthreads();
    const float decay = expf(gb[0]), beta = gb[1];
    for (int u = 0; u < 2; ++u) {
        if (u == 1) {  // the second slice: its copy has landed (every thread's pieces, then the barrier)
            cp_async_wait_rec();
            __syncthreads();
#pragma unroll
            for (int r = 0; r < kRecRows; ++r) S[r] = p.h0 ? second[r0 + r][lane] : 0.f;
        }
        const int col = u == 0 ? col0 : col1;
        const float o = rec_token(S, qs, ks, decay, beta, vs[u][lane], red, red2, warp, lane);
        if (warp == 0) store_elem(p.out, (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + col, p.out_dtype, o);
        if (p.hT) {
#pragma unroll
            for (int r = 0; r < kRecRows; ++r) p.hT[head + (int64_t)(r0 + r) * kDv + col] = S[r];
        }
    }
}

}  // namespace

cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream) {
    // Resident CTAs of gdn_recurrent_kernel: eight per SM (its registers).  A single token over more
    // (head, slice) CTAs than that goes to the pair kernel (B=32, H=16 back to back: 15.56 -> 15.15 us).
    static std::atomic<int> nsm_cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    int nsm = nsm_cache[dev].load(std::memory_order_relaxed);
    if (!nsm) {
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 1;
        nsm_cache[dev].store(nsm, std::memory_order_relaxed);
    }
    const int64_t ctas = (int64_t)p.B * p.H * kRecSlices;
    cudaError_t e = phase_event(0, stream);
    if (e != cudaSuccess) return e;
    if (p.T == 1 && ctas > 8 * (int64_t)nsm)
        gdn_recurrent_pair_kernel<<<(unsigned)(ctas / 2), kRecThreads, 0, stream>>>(p);
    else
        gdn_recurrent_kernel<<<(unsigned)ctas, kRecThreads, 0, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return phase_event(1, stream);
}

}  // namespace gdn
