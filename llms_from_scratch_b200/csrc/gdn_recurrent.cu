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
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kRecCols = 32;                 // state columns per CTA (one per lane)
constexpr int kRecSlices = kDv / kRecCols;   // CTAs per head
constexpr int kRecWarps = 4;
constexpr int kRecThreads = 32 * kRecWarps;
constexpr int kRecRows = kDk / kRecWarps;    // state rows per warp (32)

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

        // kv = (e^g S)^T k over this warp's rows (k broadcast from shared memory four rows per load), then the
        // four warps' partials
        const float decay = expf(gb[0]);
        const float beta = gb[1];
        const float vv = vs[lane];
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
        // S += k delta^T; o = S^T q
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
        red2[warp][lane] = op;
        __syncthreads();
        if (warp == 0) {
            float o = 0.f;
#pragma unroll
            for (int w = 0; w < kRecWarps; ++w) o += red2[w][lane];
            store_elem(p.out, (int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + col, p.out_dtype, o);
        }
        // No barrier before the next token: its writes of qs/ks/vs/gb come before its first barrier, and
        // every read of them (and of red) for this token came before the barrier above; red2, which warp 0
        // is still reading, is rewritten only after the next token's second barrier.
    }

    if (p.hT) {
#pragma unroll
        for (int r = 0; r < kRecRows; ++r) p.hT[sbase + (int64_t)(r0 + r) * kDv] = S[r];
    }
}

}  // namespace

cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream) {
    dim3 grid((unsigned)(p.B * p.H * kRecSlices));
    cudaError_t e = phase_event(0, stream);
    if (e != cudaSuccess) return e;
    gdn_recurrent_kernel<<<grid, kRecThreads, 0, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return phase_event(1, stream);
}

}  // namespace gdn
