// Token-recurrent gated delta rule (the decode step), HBM-bound.
//
// Follows torch_recurrent_gated_delta_rule (qwen3_5_transformers.py:190-229):
//   S *= e^g;  kv = S^T k;  delta = beta (v - kv);  S += k delta^T;  o = S^T q
// One 256-thread CTA owns one head's whole 128 x 128 fp32 state for all T tokens:
// the state is read from HBM once and written once per call (the reference
// streams it five times per token).  Warp w holds rows 16w .. 16w+15 and lane l
// columns 4l .. 4l+3 (a float4 per row), so every state load and store of a warp
// is one contiguous 512-byte row, each thread's sums over its rows stay local, and
// only the 8 warps' partial column sums meet in shared memory.  Half of a thread's
// rows live in registers, half in shared memory (filled by cp.async), which keeps
// a CTA at <= 64 registers per thread: four CTAs per SM, so a batch of 32
// sequences x 16 heads is resident at once with every state load in flight from
// the start.  q and k are normalised once per head.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kRecThreads = 256;
constexpr int kRecWarps = kRecThreads / 32;
constexpr int kRecRows = kDk / kRecWarps;  // state rows per warp (16)
constexpr int kRecRegRows = 8;             // rows 0-7 of a warp in registers, 8-15 in shared memory
constexpr int kRecSmemRows = kRecRows - kRecRegRows;

__global__ void __launch_bounds__(kRecThreads, 4) gdn_recurrent_kernel(RecurrentParams p) {
    __shared__ __align__(16) float4 srows[kRecWarps][kRecSmemRows][32];  // [warp][row][lane]: 32 KiB
    __shared__ __align__(16) float qs[kDk];
    __shared__ __align__(16) float ks[kDk];
    __shared__ __align__(16) float vs[kDv];
    __shared__ float gb[2];
    __shared__ __align__(16) float red[kRecWarps][kDv];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh % p.H;
    const int r0 = kRecRows * warp, c0 = 4 * lane;
    const float scale = rsqrtf((float)kDk);

    float S[kRecRegRows][4];
    const int64_t sbase = (int64_t)bh * kDk * kDv + c0;
    // the shared-memory rows first (asynchronous), then the register rows
#pragma unroll
    for (int r = 0; r < kRecSmemRows; ++r) {
        if (p.h0)
            cp_async16_rec(&srows[warp][r][lane], p.h0 + sbase + (int64_t)(r0 + kRecRegRows + r) * kDv);
        else
            srows[warp][r][lane] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit_rec();
#pragma unroll
    for (int r = 0; r < kRecRegRows; ++r) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.h0) v = *reinterpret_cast<const float4*>(p.h0 + sbase + (int64_t)(r0 + r) * kDv);
        S[r][0] = v.x;
        S[r][1] = v.y;
        S[r][2] = v.z;
        S[r][3] = v.w;
    }
    cp_async_wait_rec();  // a thread reads back only the shared rows it copied itself

    for (int64_t t = 0; t < p.T; ++t) {
        if (warp < 2) {  // q (warp 0) and k (warp 1), normalised as the reference does
            const View4& vw = warp == 0 ? p.q : p.k;
            const int64_t base = (int64_t)b * vw.sb + t * vw.st + (int64_t)h * vw.sh;
            float x[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = load_elem(vw.p, base + lane + 32 * i, vw.dtype);
            if (p.l2norm) {
                const float inv = l2norm_inv(x, vw.dtype);
#pragma unroll
                for (int i = 0; i < 4; ++i) x[i] = round_to(x[i] * inv, vw.dtype);
            }
            float* dst = warp == 0 ? qs : ks;
            const float sc = warp == 0 ? scale : 1.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = x[i] * sc;
        } else if (warp == 2) {
            const int64_t base = (int64_t)b * p.v.sb + t * p.v.st + (int64_t)h * p.v.sh;
#pragma unroll
            for (int i = 0; i < 4; ++i) vs[lane + 32 * i] = load_elem(p.v.p, base + lane + 32 * i, p.v.dtype);
        } else if (warp == 3 && lane == 0) {
            gb[0] = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            gb[1] = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
        __syncthreads();

        // kv = (e^g S)^T k: this thread's 16 rows, then the 8 warps' partials
        const float decay = expf(gb[0]);
        float4 part = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < kRecRegRows; ++r) {
            const float kr = ks[r0 + r];
#pragma unroll
            for (int c = 0; c < 4; ++c) S[r][c] *= decay;
            part.x += S[r][0] * kr;
            part.y += S[r][1] * kr;
            part.z += S[r][2] * kr;
            part.w += S[r][3] * kr;
        }
#pragma unroll
        for (int r = 0; r < kRecSmemRows; ++r) {
            const float kr = ks[r0 + kRecRegRows + r];
            float4 x = srows[warp][r][lane];
            x.x *= decay;
            x.y *= decay;
            x.z *= decay;
            x.w *= decay;
            srows[warp][r][lane] = x;
            part.x += x.x * kr;
            part.y += x.y * kr;
            part.z += x.z * kr;
            part.w += x.w * kr;
        }
        *reinterpret_cast<float4*>(&red[warp][c0]) = part;
        __syncthreads();
        float kv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < kRecWarps; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(&red[w][c0]);
            kv[0] += x.x;
            kv[1] += x.y;
            kv[2] += x.z;
            kv[3] += x.w;
        }
        const float4 v4 = *reinterpret_cast<const float4*>(&vs[c0]);
        const float delta[4] = {(v4.x - kv[0]) * gb[1], (v4.y - kv[1]) * gb[1], (v4.z - kv[2]) * gb[1],
                                (v4.w - kv[3]) * gb[1]};
        // S += k delta^T; o = S^T q
        float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < kRecRegRows; ++r) {
            const float kr = ks[r0 + r], qr = qs[r0 + r];
#pragma unroll
            for (int c = 0; c < 4; ++c) S[r][c] += kr * delta[c];
            op.x += S[r][0] * qr;
            op.y += S[r][1] * qr;
            op.z += S[r][2] * qr;
            op.w += S[r][3] * qr;
        }
#pragma unroll
        for (int r = 0; r < kRecSmemRows; ++r) {
            const float kr = ks[r0 + kRecRegRows + r], qr = qs[r0 + kRecRegRows + r];
            float4 x = srows[warp][r][lane];
            x.x += kr * delta[0];
            x.y += kr * delta[1];
            x.z += kr * delta[2];
            x.w += kr * delta[3];
            srows[warp][r][lane] = x;
            op.x += x.x * qr;
            op.y += x.y * qr;
            op.z += x.z * qr;
            op.w += x.w * qr;
        }
        __syncthreads();  // every warp has read red (kv) and vs/gb/qs/ks of this token
        *reinterpret_cast<float4*>(&red[warp][c0]) = op;
        __syncthreads();
        if (warp == 0) {
            float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int w = 0; w < kRecWarps; ++w) {
                const float4 x = *reinterpret_cast<const float4*>(&red[w][c0]);
                o[0] += x.x;
                o[1] += x.y;
                o[2] += x.z;
                o[3] += x.w;
            }
            const int64_t ob = (int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + c0;
#pragma unroll
            for (int c = 0; c < 4; ++c) store_elem(p.out, ob + c, p.out_dtype, o[c]);
        }
        __syncthreads();  // red is rewritten by the next token's kv partials
    }

    if (p.hT) {
#pragma unroll
        for (int r = 0; r < kRecRegRows; ++r)
            *reinterpret_cast<float4*>(p.hT + sbase + (int64_t)(r0 + r) * kDv) =
                make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
#pragma unroll
        for (int r = 0; r < kRecSmemRows; ++r)
            *reinterpret_cast<float4*>(p.hT + sbase + (int64_t)(r0 + kRecRegRows + r) * kDv) = srows[warp][r][lane];
    }
}

}  // namespace

cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream) {
    dim3 grid((unsigned)(p.B * p.H));
    cudaError_t e = phase_event(0, stream);
    if (e != cudaSuccess) return e;
    gdn_recurrent_kernel<<<grid, kRecThreads, 0, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return phase_event(1, stream);
}

}  // namespace gdn
