// Token-recurrent gated delta rule (the decode step), HBM-bound.
//
// Follows torch_recurrent_gated_delta_rule (qwen3_5_transformers.py:190-229):
//   S *= e^g;  kv = S^T k;  delta = beta (v - kv);  S += k delta^T;  o = S^T q
// State columns never interact, so one CTA owns a 128 x 16 column slice of one
// head's fp32 state and keeps it in registers across all T tokens: the state is
// read from HBM once and written once per call (the reference streams it five
// times per token).  Each thread holds 4 rows x 4 columns (a float4 per row);
// a warp covers 8 rows x 16 columns, so every load/store instruction moves
// whole 32-byte sectors.  Column sums reduce with warp shuffles, then across
// the 4 warps through shared memory.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kRecThreads = 128;
constexpr int kRecDv = 16;

__global__ void __launch_bounds__(kRecThreads) gdn_recurrent_kernel(RecurrentParams p) {
    __shared__ __align__(16) float qs[kDk];
    __shared__ __align__(16) float ks[kDk];
    __shared__ float vs[kRecDv];
    __shared__ float gb[2];
    __shared__ float red_kv[4][kRecDv];
    __shared__ float red_o[4][kRecDv];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh % p.H;
    const int dv0 = blockIdx.y * kRecDv;
    const int kg = tid >> 2;            // rows 4kg .. 4kg+3
    const int cq = (tid & 3) * 4;       // columns dv0+cq .. +3
    const float scale = rsqrtf((float)kDk);

    float S[4][4];
    const int64_t sbase = (int64_t)bh * kDk * kDv + dv0 + cq;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.h0) v = *reinterpret_cast<const float4*>(p.h0 + sbase + (int64_t)(4 * kg + r) * kDv);
        S[r][0] = v.x; S[r][1] = v.y; S[r][2] = v.z; S[r][3] = v.w;
    }

    for (int64_t t = 0; t < p.T; ++t) {
        if (warp < 2) {
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
            if (lane < kRecDv)
                vs[lane] = load_elem(p.v.p, (int64_t)b * p.v.sb + t * p.v.st + (int64_t)h * p.v.sh + dv0 + lane, p.v.dtype);
        } else if (lane == 0) {
            gb[0] = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            gb[1] = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
        __syncthreads();

        const float decay = expf(gb[0]);
        const float4 k4 = *reinterpret_cast<const float4*>(&ks[4 * kg]);
        const float kr[4] = {k4.x, k4.y, k4.z, k4.w};
        float kv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float a = 0.f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                S[r][c] *= decay;
                a += S[r][c] * kr[r];
            }
            kv[c] = a;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) kv[c] += __shfl_xor_sync(0xffffffffu, kv[c], o);
        }
        if (lane < 4) {
#pragma unroll
            for (int c = 0; c < 4; ++c) red_kv[warp][cq + c] = kv[c];
        }
        __syncthreads();

        const float4 q4 = *reinterpret_cast<const float4*>(&qs[4 * kg]);
        const float qr[4] = {q4.x, q4.y, q4.z, q4.w};
        float ov[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float kvs = red_kv[0][cq + c] + red_kv[1][cq + c] + red_kv[2][cq + c] + red_kv[3][cq + c];
            const float delta = (vs[cq + c] - kvs) * gb[1];
            float a = 0.f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                S[r][c] += kr[r] * delta;
                a += S[r][c] * qr[r];
            }
            ov[c] = a;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) ov[c] += __shfl_xor_sync(0xffffffffu, ov[c], o);
        }
        if (lane < 4) {
#pragma unroll
            for (int c = 0; c < 4; ++c) red_o[warp][cq + c] = ov[c];
        }
        __syncthreads();
        if (tid < kRecDv) {
            const float o = red_o[0][tid] + red_o[1][tid] + red_o[2][tid] + red_o[3][tid];
            store_elem(p.out, (int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + dv0 + tid, p.out_dtype, o);
        }
    }

    if (p.hT) {
#pragma unroll
        for (int r = 0; r < 4; ++r)
            *reinterpret_cast<float4*>(p.hT + sbase + (int64_t)(4 * kg + r) * kDv) =
                make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
    }
}

}  // namespace

cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream) {
    dim3 grid((unsigned)(p.B * p.H), kDv / kRecDv);
    cudaError_t e = phase_event(0, stream);
    if (e != cudaSuccess) return e;
    gdn_recurrent_kernel<<<grid, kRecThreads, 0, stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return phase_event(1, stream);
}

}  // namespace gdn
