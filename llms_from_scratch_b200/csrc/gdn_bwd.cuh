// Device helpers shared by the backward's kernels (CUDA-core and tensor-core files).
#pragma once

#include <cuda_bf16.h>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace bwd {

// Row t of q or k (4 elements a lane, zero past T); loads only, so a warp can have several rows in flight.
__device__ __forceinline__ void qk_load(const View4& v, int b, int64_t t, int64_t T, int h, int lane, float (&x)[4]) {
    const int64_t base = (int64_t)b * v.sb + (t < T ? t : 0) * v.st + (int64_t)h * v.sh;
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = t < T ? load_elem(v.p, base + lane + 32 * e, v.dtype) : 0.f;
}

// A loaded row as the forward uses it (l2-normalised in the input dtype as gdn_prep_simt does), and
// r = (sum x^2 + 1e-6)^-1/2 of the raw row in fp32 for the l2norm's derivative.  Warp-uniform in t.
__device__ __forceinline__ void qk_norm(const View4& v, int64_t t, int64_t T, int l2norm, float (&x)[4], float& r) {
    r = 1.f;
    if (t >= T) return;
    if (l2norm) {
        float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        r = rsqrtf(ss + 1e-6f);
        const float inv = l2norm_inv(x, v.dtype);
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = round_to(x[e] * inv, v.dtype);
    }
}

// Four consecutive bf16 of row t (columns 4 lane ..), zero past T; bf16 rows 8-byte aligned.
__device__ __forceinline__ void row4_bf16(const View4& v, int b, int64_t t, int64_t T, int h, int lane, float (&x)[4]) {
    if (t < T) {
        const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(v.p) + (int64_t)b * v.sb +
                                                        t * v.st + (int64_t)h * v.sh + 4 * lane);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        x[0] = lo.x;
        x[1] = lo.y;
        x[2] = hi.x;
        x[3] = hi.y;
    } else {
        x[0] = x[1] = x[2] = x[3] = 0.f;
    }
}

// g, beta of the chunk -> gc (inclusive cumsum), beta, e^gc, e^(gc_last - gc); rows past T are zero.
// warp_scan (CTA-uniform): the cumsum by one warp, two values a lane, as the tensor-core prep forms it (the
// bf16 mode's forward); otherwise in order by one thread, as the CUDA-core prep forms it.
__device__ __forceinline__ void chunk_gates(const BwdParams& p, int b, int h, int64_t t0, float* gc, float* beta,
                                            float* egc, float* ekd, bool warp_scan = false) {
    const int tid = threadIdx.x;
    if (tid < kChunk) {
        const int64_t t = t0 + tid;
        gc[tid] = t < p.T ? load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype) : 0.f;
        beta[tid] = t < p.T ? load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh,
                                        p.beta.dtype)
                            : 0.f;
    }
    __syncthreads();
    if (warp_scan) {
        if (tid >= 32 && tid < 64) {
            const int lane = tid - 32;
            const float g0 = gc[2 * lane], g1 = gc[2 * lane + 1];
            float x = g0 + g1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            const float gc0 = x - g1, gcl = __shfl_sync(0xffffffffu, x, 31);
            gc[2 * lane] = gc0;
            gc[2 * lane + 1] = x;
            egc[2 * lane] = expf(gc0);
            egc[2 * lane + 1] = expf(x);
            ekd[2 * lane] = expf(gcl - gc0);
            ekd[2 * lane + 1] = expf(gcl - x);
        }
        __syncthreads();
        return;
    }
    if (tid == 0) {  // in order, as the forward's prep sums it
        float acc = 0.f;
        for (int i = 0; i < kChunk; ++i) {
            acc += gc[i];
            gc[i] = acc;
        }
    }
    __syncthreads();
    if (tid < kChunk) {
        egc[tid] = expf(gc[tid]);
        ekd[tid] = expf(gc[kChunk - 1] - gc[tid]);
    }
    __syncthreads();
}

}  // namespace bwd
}  // namespace gdn
