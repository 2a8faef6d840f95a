// Shared device helpers for the GatedDeltaNet kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdn_b200.h"

namespace gdn {

constexpr int kChunk = 64;   // tokens per chunk (the reference's chunk_size)
constexpr int kDk = 128;     // key head dim
constexpr int kDv = 128;     // value head dim

// Strided view handed to kernels: element pointer + strides in elements.
struct View4 {
    const void* p;
    int64_t sb, st, sh;  // batch, time, head strides; the head dim is contiguous
    int dtype;
};
struct View3 {
    const void* p;
    int64_t sb, st, sh;
    int dtype;
};

// The per-device error word the kernels report into.  Kernels receive a pointer
// to `bits`; `host_mirror` is the device address of a page-locked host word the
// host registered (gdn_set_error_mirror) or null.  A kernel that gives up sets
// its bit in both, so the host can see the failure without synchronising.
struct DeviceErrorWord {
    unsigned int bits;
    unsigned int reserved;
    unsigned int* host_mirror;
};

__device__ __forceinline__ void report_device_error(unsigned int* err, unsigned int bit) {
    if (!err) return;
    atomicOr(err, bit);
    unsigned int* m = reinterpret_cast<const DeviceErrorWord*>(err)->host_mirror;
    if (m) {
        // plain stores over the bus (no system-scope atomics needed): concurrent reporters may
        // overwrite each other's bit, but the word never returns to zero
        volatile unsigned int* vm = m;
        *vm = *vm | bit;
        __threadfence_system();
    }
}

__device__ __forceinline__ float load_elem(const void* base, int64_t idx, int dtype) {
    if (dtype == GDN_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
    if (dtype == GDN_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
    return reinterpret_cast<const float*>(base)[idx];
}

__device__ __forceinline__ void store_elem(void* base, int64_t idx, int dtype, float x) {
    if (dtype == GDN_BF16) reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(x);
    else if (dtype == GDN_F16) reinterpret_cast<__half*>(base)[idx] = __float2half_rn(x);
    else reinterpret_cast<float*>(base)[idx] = x;
}

// Round an fp32 value to `dtype` and back (identity for fp32): reproduces the
// roundings a torch op in that dtype would do.
__device__ __forceinline__ float round_to(float x, int dtype) {
    if (dtype == GDN_BF16) return __bfloat162float(__float2bfloat16_rn(x));
    if (dtype == GDN_F16) return __half2float(__float2half_rn(x));
    return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Inverse L2 norm of a 128-vector spread 4 elements per lane over one warp,
// evaluated the way `x * rsqrt((x*x).sum(-1) + 1e-6)` runs in `dtype`
// (qwen3_5_transformers.py:104-107): for 16-bit inputs every elementwise
// result is rounded to that dtype and the sum accumulates in fp32.
__device__ __forceinline__ float l2norm_inv(const float (&x)[4], int dtype) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) s += round_to(x[i] * x[i], dtype);
    s = warp_sum(s);
    if (dtype == GDN_F32) return 1.0f / sqrtf(s + 1e-6f);
    s = round_to(s, dtype);
    s = round_to(s + 1e-6f, dtype);
    return round_to(1.0f / sqrtf(s), dtype);
}

// 16-byte asynchronous global -> shared copy and its group commit / wait (cp.async; CUDA-core kernels).
__device__ __forceinline__ void cp_async16_rec(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit_rec() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_rec() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

}  // namespace gdn
