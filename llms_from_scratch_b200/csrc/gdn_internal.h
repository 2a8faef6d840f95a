// Internal launch interface shared by the C ABI and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn_common.cuh"

namespace gdn {

// fp32 workspace layout of one (batch, head, chunk) for the CUDA-core path.
constexpr int64_t kWsU = 0;                          // u = T beta v          [64][128]
constexpr int64_t kWsW = kWsU + kChunk * kDv;        // w = T k_beta e^gc     [64][128]
constexpr int64_t kWsQg = kWsW + kChunk * kDk;       // q Dk^-1/2 e^gc        [64][128]
constexpr int64_t kWsKd = kWsQg + kChunk * kDk;      // k e^(gc_last - gc)    [64][128]
constexpr int64_t kWsAqk = kWsKd + kChunk * kDk;     // (q k^T * decay) causal [64][64]
constexpr int64_t kWsGamma = kWsAqk + kChunk * kChunk;  // e^gc_last
constexpr int64_t kWsChunkFloats = kWsGamma + 64;       // keeps every chunk 256-byte aligned

struct ChunkParams {
    View4 q, k, v;
    View3 g, beta;
    void* out;
    int64_t out_sb, out_st, out_sh;
    int out_dtype;
    const float* h0;  // [B,H,Dk,Dv] or null
    float* hT;        // [B,H,Dk,Dv] or null
    float* ws;
    int B, H, NC;
    int64_t T;
    int l2norm;
};

struct RecurrentParams {
    View4 q, k, v;
    View3 g, beta;
    void* out;
    int64_t out_sb, out_st, out_sh;
    int out_dtype;
    const float* h0;
    float* hT;
    int B, H;
    int64_t T;
    int l2norm;
};

// Records `fmt` as the message gdn_last_error() returns on this host thread; returns `code`.
int set_last_error(int code, const char* fmt, ...);

// Launch bookkeeping shared by all launchers: counts kernels and records the
// phase events requested through gdn_set_phase_events on this host thread.
void note_launch();
cudaError_t phase_event(int index, cudaStream_t stream);

cudaError_t launch_chunk_simt(const ChunkParams& p, cudaStream_t stream);
cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream);

}  // namespace gdn
