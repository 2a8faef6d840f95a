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

// Workspace record of one (batch, head, chunk) for the tensor-core path.  The
// scan kernel bulk-copies these straight into shared memory, so the bf16 images
// are stored already in the swizzled UMMA operand layout.
constexpr int64_t kTcM = 0;             // M_c = e^gc_last I - kd^T w, bf16 K-major image [128][128]   32 KiB
constexpr int64_t kTcQ = 32768;         // Q'_c = q e^gc Dk^-1/2 - Aqk w, bf16 K-major image [64][128] 16 KiB
constexpr int64_t kTcB = 49152;         // b_c = kd^T u, fp32 [4 column tiles][8 chunks][128 rows][4]    64 KiB
constexpr int64_t kTcO0 = 114688;       // o0_c = Aqk u, fp32 [4 column tiles][8 chunks][64 rows][4]     32 KiB
constexpr int64_t kTcChunkBytes = 147456;

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
    unsigned int* err;  // device error word (bounded waits that gave up set bits here)
    // Tensor-core scan mode: 0 = outputs + final state; 1 = shard summary (no outputs):
    // the first half of grid.y's column slices write the transition prod_c M_c to hT (state
    // started from I, b ignored), the second half the local final state (state started from 0)
    // to hT2.
    int scan_mode;
    float* hT2;
    // Packed variable-length batch (tensor-core path; B == 1): sequence n is tokens
    // [cu_seqlens[n], cu_seqlens[n+1]) of the T axis and its chunks start at its first
    // token.  Global chunk j belongs to sequence chunk_seq[j], which starts at global
    // chunk chunk_base[n]; records sit at (j * H + h).  Both tables are built on the
    // device (launch_varlen_tables).  cu_seqlens == null: fixed length, records at
    // ((b * H + h) * NC + c).  h0 / hT are then [N,H,Dk,Dv].
    const int* cu_seqlens;
    const int* chunk_base;  // [N + 1]
    const int* chunk_seq;   // [max_chunks]
    const int* seq_order;   // [N]: sequences by chunk count, longest first (the scan starts those first)
    int N;                  // sequences
    int max_chunks;         // ceil(T / 64) + N: bound of sum_n ceil(T_n / 64), the prep's grid
    // CUDA-core scan only: when set, the state at the start of every chunk is written to
    // states + ((b*H + h)*NC + c) * states_stride as [Dk][Dv] fp32 (the backward's forward
    // recompute); out may then be null.
    float* states;
    int64_t states_stride;
    // Tensor-core prep only (fixed length): when set, every chunk's u, w, Kd and Aqk are also
    // written in fp32 to bwd_tiles + ((b*H + h)*NC + c) * kWsChunkFloats at kWsU / kWsW /
    // kWsKd / kWsAqk, the tiles the backward's tensor-core kernels read, chunk-major within each
    // tile (element (row, col) at ((col / 4) * 64 + row) * 4 + col % 4).
    float* bwd_tiles;
};

// ---------------------------------------------------------------- backward
// Per-chunk backward workspace (floats), after the forward's kWsChunkFloats region of every chunk.
constexpr int64_t kBwS = 0;                    // S_c, the state at the chunk's start          [Dk][Dv]
constexpr int64_t kBwDSe = kBwS + kDk * kDv;   // dS_{c+1}, gradient at the chunk's end       [Dk][Dv]
constexpr int64_t kBwDVn = kBwDSe + kDk * kDv; // dv_new = Kd dS_{c+1} + Aqk^T do             [64][Dv]
constexpr int64_t kBwVn = kBwDVn + kChunk * kDv;   // v_new = u - w S_c                       [64][Dv]
constexpr int64_t kBwDQg = kBwVn + kChunk * kDv;   // d(q e^gc Dk^-1/2) = do S_c^T            [64][Dk]
constexpr int64_t kBwDW = kBwDQg + kChunk * kDk;   // dw = -dv_new S_c^T                      [64][Dk]
constexpr int64_t kBwDKd = kBwDW + kChunk * kDk;   // d(k e^(gc_last-gc)) = v_new dS_{c+1}^T  [64][Dk]
constexpr int64_t kBwDKp = kBwDKd + kChunk * kDk;  // dk^ through beta e^gc k^                [64][Dk]
constexpr int64_t kBwDL = kBwDKp + kChunk * kDk;   // dL (strictly lower)                     [64][64]
constexpr int64_t kBwDA = kBwDL + kChunk * kChunk; // dAqk (lower incl. diagonal)             [64][64]
constexpr int64_t kBwSmall = kBwDA + kChunk * kChunk;  // [0] <S_c, dS_{c+1}>, [64..] dbeta part, [128..] dgc part
constexpr int64_t kBwChunkFloats = kBwSmall + 192;
// With tensor-core records (bf16 mode) kBwDQg, kBwDKd and kBwDKp are chunk-major like the prep's backward
// tiles (element (row, col) at ((col / 4) * 64 + row) * 4 + col % 4); every other region is row-major.

struct Out4 {
    void* p;
    int64_t sb, st, sh;
    int dtype;
};
struct Out3 {
    void* p;
    int64_t sb, st, sh;
    int dtype;
};

struct BwdParams {
    View4 q, k, v, dout;
    View3 g, beta;
    const float* h0;    // [B,H,Dk,Dv] or null
    const float* dhT;   // gradient of the final state, or null
    float* dh0;         // gradient of the initial state, or null
    Out4 dq, dk, dv;
    Out3 dg, dbeta;
    float* fws;         // forward workspace: kWsChunkFloats per chunk (CUDA-core prep layout)
    float* bws;         // backward workspace: kBwChunkFloats per chunk
    // Tensor-core records of the forward (kTcChunkBytes per chunk; bf16 q/k/v/d_out): when set, the
    // forward recompute and the reverse scan run on the tensor cores and the chunk kernels form
    // dv_new themselves.  Null: the CUDA-core scans.
    void* tc_records;
    unsigned int* err;
    int B, H, NC;
    int64_t T;
    int l2norm;
};

// Backward of the chunked rule (CUDA-core, fp32): forward recompute (prep + scan recording the
// chunk-start states), reverse state scan, then three per-chunk gradient kernels.
cudaError_t launch_chunk_bwd(const ChunkParams& fwd, const BwdParams& p, cudaStream_t stream);
// Reverse scan on the tensor cores over the forward's records (p.tc_records): dS_c = M_c^T dS_{c+1} +
// Q'_c^T do_c; records dS_{c+1} per chunk and writes dh0.
cudaError_t launch_bwd_scan_tc(const BwdParams& p, cudaStream_t stream);
// The backward's products with S_c and dS_{c+1} on the tensor cores (p.tc_records mode): dv_new, v_new,
// dQg, dw, dKd and <S_c, dS_{c+1}> into every chunk's backward record.
cudaError_t launch_bwd_states_tc(const BwdParams& p, cudaStream_t stream);
// The chain rule of every chunk on the tensor cores (p.tc_records mode): dq, dk, dg, dbeta from the records of
// gdn_bwd_wy and gdn_bwd_states_tc.
cudaError_t launch_bwd_grads_tc(const BwdParams& p, cudaStream_t stream);
// The WY terms of every chunk with their products on the tensor cores (p.tc_records mode): dv, the dKp,
// dL and dAqk records and the dbeta / dgc parts.
cudaError_t launch_bwd_wy_tc(const BwdParams& p, cudaStream_t stream);

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

// Error bits a kernel ORs into the device error word.
enum : unsigned int { kErrTimeoutPrep = 1u, kErrTimeoutScan = 2u, kErrBadSeqlens = 8u, kErrWaitSelftest = 16u };

cudaError_t launch_chunk_simt(const ChunkParams& p, cudaStream_t stream);
cudaError_t launch_chunk_tc(const ChunkParams& p, cudaStream_t stream);
// The two halves of the tensor-core path: prep fills the workspace records; scan reads them
// (in p.scan_mode) -- the sequence-parallel entry points run them separately.
cudaError_t launch_chunk_tc_prep(const ChunkParams& p, cudaStream_t stream);
cudaError_t launch_chunk_tc_scan(const ChunkParams& p, cudaStream_t stream);
// Varlen: builds chunk_base / chunk_seq from cu_seqlens (one CTA); bad offsets set kErrBadSeqlens and
// leave zero chunks, so nothing runs.
cudaError_t launch_varlen_tables(const ChunkParams& p, cudaStream_t stream);
cudaError_t launch_recurrent(const RecurrentParams& p, cudaStream_t stream);
// One kernel whose bounded barrier wait runs out after timeout_ns and reports kErrWaitSelftest.
cudaError_t launch_selftest_wait(unsigned int* err, uint64_t timeout_ns, cudaStream_t stream);

}  // namespace gdn
