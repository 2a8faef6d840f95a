// Chunked gated delta rule, CUDA-core (FFMA) path in fp32 throughout.
//
// Two kernels, one launch each:
//   gdn_prep_simt   one CTA per (batch, head, 64-token chunk), all in parallel:
//                   l2norm, per-chunk cumsum of g, the strictly-lower
//                   beta*decay*K K^T, its unit-triangular inverse applied to
//                   [beta v | beta k e^gc] (the WY form: u and w), the causal
//                   intra-chunk attention q k^T * decay, and the decayed q / k
//                   the state recurrence consumes.  Results go to a workspace.
//   gdn_scan_simt   one CTA per (batch, head, 16-column slice of Dv) walking the
//                   chunks in order with its 128x16 slice of the fp32 state in
//                   shared memory (state columns never interact).
//
// This path serves fp32 inputs (fp32-accurate to the reference) and any dtype
// mix the tensor-core path does not take.  The maths follows
// torch_chunk_gated_delta_rule (qwen3_5_transformers.py:110-187).
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

constexpr int kThreads = 256;
constexpr int kRowPad = 132;   // fp32 row stride of 128-wide smem tiles (float4 aligned, conflict-free)
constexpr int kScanDv = 16;    // state columns per scan CTA

struct PrepSmem {
    float K[kChunk][kRowPad];   // l2-normalised k (fp32)
    float Q[kChunk][kRowPad];   // l2-normalised q * Dk^-1/2
    float L[kChunk][kChunk];    // -(beta_i k_i.k_j) e^(gc_i-gc_j), strictly lower
    float gc[kChunk];
    float beta[kChunk];
    float egc[kChunk];          // e^(gc_i)
    float ekd[kChunk];          // e^(gc_last - gc_i)
};

// Load one 128-long row (4 elements per lane) of a [B,T,H,D] view as fp32.
__device__ __forceinline__ void load_row4(const View4& v, int b, int64_t t, int h, int lane, float (&x)[4]) {
    const int64_t base = (int64_t)b * v.sb + t * v.st + (int64_t)h * v.sh;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = load_elem(v.p, base + lane + 32 * i, v.dtype);
}

__global__ void __launch_bounds__(kThreads) gdn_prep_simt(ChunkParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrepSmem& s = *reinterpret_cast<PrepSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t chunk = blockIdx.x;               // (b*H + h)*NC + c
    const int c = (int)(chunk % p.NC);
    const int bh = (int)(chunk / p.NC);
    const int b = bh / p.H, h = bh % p.H;
    const int64_t t0 = (int64_t)c * kChunk;
    const float scale = rsqrtf((float)kDk);

    // 1. q, k rows: l2norm in the input dtype (qwen3_5_transformers.py:122-124), then
    //    fp32, then q * Dk^-1/2 (:138-139).  Rows past T are the zero padding (:131-137).
    for (int i = warp; i < kChunk; i += kThreads / 32) {
        const int64_t t = t0 + i;
        float q[4], k[4];
        if (t < p.T) {
            load_row4(p.q, b, t, h, lane, q);
            load_row4(p.k, b, t, h, lane, k);
            if (p.l2norm) {
                const float iq = l2norm_inv(q, p.q.dtype), ik = l2norm_inv(k, p.k.dtype);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    q[e] = round_to(q[e] * iq, p.q.dtype);
                    k[e] = round_to(k[e] * ik, p.k.dtype);
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) q[e] = k[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            s.Q[i][lane + 32 * e] = q[e] * scale;
            s.K[i][lane + 32 * e] = k[e];
        }
    }
    if (tid < kChunk) {
        const int64_t t = t0 + tid;
        float gv = 0.f, bv = 0.f;
        if (t < p.T) {
            gv = load_elem(p.g.p, (int64_t)b * p.g.sb + t * p.g.st + (int64_t)h * p.g.sh, p.g.dtype);
            bv = load_elem(p.beta.p, (int64_t)b * p.beta.sb + t * p.beta.st + (int64_t)h * p.beta.sh, p.beta.dtype);
        }
        s.gc[tid] = gv;
        s.beta[tid] = bv;
    }
    __syncthreads();
    // 2. per-chunk cumulative sum of g, in order (:151).
    if (tid == 0) {
        float acc = 0.f;
        for (int i = 0; i < kChunk; ++i) { acc += s.gc[i]; s.gc[i] = acc; }
    }
    __syncthreads();
    if (tid < kChunk) {
        s.egc[tid] = expf(s.gc[tid]);
        s.ekd[tid] = expf(s.gc[kChunk - 1] - s.gc[tid]);
    }

    // 3. L = -(k_beta k^T * decay) strictly lower (:152-153) and the causal
    //    intra-chunk attention (q k^T * decay) incl. the diagonal (:172).
    //    Thread (ty, tx) owns rows ty+16r and columns tx+16c.
    float* ws = p.ws + chunk * kWsChunkFloats;
    {
        const int ty = tid >> 4, tx = tid & 15;
        float kk[4][4], qk[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) kk[r][cc] = qk[r][cc] = 0.f;
        for (int d = 0; d < kDk; d += 4) {
            float4 ki[4], qi[4], kj[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                ki[r] = *reinterpret_cast<const float4*>(&s.K[ty + 16 * r][d]);
                qi[r] = *reinterpret_cast<const float4*>(&s.Q[ty + 16 * r][d]);
                kj[r] = *reinterpret_cast<const float4*>(&s.K[tx + 16 * r][d]);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    kk[r][cc] += ki[r].x * kj[cc].x + ki[r].y * kj[cc].y + ki[r].z * kj[cc].z + ki[r].w * kj[cc].w;
                    qk[r][cc] += qi[r].x * kj[cc].x + qi[r].y * kj[cc].y + qi[r].z * kj[cc].z + qi[r].w * kj[cc].w;
                }
        }
        __syncthreads();  // gc must be final before the decay below (written above by tid<64)
        float* aqk = ws + kWsAqk;
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const int i = ty + 16 * r, j = tx + 16 * cc;
                const float dec = (i >= j) ? expf(s.gc[i] - s.gc[j]) : 0.f;
                s.L[i][j] = (i > j) ? -(s.beta[i] * kk[r][cc]) * dec : 0.f;
                aqk[i * kChunk + j] = (i >= j) ? qk[r][cc] * dec : 0.f;
            }
    }
    __syncthreads();

    // 4. WY form by forward substitution (the loop at :154-158 applied to the
    //    right-hand sides): thread c solves (I - L) x = rhs for column c of
    //    [beta v | beta k e^gc], giving u = T beta v (:159) and w = T (k_beta e^gc) (:160).
    {
        const int col = tid;  // 0..127: v column, 128..255: k column
        float x[kChunk];
        if (col < kDv) {
            const int64_t base = (int64_t)b * p.v.sb + (int64_t)h * p.v.sh + col;
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                const int64_t t = t0 + i;
                const float vv = (t < p.T) ? load_elem(p.v.p, base + t * p.v.st, p.v.dtype) : 0.f;
                x[i] = vv * s.beta[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < kChunk; ++i) x[i] = (s.K[i][col - kDv] * s.beta[i]) * s.egc[i];
        }
#pragma unroll
        for (int i = 1; i < kChunk; ++i) {
            float acc = x[i];
#pragma unroll
            for (int m4 = 0; m4 < (i + 3) / 4; ++m4) {
                // L[i][m] = 0 for m >= i, so the tail of the last group adds 0 * rhs.
                const float4 l = *reinterpret_cast<const float4*>(&s.L[i][4 * m4]);
                acc += l.x * x[4 * m4] + l.y * x[4 * m4 + 1] + l.z * x[4 * m4 + 2] + l.w * x[4 * m4 + 3];
            }
            x[i] = acc;
        }
        float* dst = ws + (col < kDv ? kWsU + col : kWsW + (col - kDv));
#pragma unroll
        for (int i = 0; i < kChunk; ++i) dst[i * kDk] = x[i];
    }

    // 5. decayed q / k for the recurrence (:175, :179) and e^(gc_last) (:178).
    for (int idx = tid; idx < kChunk * kDk; idx += kThreads) {
        const int i = idx >> 7, d = idx & 127;
        ws[kWsQg + idx] = s.Q[i][d] * s.egc[i];
        ws[kWsKd + idx] = s.K[i][d] * s.ekd[i];
    }
    if (tid == 0) ws[kWsGamma] = expf(s.gc[kChunk - 1]);
}

struct ScanSmem {
    float W[kChunk][kRowPad];
    float Qg[kChunk][kRowPad];
    float Kd[kChunk][kDk];
    float A[kChunk][kChunk + 4];
    float U[kChunk][kScanDv];
    float Vn[kChunk][kScanDv];
    float S[kDk][kScanDv];
};

// State recurrence over chunks (the loop at qwen3_5_transformers.py:170-180):
//   v_new = u - w S;  o = (q e^gc) S + Aqk v_new;  S = e^gc_last S + (k e^(gc_last-gc))^T v_new
__global__ void __launch_bounds__(kThreads) gdn_scan_simt(ChunkParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ScanSmem& s = *reinterpret_cast<ScanSmem*>(smem_raw);
    const int tid = threadIdx.x;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh % p.H;
    const int dv0 = blockIdx.y * kScanDv;

    const int64_t sbase = (int64_t)bh * kDk * kDv;
    for (int idx = tid; idx < kDk * kScanDv; idx += kThreads) {
        const int d = idx / kScanDv, cc = idx % kScanDv;
        s.S[d][cc] = p.h0 ? p.h0[sbase + (int64_t)d * kDv + dv0 + cc] : 0.f;
    }

    const int r = tid >> 2, cq = (tid & 3) * 4;         // v_new / o: row r, 4 columns
    const int sd = tid >> 1, sc = (tid & 1) * 8;        // state update: row sd, 8 columns
    for (int c = 0; c < p.NC; ++c) {
        const float* ws = p.ws + ((int64_t)bh * p.NC + c) * kWsChunkFloats;
        __syncthreads();  // previous chunk's readers of the tiles are done
        // the chunk's tiles, every 16-byte piece in flight at once (asynchronous copies, no register round trip)
        for (int idx = tid; idx < kChunk * kDk / 4; idx += kThreads) {
            const int i = idx >> 5, d4 = (idx & 31) * 4;
            cp_async16_rec(&s.W[i][d4], ws + kWsW + i * kDk + d4);
            cp_async16_rec(&s.Qg[i][d4], ws + kWsQg + i * kDk + d4);
            cp_async16_rec(&s.Kd[i][d4], ws + kWsKd + i * kDk + d4);
        }
        for (int idx = tid; idx < kChunk * kChunk / 4; idx += kThreads) {
            const int i = idx >> 4, j4 = (idx & 15) * 4;
            cp_async16_rec(&s.A[i][j4], ws + kWsAqk + i * kChunk + j4);
        }
        {
            const int i = tid >> 2, q4 = (tid & 3) * 4;
            cp_async16_rec(&s.U[i][q4], ws + kWsU + i * kDv + dv0 + q4);
        }
        cp_async_commit_rec();
        const float gamma = ws[kWsGamma];
        cp_async_wait_rec();
        if (p.states) {  // S at the start of chunk c (S is stable here: the last update precedes the barrier above)
            float* dst = p.states + ((int64_t)bh * p.NC + c) * p.states_stride;
            for (int idx = tid; idx < kDk * kScanDv / 4; idx += kThreads) {
                const int d = idx / (kScanDv / 4), c4 = (idx % (kScanDv / 4)) * 4;
                *reinterpret_cast<float4*>(dst + (int64_t)d * kDv + dv0 + c4) =
                    *reinterpret_cast<const float4*>(&s.S[d][c4]);
            }
        }
        __syncthreads();

        // v_new = u - w S  (:173-174)
        float vn[4];
        {
            const float4 u4 = *reinterpret_cast<const float4*>(&s.U[r][cq]);
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            for (int d = 0; d < kDk; d += 4) {
                const float4 w4 = *reinterpret_cast<const float4*>(&s.W[r][d]);
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 s4 = *reinterpret_cast<const float4*>(&s.S[d + e][cq]);
                    a0 += wv[e] * s4.x; a1 += wv[e] * s4.y; a2 += wv[e] * s4.z; a3 += wv[e] * s4.w;
                }
            }
            vn[0] = u4.x - a0; vn[1] = u4.y - a1; vn[2] = u4.z - a2; vn[3] = u4.w - a3;
            *reinterpret_cast<float4*>(&s.Vn[r][cq]) = make_float4(vn[0], vn[1], vn[2], vn[3]);
        }
        __syncthreads();

        // o = (q e^gc) S + Aqk v_new  (:175-176)
        {
            float a[4] = {0.f, 0.f, 0.f, 0.f};
            for (int d = 0; d < kDk; d += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(&s.Qg[r][d]);
                const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 s4 = *reinterpret_cast<const float4*>(&s.S[d + e][cq]);
                    a[0] += qv[e] * s4.x; a[1] += qv[e] * s4.y; a[2] += qv[e] * s4.z; a[3] += qv[e] * s4.w;
                }
            }
            float o[4] = {0.f, 0.f, 0.f, 0.f};
            for (int j = 0; j <= r; ++j) {
                const float av = s.A[r][j];
                const float4 v4 = *reinterpret_cast<const float4*>(&s.Vn[j][cq]);
                o[0] += av * v4.x; o[1] += av * v4.y; o[2] += av * v4.z; o[3] += av * v4.w;
            }
            const int64_t t = (int64_t)c * kChunk + r;
            if (p.out && t < p.T) {
                const int64_t ob = (int64_t)b * p.out_sb + t * p.out_st + (int64_t)h * p.out_sh + dv0 + cq;
#pragma unroll
                for (int e = 0; e < 4; ++e) store_elem(p.out, ob + e, p.out_dtype, a[e] + o[e]);
            }
        }
        __syncthreads();

        // S = e^gc_last S + (k e^(gc_last-gc))^T v_new  (:177-180)
        {
            float a[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = 0.f;
            for (int j = 0; j < kChunk; ++j) {
                const float kv = s.Kd[j][sd];
                const float4 v0 = *reinterpret_cast<const float4*>(&s.Vn[j][sc]);
                const float4 v1 = *reinterpret_cast<const float4*>(&s.Vn[j][sc + 4]);
                a[0] += kv * v0.x; a[1] += kv * v0.y; a[2] += kv * v0.z; a[3] += kv * v0.w;
                a[4] += kv * v1.x; a[5] += kv * v1.y; a[6] += kv * v1.z; a[7] += kv * v1.w;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) s.S[sd][sc + e] = s.S[sd][sc + e] * gamma + a[e];
        }
    }
    __syncthreads();
    if (p.hT) {
        for (int idx = tid; idx < kDk * kScanDv; idx += kThreads) {
            const int d = idx / kScanDv, cc = idx % kScanDv;
            p.hT[sbase + (int64_t)d * kDv + dv0 + cc] = s.S[d][cc];
        }
    }
}

}  // namespace

cudaError_t launch_chunk_simt(const ChunkParams& p, cudaStream_t stream) {
    static_assert(sizeof(PrepSmem) <= 227 * 1024, "prep smem");
    static_assert(sizeof(ScanSmem) <= 227 * 1024, "scan smem");
    cudaError_t e = cudaFuncSetAttribute(gdn_prep_simt, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PrepSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(gdn_scan_simt, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(ScanSmem));
    if (e != cudaSuccess) return e;
    const int64_t nchunks = (int64_t)p.B * p.H * p.NC;
    if ((e = phase_event(0, stream)) != cudaSuccess) return e;
    gdn_prep_simt<<<(unsigned)nchunks, kThreads, sizeof(PrepSmem), stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    if ((e = phase_event(1, stream)) != cudaSuccess) return e;
    dim3 grid((unsigned)(p.B * p.H), kDv / kScanDv);
    gdn_scan_simt<<<grid, kThreads, sizeof(ScanSmem), stream>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return phase_event(2, stream);
}

}  // namespace gdn
