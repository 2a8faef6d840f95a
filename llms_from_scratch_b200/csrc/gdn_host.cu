// Chunked forward over host buffers: the sequence is cut into time slices and
// each slice's host->device copies, its chunk kernels and its device->host
// copies run on three streams, so slice s+1's inputs cross PCIe while slice s
// computes and slice s-1's outputs come back.  The input copies bound the
// whole call (52 MB at ~51 GB/s for B=1, T=4096, H=16 bf16), so slices are
// as large as keeps the link at full rate while the compute stays hidden.
//
// The reference hands device tensors to its op (qwen3_5_cutedsl_kernels.py:462-567)
// and a caller with host data copies them in and out around it, one after the
// other.  Here the copies are the op's own, overlapped with the compute; each
// slice runs the device entry point (gdn_chunk_gated_delta_rule) on staged
// copies with the state carried in place between slices.  Slices start on
// 64-token chunk boundaries and the state passes between them in fp32, the
// precision the scan keeps it in, so the result equals one device call on the
// whole sequence.
#include <cstring>
#include <mutex>

#include "gdn_internal.h"

namespace {

constexpr int kSlots = 2;  // staging buffers per direction

size_t esize(int dtype) { return dtype == GDN_F32 ? 4 : 2; }
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Per-device copy streams and events, created on first use and kept.
struct Pipe {
    bool ready = false;
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, end = nullptr;
    cudaEvent_t in_done[kSlots] = {}, comp_done[kSlots] = {}, out_done[kSlots] = {};
};
Pipe g_pipes[64];
std::mutex g_pipe_mutex[64];

cudaError_t pipe_init(Pipe& p) {
    if (p.ready) return cudaSuccess;
    cudaError_t e;
    if ((e = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking)) != cudaSuccess) return e;
    if ((e = cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking)) != cudaSuccess) return e;
    cudaEvent_t* all[2 + 3 * kSlots] = {&p.start, &p.end};
    for (int s = 0; s < kSlots; ++s) {
        all[2 + 3 * s] = &p.in_done[s];
        all[3 + 3 * s] = &p.comp_done[s];
        all[4 + 3 * s] = &p.out_done[s];
    }
    for (cudaEvent_t* ev : all)
        if ((e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming)) != cudaSuccess) return e;
    p.ready = true;
    return cudaSuccess;
}

// Largest slice, in tokens: the caller's, else about 12 MiB of q/k/v per slice
// (1024 tokens at B=1, H=16, bf16), where a host->device copy runs at the
// link's full rate; never more than the sequence rounded up to a chunk.
int64_t max_slice(int64_t B, int64_t T, int64_t H, size_t qkv_es, int64_t slice_tokens) {
    int64_t s = slice_tokens;
    if (s <= 0) {
        const int64_t per_token = B * H * (2 * gdn::kDk + gdn::kDv) * (int64_t)qkv_es;
        s = (int64_t(12) << 20) / (per_token > 0 ? per_token : 1) / gdn::kChunk * gdn::kChunk;
        if (s < gdn::kChunk) s = gdn::kChunk;
        if (s > 4096) s = 4096;
    }
    const int64_t whole = (T + gdn::kChunk - 1) / gdn::kChunk * gdn::kChunk;
    return s < whole ? s : whole;
}

// Slice lengths in chunks, in time order: full-size slices, the first taking
// the remainder.  Each copy has a fixed cost of ~4.5 us on the link and the
// last slice's compute and output copy are left over after the final input
// copy; measured at B=1, T=4096, H=16, uniform 1024-token slices (1.24 ms per
// call) beat halving the last slices down to 128 tokens (1.30 ms) and one
// unsliced pass (1.53 ms).
int schedule(int64_t T, int64_t Ts, int64_t* chunks, int cap) {
    const int64_t nc = (T + gdn::kChunk - 1) / gdn::kChunk;
    const int64_t full = Ts / gdn::kChunk;
    const int64_t n = (nc + full - 1) / full;
    if (n > cap) return -1;
    for (int64_t i = 0; i < n; ++i) chunks[i] = full;
    chunks[0] -= n * full - nc;
    return (int)n;
}

struct Layout {
    size_t ws, state, q, k, v, g, beta, out, slot_in, slot_out, total;
};

// Device bytes for one problem: the chunk workspace of one slice, the carried
// state, g and beta of the whole sequence (a few hundred KB, copied once), and
// kSlots staging buffers of one slice of q/k/v and of out each.
Layout layout(int64_t B, int64_t T, int64_t Ts, int64_t H, size_t qkv_es, size_t gb_es, size_t out_es) {
    Layout L{};
    const size_t rows = (size_t)(B * Ts * H);
    L.ws = align256(gdn_chunk_workspace_bytes(B, Ts, H, gdn::kDk, gdn::kDv, GDN_BF16));
    L.state = align256((size_t)B * H * gdn::kDk * gdn::kDv * sizeof(float));
    L.g = align256((size_t)(B * T * H) * gb_es);
    L.beta = L.g;
    L.q = align256(rows * gdn::kDk * qkv_es);
    L.k = L.q;
    L.v = align256(rows * gdn::kDv * qkv_es);
    L.out = align256(rows * gdn::kDv * out_es);
    L.slot_in = L.q + L.k + L.v;
    L.slot_out = L.out;
    L.total = L.ws + L.state + L.g + L.beta + kSlots * (L.slot_in + L.slot_out);
    return L;
}

// Host views must hold whole tokens back to back ([B][T][H][D] with only the
// batch stride free), so that a time slice of one sequence is one contiguous run.
int check_packed4(const char* name, const gdn_tensor* t) {
    if (t->stride[3] != 1 || t->stride[2] != t->shape[3] || t->stride[1] != t->shape[2] * t->shape[3] ||
        (t->shape[0] > 1 && t->stride[0] < t->shape[1] * t->stride[1]))
        return gdn::set_last_error(GDN_ERR_UNSUPPORTED,
                                   "%s: host buffers must be packed [B][T][H][D] (token stride H*D, head stride D)", name);
    return GDN_OK;
}

int check_packed3(const char* name, const gdn_tensor* t) {
    if (t->stride[2] != 1 || t->stride[1] != t->shape[2] ||
        (t->shape[0] > 1 && t->stride[0] < t->shape[1] * t->stride[1]))
        return gdn::set_last_error(GDN_ERR_UNSUPPORTED, "%s: host buffers must be packed [B][T][H] (token stride H)",
                                   name);
    return GDN_OK;
}

int check_shapes(const gdn_tensor* q, const gdn_tensor* k, const gdn_tensor* v, const gdn_tensor* g,
                 const gdn_tensor* beta, const gdn_tensor* out) {
    const gdn_tensor* t4[4] = {q, k, v, out};
    const char* n4[4] = {"query", "key", "value", "out"};
    for (int i = 0; i < 4; ++i) {
        if (!t4[i]) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s is NULL", n4[i]);
        if (t4[i]->ndim != 4)
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s must be 4-D [B,T,H,D], got ndim=%d", n4[i],
                                       t4[i]->ndim);
        if (t4[i]->dtype != GDN_F32 && t4[i]->dtype != GDN_BF16 && t4[i]->dtype != GDN_F16)
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s has unsupported dtype code %d", n4[i],
                                       t4[i]->dtype);
        if (t4[i]->shape[0] != q->shape[0] || t4[i]->shape[1] != q->shape[1] || t4[i]->shape[2] != q->shape[2])
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s: [B,T,H] differs from query's", n4[i]);
        if (t4[i]->shape[3] != (i < 2 ? gdn::kDk : gdn::kDv))
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s head dim must be %d, got %lld", n4[i],
                                       i < 2 ? gdn::kDk : gdn::kDv, (long long)t4[i]->shape[3]);
    }
    const gdn_tensor* t3[2] = {g, beta};
    const char* n3[2] = {"g", "beta"};
    for (int i = 0; i < 2; ++i) {
        if (!t3[i]) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s is NULL", n3[i]);
        if (t3[i]->ndim != 3)
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s must be 3-D [B,T,H], got ndim=%d", n3[i],
                                       t3[i]->ndim);
        if (t3[i]->dtype != GDN_F32 && t3[i]->dtype != GDN_BF16 && t3[i]->dtype != GDN_F16)
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s has unsupported dtype code %d", n3[i],
                                       t3[i]->dtype);
        if (t3[i]->shape[0] != q->shape[0] || t3[i]->shape[1] != q->shape[1] || t3[i]->shape[2] != q->shape[2])
            return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "%s: [B,T,H] differs from query's", n3[i]);
    }
    int rc;
    for (int i = 0; i < 4; ++i)
        if ((rc = check_packed4(n4[i], t4[i]))) return rc;
    for (int i = 0; i < 2; ++i)
        if ((rc = check_packed3(n3[i], t3[i]))) return rc;
    return GDN_OK;
}

// Copy tokens [t0, t0+n) of every sequence between a packed host view and a
// staging buffer holding `cap` tokens per sequence.
cudaError_t copy_slice(void* dev, const gdn_tensor* host, int64_t t0, int64_t n, int64_t cap, bool to_device,
                       cudaStream_t st) {
    const size_t es = esize(host->dtype);
    const size_t tok = (size_t)host->stride[1] * es;  // bytes per token (H*D or H elements)
    const size_t width = (size_t)n * tok;
    const size_t dpitch = (size_t)cap * tok;
    const size_t hpitch = host->shape[0] > 1 ? (size_t)host->stride[0] * es : width;
    unsigned char* h = reinterpret_cast<unsigned char*>(host->data) + (size_t)t0 * tok;
    if (host->shape[0] == 1 || (hpitch == width && dpitch == width)) {  // one run: a plain copy is faster
        const size_t bytes = width * (size_t)host->shape[0];
        return to_device ? cudaMemcpyAsync(dev, h, bytes, cudaMemcpyHostToDevice, st)
                         : cudaMemcpyAsync(h, dev, bytes, cudaMemcpyDeviceToHost, st);
    }
    if (to_device)
        return cudaMemcpy2DAsync(dev, dpitch, h, hpitch, width, (size_t)host->shape[0], cudaMemcpyHostToDevice, st);
    return cudaMemcpy2DAsync(h, hpitch, dev, dpitch, width, (size_t)host->shape[0], cudaMemcpyDeviceToHost, st);
}

// View of tokens [t0, t0+n) of a device copy holding `cap` tokens per sequence.
gdn_tensor staged(const gdn_tensor* host, void* dev, int64_t t0, int64_t n, int64_t cap) {
    gdn_tensor t = *host;
    t.data = reinterpret_cast<unsigned char*>(dev) + (size_t)(t0 * host->stride[1]) * esize(host->dtype);
    t.shape[1] = n;
    t.stride[0] = cap * host->stride[1];
    return t;
}

}  // namespace

extern "C" {

size_t gdn_chunk_host_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype,
                                      int64_t slice_tokens) {
    (void)Dk;
    (void)Dv;
    if (B <= 0 || T <= 0 || H <= 0 || slice_tokens < 0 || slice_tokens % gdn::kChunk) return 0;
    const size_t es = esize(qkv_dtype);
    return layout(B, T, max_slice(B, T, H, es, slice_tokens), H, es, 4, es).total;
}

int gdn_chunk_gated_delta_rule_host(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                    const gdn_tensor* g, const gdn_tensor* beta, int chunk_size,
                                    const float* initial_state, int output_final_state, int use_qk_l2norm_in_kernel,
                                    gdn_tensor* out, float* final_state, int64_t slice_tokens, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (chunk_size != gdn::kChunk)
        return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "chunk_size must be %d, got %d", gdn::kChunk, chunk_size);
    if (slice_tokens < 0 || slice_tokens % gdn::kChunk)
        return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "slice_tokens must be 0 or a positive multiple of %d",
                                   gdn::kChunk);
    int rc = check_shapes(query, key, value, g, beta, out);
    if (rc) return rc;
    const int64_t B = query->shape[0], T = query->shape[1], H = query->shape[2];
    if (B < 0 || T < 0 || H < 0) return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "negative dimension in query");
    if (output_final_state && !final_state && B * H > 0)
        return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "output_final_state is set but final_state is NULL");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const size_t state_bytes = (size_t)B * H * gdn::kDk * gdn::kDv * sizeof(float);
    if (B * H == 0) return GDN_OK;
    if (T == 0) {  // no tokens: the final state is the initial state (or zeros)
        if (!output_final_state) return GDN_OK;
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return gdn::set_last_error(GDN_ERR_CUDA, "cudaStreamSynchronize: %s", cudaGetErrorName(e));
        if (!initial_state) std::memset(final_state, 0, state_bytes);
        else if (initial_state != final_state) std::memcpy(final_state, initial_state, state_bytes);
        return GDN_OK;
    }

    size_t qkv_es = esize(query->dtype);
    if (esize(key->dtype) > qkv_es) qkv_es = esize(key->dtype);
    if (esize(value->dtype) > qkv_es) qkv_es = esize(value->dtype);
    const int64_t Ts = max_slice(B, T, H, esize(query->dtype), slice_tokens);
    static thread_local int64_t chunks[4096];
    const int nslices = schedule(T, Ts, chunks, 4096);
    if (nslices < 0)
        return gdn::set_last_error(GDN_ERR_INVALID_ARGUMENT, "more than 4096 slices: raise slice_tokens");
    const size_t gb_es = esize(g->dtype) > esize(beta->dtype) ? esize(g->dtype) : esize(beta->dtype);
    const Layout L = layout(B, T, Ts, H, qkv_es, gb_es, esize(out->dtype));
    if (!workspace || workspace_bytes < L.total)
        return gdn::set_last_error(GDN_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", L.total,
                                   workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return gdn::set_last_error(GDN_ERR_WORKSPACE, "workspace must be 256-byte aligned");

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return gdn::set_last_error(GDN_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorName(e));
    if (dev < 0 || dev >= 64) return gdn::set_last_error(GDN_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_pipe_mutex[dev]);
    Pipe& P = g_pipes[dev];
    if ((e = pipe_init(P)) != cudaSuccess)
        return gdn::set_last_error(GDN_ERR_CUDA, "copy streams: %s", cudaGetErrorName(e));

    unsigned char* base = reinterpret_cast<unsigned char*>(workspace);
    void* ws = base;
    float* state = reinterpret_cast<float*>(base + L.ws);
    void* dg = base + L.ws + L.state;
    void* db = base + L.ws + L.state + L.g;
    unsigned char* slot_in[kSlots];
    unsigned char* slot_out[kSlots];
    for (int s = 0; s < kSlots; ++s) {
        slot_in[s] = base + L.ws + L.state + L.g + L.beta + s * L.slot_in;
        slot_out[s] = base + L.ws + L.state + L.g + L.beta + kSlots * L.slot_in + s * L.slot_out;
    }

#define GDN_TRY(call, what)                                                                                        \
    do {                                                                                                           \
        cudaError_t e_ = (call);                                                                                   \
        if (e_ != cudaSuccess) return gdn::set_last_error(GDN_ERR_CUDA, "%s: %s", what, cudaGetErrorName(e_));     \
    } while (0)

    // everything already queued on the caller's stream comes first
    GDN_TRY(cudaEventRecord(P.start, st), "cudaEventRecord");
    GDN_TRY(cudaStreamWaitEvent(P.in, P.start, 0), "cudaStreamWaitEvent");
    GDN_TRY(cudaStreamWaitEvent(P.out, P.start, 0), "cudaStreamWaitEvent");
    if (initial_state)
        GDN_TRY(cudaMemcpyAsync(state, initial_state, state_bytes, cudaMemcpyHostToDevice, P.in), "initial state copy");
    GDN_TRY(copy_slice(dg, g, 0, T, T, true, P.in), "g copy");
    GDN_TRY(copy_slice(db, beta, 0, T, T, true, P.in), "beta copy");

    int64_t t0 = 0;
    for (int s = 0; s < nslices; t0 += chunks[s] * gdn::kChunk, ++s) {
        const int slot = s % kSlots;
        const int64_t n = (T - t0 < chunks[s] * gdn::kChunk) ? T - t0 : chunks[s] * gdn::kChunk;
        unsigned char* in = slot_in[slot];
        void* dq = in;
        void* dk = in + L.q;
        void* dv = in + L.q + L.k;
        if (s >= kSlots) GDN_TRY(cudaStreamWaitEvent(P.in, P.comp_done[slot], 0), "cudaStreamWaitEvent");
        GDN_TRY(copy_slice(dq, query, t0, n, Ts, true, P.in), "query copy");
        GDN_TRY(copy_slice(dk, key, t0, n, Ts, true, P.in), "key copy");
        GDN_TRY(copy_slice(dv, value, t0, n, Ts, true, P.in), "value copy");
        GDN_TRY(cudaEventRecord(P.in_done[slot], P.in), "cudaEventRecord");

        GDN_TRY(cudaStreamWaitEvent(st, P.in_done[slot], 0), "cudaStreamWaitEvent");
        if (s >= kSlots) GDN_TRY(cudaStreamWaitEvent(st, P.out_done[slot], 0), "cudaStreamWaitEvent");
        const gdn_tensor sq = staged(query, dq, 0, n, Ts), sk = staged(key, dk, 0, n, Ts);
        const gdn_tensor sv = staged(value, dv, 0, n, Ts);
        const gdn_tensor sg = staged(g, dg, t0, n, T), sb = staged(beta, db, t0, n, T);
        gdn_tensor so = staged(out, slot_out[slot], 0, n, Ts);
        const float* h0 = (s == 0 && !initial_state) ? nullptr : state;
        rc = gdn_chunk_gated_delta_rule(&sq, &sk, &sv, &sg, &sb, chunk_size, h0, 1, use_qk_l2norm_in_kernel, &so,
                                        state, ws, L.ws, st);
        if (rc) return rc;
        GDN_TRY(cudaEventRecord(P.comp_done[slot], st), "cudaEventRecord");

        GDN_TRY(cudaStreamWaitEvent(P.out, P.comp_done[slot], 0), "cudaStreamWaitEvent");
        GDN_TRY(copy_slice(slot_out[slot], out, t0, n, Ts, false, P.out), "out copy");
        GDN_TRY(cudaEventRecord(P.out_done[slot], P.out), "cudaEventRecord");
    }
    if (output_final_state)
        GDN_TRY(cudaMemcpyAsync(final_state, state, state_bytes, cudaMemcpyDeviceToHost, P.out), "final state copy");
    // the caller's stream continues once the last copy has landed
    GDN_TRY(cudaEventRecord(P.end, P.out), "cudaEventRecord");
    GDN_TRY(cudaStreamWaitEvent(st, P.end, 0), "cudaStreamWaitEvent");
#undef GDN_TRY
    return GDN_OK;
}

}  // extern "C"
