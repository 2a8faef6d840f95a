// C ABI: argument validation, dispatch and error reporting.
//
// Mirrors the reference's Python contract for this path
// (fast_chunk_gated_delta_rule, qwen3_5_cutedsl_kernels.py:462-567;
//  torch_recurrent_gated_delta_rule, qwen3_5_transformers.py:190-229):
// same argument meaning, output in the query dtype, final state in fp32,
// inputs never modified.  Where the reference raises, this returns
// GDN_ERR_INVALID_ARGUMENT / GDN_ERR_UNSUPPORTED with a message.
#include <atomic>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <mutex>
#include <string>

#include "gdn_internal.h"

namespace {

thread_local std::string g_last_error;

// Sticky device error word: bounded waits inside the kernels that give up OR a
// bit in here (gdn_internal.h) instead of hanging or trapping, and also store it
// in a page-locked host mirror, so gdn_device_error_pending() can report it
// without synchronising.  The mirror is a page of this library's own host data
// (one word per device ordinal), page-locked and mapped into every device on the
// first call that needs an error word; its device address is written into the
// device word's `host_mirror` field then, once per device.
__device__ gdn::DeviceErrorWord g_device_error;
std::mutex g_err_mu;
void* g_device_error_addr[64];
alignas(4096) unsigned int g_mirror_page[1024];  // host words; [dev] mirrors device `dev`
bool g_mirror_tried = false, g_mirror_ok = false;
bool g_mirror_on[64];

// With g_err_mu held: the device address of device `dev`'s mirror word, or null if the page could not be
// page-locked (the error word then works without a host mirror).
unsigned int* mirror_alias(int dev) {
    if (!g_mirror_tried) {
        g_mirror_tried = true;
        g_mirror_ok = cudaHostRegister(g_mirror_page, sizeof(g_mirror_page),
                                       cudaHostRegisterPortable | cudaHostRegisterMapped) == cudaSuccess;
        if (!g_mirror_ok) cudaGetLastError();  // a failed registration leaves a (non-sticky) error behind
    }
    if (!g_mirror_ok) return nullptr;
    void* d = nullptr;
    if (cudaHostGetDevicePointer(&d, &g_mirror_page[dev], 0) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<unsigned int*>(d);
}

unsigned int* device_error_word(int dev) {
    if (dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_err_mu);
    if (!g_device_error_addr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
        unsigned int* alias = mirror_alias(dev);
        if (alias) {
            unsigned char* field = reinterpret_cast<unsigned char*>(ptr) + offsetof(gdn::DeviceErrorWord, host_mirror);
            if (cudaMemcpy(field, &alias, sizeof(alias), cudaMemcpyHostToDevice) == cudaSuccess) {
                g_mirror_on[dev] = true;
            } else {
                cudaGetLastError();
            }
        }
        g_device_error_addr[dev] = ptr;
    }
    return reinterpret_cast<unsigned int*>(g_device_error_addr[dev]);
}

// The tensor-core chunk path takes bf16 q/k/v/out whose rows are 16-byte aligned
// (its 16-byte asynchronous row copies need that); everything else runs on the
// CUDA-core path.
bool tc_eligible(const gdn_tensor* q, const gdn_tensor* k, const gdn_tensor* v, const gdn_tensor* out) {
    const gdn_tensor* in[3] = {q, k, v};
    for (const gdn_tensor* t : in) {
        if (t->dtype != GDN_BF16) return false;
        if ((reinterpret_cast<uintptr_t>(t->data) & 15) || (t->stride[0] & 7) || (t->stride[1] & 7) || (t->stride[2] & 7))
            return false;
    }
    if (out->dtype != GDN_BF16) return false;
    if ((reinterpret_cast<uintptr_t>(out->data) & 15) || (out->stride[0] & 7) || (out->stride[1] & 7) ||
        (out->stride[2] & 7))
        return false;
    return true;
}
thread_local void* const* g_phase_events = nullptr;
thread_local int g_phase_event_count = 0;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(GDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool valid_dtype(int d) { return d == GDN_F32 || d == GDN_BF16 || d == GDN_F16; }

// The kernels are compiled for sm_100a only; anything else cannot load them.
int check_device() {
    static std::atomic<int> major_plus1[64];  // compute capability major + 1 per device; 0 = not yet read
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(GDN_ERR_DEVICE, "device ordinal %d out of range", dev);
    int major = major_plus1[dev].load(std::memory_order_relaxed) - 1;
    if (major < 0) {
        e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        major_plus1[dev].store(major + 1, std::memory_order_relaxed);
    }
    if (major != 10)
        return fail(GDN_ERR_DEVICE, "device %d has compute capability %d.x; this library is built for sm_100a (B200)",
                    dev, major);
    return GDN_OK;
}

int check4(const char* name, const gdn_tensor* t, int64_t B, int64_t T, int64_t H, int64_t D) {
    if (!t) return fail(GDN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (t->ndim != 4) return fail(GDN_ERR_INVALID_ARGUMENT, "%s must be 4-D [B,T,H,D], got ndim=%d", name, t->ndim);
    if (!valid_dtype(t->dtype)) return fail(GDN_ERR_INVALID_ARGUMENT, "%s has unsupported dtype code %d", name, t->dtype);
    const int64_t want[4] = {B, T, H, D};
    for (int i = 0; i < 4; ++i)
        if (t->shape[i] != want[i])
            return fail(GDN_ERR_INVALID_ARGUMENT, "%s has shape [%lld,%lld,%lld,%lld], expected [%lld,%lld,%lld,%lld]", name,
                        (long long)t->shape[0], (long long)t->shape[1], (long long)t->shape[2], (long long)t->shape[3],
                        (long long)B, (long long)T, (long long)H, (long long)D);
    if (t->stride[3] != 1)
        return fail(GDN_ERR_INVALID_ARGUMENT, "%s: the head dimension must be contiguous (stride %lld)", name,
                    (long long)t->stride[3]);
    if (B * T * H > 0 && !t->data) return fail(GDN_ERR_INVALID_ARGUMENT, "%s has a NULL data pointer", name);
    return GDN_OK;
}

int check3(const char* name, const gdn_tensor* t, int64_t B, int64_t T, int64_t H) {
    if (!t) return fail(GDN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    if (t->ndim != 3) return fail(GDN_ERR_INVALID_ARGUMENT, "%s must be 3-D [B,T,H], got ndim=%d", name, t->ndim);
    if (!valid_dtype(t->dtype)) return fail(GDN_ERR_INVALID_ARGUMENT, "%s has unsupported dtype code %d", name, t->dtype);
    if (t->shape[0] != B || t->shape[1] != T || t->shape[2] != H)
        return fail(GDN_ERR_INVALID_ARGUMENT, "%s has shape [%lld,%lld,%lld], expected [%lld,%lld,%lld]", name,
                    (long long)t->shape[0], (long long)t->shape[1], (long long)t->shape[2], (long long)B, (long long)T,
                    (long long)H);
    if (B * T * H > 0 && !t->data) return fail(GDN_ERR_INVALID_ARGUMENT, "%s has a NULL data pointer", name);
    return GDN_OK;
}

gdn::View4 view4(const gdn_tensor* t) { return {t->data, t->stride[0], t->stride[1], t->stride[2], t->dtype}; }
gdn::View3 view3(const gdn_tensor* t) { return {t->data, t->stride[0], t->stride[1], t->stride[2], t->dtype}; }

// Shared checks of the two entry points; fills B, T, H.
int check_common(const gdn_tensor* q, const gdn_tensor* k, const gdn_tensor* v, const gdn_tensor* g,
                 const gdn_tensor* beta, const gdn_tensor* out, const float* h0, int output_final_state,
                 const float* hT, int64_t* B, int64_t* T, int64_t* H) {
    if (!q) return fail(GDN_ERR_INVALID_ARGUMENT, "query is NULL");
    if (q->ndim != 4) return fail(GDN_ERR_INVALID_ARGUMENT, "query must be 4-D [B,T,H,Dk], got ndim=%d", q->ndim);
    *B = q->shape[0];
    *T = q->shape[1];
    *H = q->shape[2];
    if (*B < 0 || *T < 0 || *H < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "negative dimension in query");
    if (q->shape[3] != gdn::kDk)
        return fail(GDN_ERR_INVALID_ARGUMENT, "key head dim must be %d, got %lld", gdn::kDk, (long long)q->shape[3]);
    if (!v) return fail(GDN_ERR_INVALID_ARGUMENT, "value is NULL");
    if (v->ndim == 4 && v->shape[3] != gdn::kDv)
        return fail(GDN_ERR_INVALID_ARGUMENT, "value head dim must be %d, got %lld", gdn::kDv, (long long)v->shape[3]);
    int rc;
    if ((rc = check4("query", q, *B, *T, *H, gdn::kDk))) return rc;
    if ((rc = check4("key", k, *B, *T, *H, gdn::kDk))) return rc;
    if ((rc = check4("value", v, *B, *T, *H, gdn::kDv))) return rc;
    if ((rc = check3("g", g, *B, *T, *H))) return rc;
    if ((rc = check3("beta", beta, *B, *T, *H))) return rc;
    if ((rc = check4("out", out, *B, *T, *H, gdn::kDv))) return rc;
    if (*B * *H > 0x7fffffffLL) return fail(GDN_ERR_INVALID_ARGUMENT, "B*H too large");
    if (h0 && (reinterpret_cast<uintptr_t>(h0) & 15))
        return fail(GDN_ERR_INVALID_ARGUMENT, "initial_state must be 16-byte aligned");
    if (output_final_state && !hT && *B * *H > 0)
        return fail(GDN_ERR_INVALID_ARGUMENT, "output_final_state is set but final_state is NULL");
    if (hT && (reinterpret_cast<uintptr_t>(hT) & 15))
        return fail(GDN_ERR_INVALID_ARGUMENT, "final_state must be 16-byte aligned");
    return GDN_OK;
}

// T == 0: no tokens; the final state is the initial state (or zeros).
int empty_sequence(int64_t B, int64_t H, const float* h0, float* hT, cudaStream_t stream) {
    if (!hT) return GDN_OK;
    const size_t bytes = (size_t)B * H * gdn::kDk * gdn::kDv * sizeof(float);
    cudaError_t e = cudaSuccess;
    if (!h0) e = cudaMemsetAsync(hT, 0, bytes, stream);
    else if (h0 != hT) e = cudaMemcpyAsync(hT, h0, bytes, cudaMemcpyDeviceToDevice, stream);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "final state copy");
}

}  // namespace

namespace gdn {

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_last_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

cudaError_t phase_event(int index, cudaStream_t stream) {
    if (!g_phase_events || index >= g_phase_event_count || !g_phase_events[index]) return cudaSuccess;
    return cudaEventRecord(reinterpret_cast<cudaEvent_t>(g_phase_events[index]), stream);
}

}  // namespace gdn

extern "C" {

uint64_t gdn_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

void gdn_set_phase_events(void* const* events, int n) {
    g_phase_events = events;
    g_phase_event_count = events ? n : 0;
}

size_t gdn_chunk_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype) {
    (void)Dk;
    (void)Dv;
    (void)qkv_dtype;
    if (B <= 0 || T <= 0 || H <= 0) return 0;
    const int64_t NC = (T + gdn::kChunk - 1) / gdn::kChunk;
    const size_t per_chunk = (size_t)gdn::kWsChunkFloats * sizeof(float) > (size_t)gdn::kTcChunkBytes
                                 ? (size_t)gdn::kWsChunkFloats * sizeof(float)
                                 : (size_t)gdn::kTcChunkBytes;
    return (size_t)(B * H * NC) * per_chunk;
}

int gdn_chunk_gated_delta_rule(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                               const gdn_tensor* g, const gdn_tensor* beta, int chunk_size,
                               const float* initial_state, int output_final_state, int use_qk_l2norm_in_kernel,
                               gdn_tensor* out, float* final_state, void* workspace, size_t workspace_bytes,
                               void* stream) {
    g_last_error.clear();
    if (chunk_size != gdn::kChunk)
        return fail(GDN_ERR_INVALID_ARGUMENT, "chunk_size must be %d, got %d", gdn::kChunk, chunk_size);
    int64_t B, T, H;
    int rc = check_common(query, key, value, g, beta, out, initial_state, output_final_state, final_state, &B, &T, &H);
    if (rc) return rc;
    if ((rc = check_device())) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* hT = output_final_state ? final_state : nullptr;
    if (B * H == 0) return GDN_OK;
    if (T == 0) return empty_sequence(B, H, initial_state, hT, st);

    int dev = 0;
    cudaGetDevice(&dev);
    const size_t need = gdn_chunk_workspace_bytes(B, T, H, gdn::kDk, gdn::kDv, query->dtype);
    if (!workspace || workspace_bytes < need)
        return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(GDN_ERR_WORKSPACE, "workspace must be 256-byte aligned");

    gdn::ChunkParams p{};
    p.q = view4(query);
    p.k = view4(key);
    p.v = view4(value);
    p.g = view3(g);
    p.beta = view3(beta);
    p.out = out->data;
    p.out_sb = out->stride[0];
    p.out_st = out->stride[1];
    p.out_sh = out->stride[2];
    p.out_dtype = out->dtype;
    p.h0 = initial_state;
    p.hT = hT;
    p.ws = reinterpret_cast<float*>(workspace);
    p.B = (int)B;
    p.H = (int)H;
    p.T = T;
    p.NC = (int)((T + gdn::kChunk - 1) / gdn::kChunk);
    p.l2norm = use_qk_l2norm_in_kernel ? 1 : 0;
    p.err = device_error_word(dev);
    cudaError_t e = tc_eligible(query, key, value, out) ? gdn::launch_chunk_tc(p, st) : gdn::launch_chunk_simt(p, st);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "chunk kernels launch");
}

size_t gdn_chunk_varlen_workspace_bytes(int64_t T, int64_t N, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype) {
    (void)Dk;
    (void)Dv;
    (void)qkv_dtype;
    if (T < 0 || N <= 0 || H <= 0) return 0;
    const int64_t max_chunks = (T + gdn::kChunk - 1) / gdn::kChunk + N;
    // tables: chunk bases (N + 1), chunk -> sequence (max_chunks), the scan's sequence order (N)
    const size_t header = ((size_t)(2 * N + 1 + max_chunks) * sizeof(int) + 255) & ~size_t(255);
    return header + (size_t)(max_chunks * H) * (size_t)gdn::kTcChunkBytes;
}

int gdn_chunk_gated_delta_rule_varlen(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                      const gdn_tensor* g, const gdn_tensor* beta, const int32_t* cu_seqlens,
                                      int64_t num_seqs, int chunk_size, const float* initial_state,
                                      int output_final_state, int use_qk_l2norm_in_kernel, gdn_tensor* out,
                                      float* final_state, void* workspace, size_t workspace_bytes, void* stream) {
    g_last_error.clear();
    if (chunk_size != gdn::kChunk)
        return fail(GDN_ERR_INVALID_ARGUMENT, "chunk_size must be %d, got %d", gdn::kChunk, chunk_size);
    int64_t B, T, H;
    int rc = check_common(query, key, value, g, beta, out, initial_state, output_final_state, final_state, &B, &T, &H);
    if (rc) return rc;
    if (B != 1) return fail(GDN_ERR_INVALID_ARGUMENT, "packed sequences need B == 1, got B=%lld", (long long)B);
    if (num_seqs <= 0 || num_seqs > 0x7fffffffLL || T > 0x7fffffffLL || num_seqs * H > 0x7fffffffLL)
        return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs must be in [1, 2^31) and T < 2^31");
    if (!cu_seqlens) return fail(GDN_ERR_INVALID_ARGUMENT, "cu_seqlens is NULL");
    if (H > 0 && !tc_eligible(query, key, value, out))
        return fail(GDN_ERR_UNSUPPORTED, "packed sequences need bf16 q/k/v/out with 16-byte aligned rows");
    if ((rc = check_device())) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* hT = output_final_state ? final_state : nullptr;
    if (H == 0) return GDN_OK;
    if (T == 0) return empty_sequence(num_seqs, H, initial_state, hT, st);
    const size_t need = gdn_chunk_varlen_workspace_bytes(T, num_seqs, H, gdn::kDk, gdn::kDv, query->dtype);
    if (!workspace || workspace_bytes < need)
        return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(GDN_ERR_WORKSPACE, "workspace must be 256-byte aligned");

    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t max_chunks = (T + gdn::kChunk - 1) / gdn::kChunk + num_seqs;
    const size_t header = ((size_t)(2 * num_seqs + 1 + max_chunks) * sizeof(int) + 255) & ~size_t(255);
    int* tables = reinterpret_cast<int*>(workspace);
    gdn::ChunkParams p{};
    p.q = view4(query);
    p.k = view4(key);
    p.v = view4(value);
    p.g = view3(g);
    p.beta = view3(beta);
    p.out = out->data;
    p.out_sb = out->stride[0];
    p.out_st = out->stride[1];
    p.out_sh = out->stride[2];
    p.out_dtype = out->dtype;
    p.h0 = initial_state;
    p.hT = hT;
    p.ws = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(workspace) + header);
    p.B = 1;
    p.H = (int)H;
    p.T = T;
    p.NC = (int)((T + gdn::kChunk - 1) / gdn::kChunk);
    p.l2norm = use_qk_l2norm_in_kernel ? 1 : 0;
    p.err = device_error_word(dev);
    p.cu_seqlens = cu_seqlens;
    p.chunk_base = tables;
    p.chunk_seq = tables + num_seqs + 1;
    p.seq_order = tables + num_seqs + 1 + max_chunks;
    p.N = (int)num_seqs;
    p.max_chunks = (int)max_chunks;
    cudaError_t e = gdn::launch_varlen_tables(p, st);
    if (e == cudaSuccess) e = gdn::launch_chunk_tc(p, st);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "packed-sequence chunk kernels launch");
}

size_t gdn_chunk_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t Dk, int64_t Dv, int qkv_dtype) {
    (void)Dk;
    (void)Dv;
    (void)qkv_dtype;
    if (B <= 0 || T <= 0 || H <= 0) return 0;
    const int64_t NC = (T + gdn::kChunk - 1) / gdn::kChunk;
    // CUDA-core forward tiles + backward records + the tensor-core forward records (bf16 inputs)
    return (size_t)(B * H * NC) * ((size_t)(gdn::kWsChunkFloats + gdn::kBwChunkFloats) * sizeof(float) +
                                   (size_t)gdn::kTcChunkBytes);
}

int gdn_chunk_gated_delta_rule_bwd(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                   const gdn_tensor* g, const gdn_tensor* beta, const gdn_tensor* d_out, int chunk_size,
                                   const float* initial_state, const float* d_final_state, int use_qk_l2norm_in_kernel,
                                   gdn_tensor* dq, gdn_tensor* dk, gdn_tensor* dv, gdn_tensor* dg, gdn_tensor* dbeta,
                                   float* dh0, void* workspace, size_t workspace_bytes, void* stream) {
    g_last_error.clear();
    if (chunk_size != gdn::kChunk)
        return fail(GDN_ERR_INVALID_ARGUMENT, "chunk_size must be %d, got %d", gdn::kChunk, chunk_size);
    int64_t B, T, H;
    int rc = check_common(query, key, value, g, beta, d_out, initial_state, 0, nullptr, &B, &T, &H);
    if (rc) return rc;
    if ((rc = check4("dq", dq, B, T, H, gdn::kDk))) return rc;
    if ((rc = check4("dk", dk, B, T, H, gdn::kDk))) return rc;
    if ((rc = check4("dv", dv, B, T, H, gdn::kDv))) return rc;
    if ((rc = check3("dg", dg, B, T, H))) return rc;
    if ((rc = check3("dbeta", dbeta, B, T, H))) return rc;
    if ((rc = check_device())) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (B * H == 0) return GDN_OK;
    if (T == 0) {  // no tokens: the initial state's gradient is the final state's
        if (!dh0) return GDN_OK;
        const size_t bytes = (size_t)B * H * gdn::kDk * gdn::kDv * sizeof(float);
        cudaError_t e = d_final_state ? cudaMemcpyAsync(dh0, d_final_state, bytes, cudaMemcpyDeviceToDevice, st)
                                      : cudaMemsetAsync(dh0, 0, bytes, st);
        return e == cudaSuccess ? GDN_OK : cuda_fail(e, "initial-state gradient copy");
    }
    const size_t need = gdn_chunk_bwd_workspace_bytes(B, T, H, gdn::kDk, gdn::kDv, query->dtype);
    if (!workspace || workspace_bytes < need)
        return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(GDN_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    gdn::ChunkParams f{};
    f.q = view4(query);
    f.k = view4(key);
    f.v = view4(value);
    f.g = view3(g);
    f.beta = view3(beta);
    f.h0 = initial_state;
    f.B = (int)B;
    f.H = (int)H;
    f.T = T;
    f.NC = (int)((T + gdn::kChunk - 1) / gdn::kChunk);
    f.l2norm = use_qk_l2norm_in_kernel ? 1 : 0;
    f.err = device_error_word(dev);
    gdn::BwdParams p{};
    p.q = f.q;
    p.k = f.k;
    p.v = f.v;
    p.g = f.g;
    p.beta = f.beta;
    p.dout = view4(d_out);
    p.h0 = initial_state;
    p.dhT = d_final_state;
    p.dh0 = dh0;
    p.dq = {dq->data, dq->stride[0], dq->stride[1], dq->stride[2], dq->dtype};
    p.dk = {dk->data, dk->stride[0], dk->stride[1], dk->stride[2], dk->dtype};
    p.dv = {dv->data, dv->stride[0], dv->stride[1], dv->stride[2], dv->dtype};
    p.dg = {dg->data, dg->stride[0], dg->stride[1], dg->stride[2], dg->dtype};
    p.dbeta = {dbeta->data, dbeta->stride[0], dbeta->stride[1], dbeta->stride[2], dbeta->dtype};
    p.fws = reinterpret_cast<float*>(workspace);
    p.bws = p.fws + (size_t)(B * H * f.NC) * gdn::kWsChunkFloats;
    // bf16 q/k/v/d_out with 16-byte aligned rows: the forward recompute and the reverse scan on the tensor cores
    p.tc_records = tc_eligible(query, key, value, d_out)
                       ? reinterpret_cast<void*>(p.bws + (size_t)(B * H * f.NC) * gdn::kBwChunkFloats)
                       : nullptr;
    p.err = f.err;
    p.B = f.B;
    p.H = f.H;
    p.NC = f.NC;
    p.T = T;
    p.l2norm = f.l2norm;
    cudaError_t e = gdn::launch_chunk_bwd(f, p, st);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "backward kernels launch");
}

int gdn_recurrent_gated_delta_rule(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value,
                                   const gdn_tensor* g, const gdn_tensor* beta, const float* initial_state,
                                   int output_final_state, int use_qk_l2norm_in_kernel, gdn_tensor* out,
                                   float* final_state, void* stream) {
    g_last_error.clear();
    int64_t B, T, H;
    int rc = check_common(query, key, value, g, beta, out, initial_state, output_final_state, final_state, &B, &T, &H);
    if (rc) return rc;
    if ((rc = check_device())) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* hT = output_final_state ? final_state : nullptr;
    if (B * H == 0) return GDN_OK;
    if (B * H > 0x7fffffffLL / 4) return fail(GDN_ERR_INVALID_ARGUMENT, "B*H too large for the recurrent rule");
    if (T == 0) return empty_sequence(B, H, initial_state, hT, st);

    gdn::RecurrentParams p{};
    p.q = view4(query);
    p.k = view4(key);
    p.v = view4(value);
    p.g = view3(g);
    p.beta = view3(beta);
    p.out = out->data;
    p.out_sb = out->stride[0];
    p.out_st = out->stride[1];
    p.out_sh = out->stride[2];
    p.out_dtype = out->dtype;
    p.h0 = initial_state;
    p.hT = hT;
    p.B = (int)B;
    p.H = (int)H;
    p.T = T;
    p.l2norm = use_qk_l2norm_in_kernel ? 1 : 0;
    cudaError_t e = gdn::launch_recurrent(p, st);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "recurrent kernel launch");
}

// ---------------------------------------------------------------- sequence parallelism

namespace {

// Validates a time shard for the sequence-parallel calls and fills the shared kernel parameters.
int sp_params(const gdn_tensor* q, const gdn_tensor* k, const gdn_tensor* v, const gdn_tensor* g,
              const gdn_tensor* beta, int chunk_size, int use_qk_l2norm, const gdn_tensor* out, const void* ws,
              size_t ws_bytes, gdn::ChunkParams* p) {
    if (chunk_size != gdn::kChunk)
        return fail(GDN_ERR_INVALID_ARGUMENT, "chunk_size must be %d, got %d", gdn::kChunk, chunk_size);
    if (!q || q->ndim != 4) return fail(GDN_ERR_INVALID_ARGUMENT, "query must be 4-D [B,T,H,Dk]");
    const int64_t B = q->shape[0], T = q->shape[1], H = q->shape[2];
    if (B <= 0 || T <= 0 || H <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "a time shard needs B, T, H > 0");
    int rc;
    if ((rc = check4("query", q, B, T, H, gdn::kDk))) return rc;
    if ((rc = check4("key", k, B, T, H, gdn::kDk))) return rc;
    if ((rc = check4("value", v, B, T, H, gdn::kDv))) return rc;
    if ((rc = check3("g", g, B, T, H))) return rc;
    if ((rc = check3("beta", beta, B, T, H))) return rc;
    if (out && (rc = check4("out", out, B, T, H, gdn::kDv))) return rc;
    if (!tc_eligible(q, k, v, out ? out : v))
        return fail(GDN_ERR_UNSUPPORTED, "sequence-parallel shards need bf16 q/k/v%s with 16-byte aligned rows",
                    out ? "/out" : "");
    if ((rc = check_device())) return rc;
    const size_t need = gdn_chunk_workspace_bytes(B, T, H, gdn::kDk, gdn::kDv, q->dtype);
    if (!ws || ws_bytes < need)
        return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, ws ? ws_bytes : 0);
    if (reinterpret_cast<uintptr_t>(ws) & 255) return fail(GDN_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    *p = gdn::ChunkParams{};
    p->q = view4(q);
    p->k = view4(k);
    p->v = view4(v);
    p->g = view3(g);
    p->beta = view3(beta);
    p->ws = reinterpret_cast<float*>(const_cast<void*>(ws));
    p->B = (int)B;
    p->H = (int)H;
    p->T = T;
    p->NC = (int)((T + gdn::kChunk - 1) / gdn::kChunk);
    p->l2norm = use_qk_l2norm ? 1 : 0;
    p->err = device_error_word(dev);
    return GDN_OK;
}

}  // namespace

int gdn_chunk_sp_summary(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value, const gdn_tensor* g,
                         const gdn_tensor* beta, int chunk_size, int use_qk_l2norm_in_kernel, float* transition,
                         float* local_state, void* workspace, size_t workspace_bytes, void* stream) {
    g_last_error.clear();
    gdn::ChunkParams p;
    int rc = sp_params(query, key, value, g, beta, chunk_size, use_qk_l2norm_in_kernel, nullptr, workspace,
                       workspace_bytes, &p);
    if (rc) return rc;
    if (!transition || !local_state || (reinterpret_cast<uintptr_t>(transition) & 15) ||
        (reinterpret_cast<uintptr_t>(local_state) & 15))
        return fail(GDN_ERR_INVALID_ARGUMENT, "transition and local_state must be 16-byte aligned fp32 buffers");
    p.scan_mode = 1;
    p.hT = transition;
    p.hT2 = local_state;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = gdn::launch_chunk_tc_prep(p, st);
    if (e == cudaSuccess) e = gdn::launch_chunk_tc_scan(p, st);
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "shard summary launch");
}

int gdn_chunk_sp_finish(const gdn_tensor* query, const gdn_tensor* key, const gdn_tensor* value, const gdn_tensor* g,
                        const gdn_tensor* beta, int chunk_size, const float* initial_state, int output_final_state,
                        int use_qk_l2norm_in_kernel, gdn_tensor* out, float* final_state, const void* workspace,
                        size_t workspace_bytes, void* stream) {
    g_last_error.clear();
    if (!out) return fail(GDN_ERR_INVALID_ARGUMENT, "out is NULL");
    gdn::ChunkParams p;
    int rc = sp_params(query, key, value, g, beta, chunk_size, use_qk_l2norm_in_kernel, out, workspace,
                       workspace_bytes, &p);
    if (rc) return rc;
    if (initial_state && (reinterpret_cast<uintptr_t>(initial_state) & 15))
        return fail(GDN_ERR_INVALID_ARGUMENT, "initial_state must be 16-byte aligned");
    if (output_final_state && (!final_state || (reinterpret_cast<uintptr_t>(final_state) & 15)))
        return fail(GDN_ERR_INVALID_ARGUMENT, "final_state must be a 16-byte aligned fp32 buffer");
    p.out = out->data;
    p.out_sb = out->stride[0];
    p.out_st = out->stride[1];
    p.out_sh = out->stride[2];
    p.out_dtype = out->dtype;
    p.h0 = initial_state;
    p.hT = output_final_state ? final_state : nullptr;
    cudaError_t e = gdn::launch_chunk_tc_scan(p, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "shard finish launch");
}

unsigned int gdn_device_error(int clear) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    unsigned int* w = device_error_word(dev);
    if (!w) return 0;
    unsigned int v = 0;
    if (cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    volatile unsigned int* mirror = g_mirror_on[dev] ? &g_mirror_page[dev] : nullptr;
    if (mirror) v |= *mirror;
    if (clear && v) {
        const unsigned int zero = 0;
        cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice);
        if (mirror) *mirror = 0;
    }
    return v;
}

unsigned int gdn_device_error_pending(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    return g_mirror_on[dev] ? *reinterpret_cast<volatile unsigned int*>(&g_mirror_page[dev]) : 0u;
}

int gdn_selftest_bounded_wait(uint64_t timeout_ns, void* stream) {
    g_last_error.clear();
    int rc = check_device();
    if (rc) return rc;
    if (timeout_ns < 1000ull || timeout_ns > 100000000ull)
        return fail(GDN_ERR_INVALID_ARGUMENT, "timeout_ns must be in [1e3, 1e8], got %llu",
                    (unsigned long long)timeout_ns);
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned int* w = device_error_word(dev);
    if (!w) return fail(GDN_ERR_CUDA, "device error word not found");
    cudaError_t e = gdn::launch_selftest_wait(w, timeout_ns, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? GDN_OK : cuda_fail(e, "bounded-wait self-test launch");
}

const char* gdn_last_error(void) { return g_last_error.c_str(); }

const char* gdn_status_name(int status) {
    switch (status) {
        case GDN_OK: return "GDN_OK";
        case GDN_ERR_INVALID_ARGUMENT: return "GDN_ERR_INVALID_ARGUMENT";
        case GDN_ERR_UNSUPPORTED: return "GDN_ERR_UNSUPPORTED";
        case GDN_ERR_WORKSPACE: return "GDN_ERR_WORKSPACE";
        case GDN_ERR_CUDA: return "GDN_ERR_CUDA";
        case GDN_ERR_DEVICE: return "GDN_ERR_DEVICE";
        case GDN_ERR_KERNEL: return "GDN_ERR_KERNEL";
        default: return "GDN_UNKNOWN_STATUS";
    }
}

int gdn_abi_version(void) { return GDN_ABI_VERSION; }

}  // extern "C"
