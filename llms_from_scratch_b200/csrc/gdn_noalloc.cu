// Chunked forward for callers that cannot allocate device memory.
//
// gdn_chunk_gated_delta_rule needs a workspace the caller allocates.  Some
// callers cannot do that at the point they run the op: a runtime that plans
// every device buffer ahead of time and hands out no memory while a graph of
// ops executes, a plugin whose host framework owns all allocations and exposes
// no allocator to it, or code running where calling cudaMalloc would
// synchronise the device or fail (for example while another component holds
// all free memory).  This entry point takes inputs and outputs only and uses a
// fixed scratch array compiled into the library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes; every
// GPU that loads this library holds it until the process exits.  Host code
// cannot use the array's name as a device address (in host code it names a
// host-side stand-in), so the first call on each device looks up the real
// device address with cudaGetSymbolAddress, with that device current, and
// caches it; later calls reuse it.  All calls share the one array:
//   * nothing in it has to start at zero: the prep kernel writes every
//     workspace element the scan kernel reads, within the same call;
//   * it keeps the previous call's contents, and two calls that overlap on the
//     GPU (different streams, or different host threads) race on it; callers
//     must order such calls on one stream or synchronise between them.
#include <cstdio>
#include <mutex>

#include "gdn_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = GDN_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64];  // device address of g_noalloc_scratch, per device ordinal

// Looks up (once per device) the device address of the scratch array on the current device.
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return gdn::set_last_error(GDN_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return gdn::set_last_error(GDN_ERR_DEVICE, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return gdn::set_last_error(GDN_ERR_CUDA, "cudaGetSymbolAddress of the fixed scratch failed: %s",
                                       cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return GDN_OK;
}

}  // namespace

extern "C" int gdn_chunk_gated_delta_rule_noalloc(const gdn_tensor* query, const gdn_tensor* key,
                                                  const gdn_tensor* value, const gdn_tensor* g,
                                                  const gdn_tensor* beta, int chunk_size,
                                                  const float* initial_state, int output_final_state,
                                                  int use_qk_l2norm_in_kernel, gdn_tensor* out,
                                                  float* final_state, void* stream) {
    if (query && query->ndim == 4) {
        const size_t need = gdn_chunk_workspace_bytes(query->shape[0], query->shape[1], query->shape[2],
                                                      query->shape[3], value ? value->shape[3] : 0, query->dtype);
        if (need > kNoAllocScratchBytes)
            return gdn::set_last_error(
                GDN_ERR_WORKSPACE,
                "problem too large for the fixed scratch: B=%lld T=%lld H=%lld needs %zu bytes, the fixed "
                "scratch holds %zu bytes (use gdn_chunk_gated_delta_rule with a caller workspace)",
                (long long)query->shape[0], (long long)query->shape[1], (long long)query->shape[2], need,
                kNoAllocScratchBytes);
    }
    void* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc != GDN_OK) return rc;
    return gdn_chunk_gated_delta_rule(query, key, value, g, beta, chunk_size, initial_state, output_final_state,
                                      use_qk_l2norm_in_kernel, out, final_state, scratch, kNoAllocScratchBytes,
                                      stream);
}
