// trident_search_noalloc: the query path for callers that cannot allocate device memory.
//
// Some callers cannot allocate: for example code running where cudaMalloc is forbidden or
// unavailable (an allocator-less embedding, a host that hands the library only fixed buffers, or
// a runtime that must not trigger device allocations once serving has started). For them this
// entry point runs the same search as trident_search, but its workspace is a fixed array compiled
// into the library instead of a buffer the caller provides. The caller still provides the queries
// and the output buffers.
//
// The array is TRIDENT_NOALLOC_WORKSPACE_BYTES (32 MiB) per GPU. Every GPU that loads the library
// keeps it until the process exits. All calls on a device share it, so calls whose GPU work overlaps
// in time (different streams, or threads issuing concurrently) race and corrupt each other's results.
// Such callers must serialise. The search resets the counters it needs on every call
// (cudaMemsetAsync on the stream, which is not an allocation) and writes every other workspace
// value before reading it, so the contents left by the previous call do no harm.
//
// The first call on each device looks up the array's device address (cudaGetSymbolAddress, with
// that device current) and caches it. Like trident_search, the first search from each host thread on
// each device also creates the library's side stream and its four events (which are not device
// memory allocations, but are not allowed during stream capture either): make that first call
// before capturing any stream.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "tb_internal.h"
#include "trident_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_ws[TRIDENT_NOALLOC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ws_ptr[kMaxDevices] = {nullptr};

// Device address of this device's array, looked up once per device with that device current.
// In host code g_noalloc_ws is only a stand-in symbol, never a device address.
cudaError_t workspace_of_current_device(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ws_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_ws);
        if (e != cudaSuccess) return e;
        g_ws_ptr[dev] = p;
    }
    *out = g_ws_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int trident_search_noalloc(const trident_index* idx, const float* xq, int32_t B, int32_t K,
                                      int32_t nprobe, int32_t mode, int32_t ub_seed, float* out_d, int64_t* out_i,
                                      int64_t* stats, void* stream) {
    size_t need = 0;
    const int rc = trident_workspace_size(idx, B, K, nprobe, &need);
    if (rc) return rc;
    char msg[256];
    if (need > (size_t)TRIDENT_NOALLOC_WORKSPACE_BYTES) {
        snprintf(msg, sizeof(msg),
                 "trident_search_noalloc: B=%d K=%d nprobe=%d needs %zu workspace bytes, more than the fixed "
                 "%zu-byte no-alloc workspace; split the batch or use trident_search",
                 B, K, nprobe, need, (size_t)TRIDENT_NOALLOC_WORKSPACE_BYTES);
        return tb::record_error(TRIDENT_ERR_WORKSPACE, msg);
    }
    void* ws = nullptr;
    const cudaError_t e = workspace_of_current_device(&ws);
    if (e != cudaSuccess || !ws) {
        snprintf(msg, sizeof(msg), "trident_search_noalloc: cudaGetSymbolAddress of the fixed workspace failed: %s",
                 cudaGetErrorString(e));
        return tb::record_error(TRIDENT_ERR_CUDA, msg);
    }
    return trident_search(idx, xq, B, K, nprobe, mode, ub_seed, ws, (size_t)TRIDENT_NOALLOC_WORKSPACE_BYTES, out_d,
                          out_i, stats, stream);
}

extern "C" size_t trident_noalloc_workspace_bytes(void) { return (size_t)TRIDENT_NOALLOC_WORKSPACE_BYTES; }
