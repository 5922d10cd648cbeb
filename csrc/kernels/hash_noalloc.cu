// ofld_hash_noalloc: the 128-bit content hash (ssh128) of a device buffer,
// computed without allocating any memory.
//
// This entry point has no counterpart in StateSpectre; it is an addition of
// this library.
//
// Who needs it. Some callers cannot call cudaMalloc (or anything that
// allocates) at the moment they need a checksum:
//   * code running inside a memory allocator's own hooks (a caching
//     allocator's alloc/free callback or an OOM handler), where allocating
//     would re-enter the allocator;
//   * inference servers and training frameworks that reserve all device
//     memory up front in their own pool, so a foreign cudaMalloc fails or
//     fragments the pool;
//   * latency-critical or real-time paths that cannot afford cudaMalloc's
//     implicit device-wide synchronization;
//   * crash and watchdog handlers that record the integrity of GPU state
//     while the process is already out of memory.
// The regular path (hash_device + fold_digests) needs a caller-provided
// digest buffer of 8 bytes per 64 KiB; this entry point keeps those digests in
// a fixed device array compiled into the library instead.
//
// Contract:
//   int ofld_hash_noalloc(const void* src, uint64_t nbytes, uint64_t* out, cudaStream_t stream)
//     src    device pointer to the bytes to hash (any alignment)
//     nbytes at most OFLD_NOALLOC_MAX_BYTES (8 GiB; ofld/hash_noalloc.h)
//     out    device pointer receiving two uint64 values {lo, hi}
//     stream the stream both kernels are enqueued on
//   returns 0 on success (the hash is in `out` once the stream reaches it), or
//     1  nbytes exceeds OFLD_NOALLOC_MAX_BYTES (nothing launched)
//     2  null src (with nbytes > 0) or null out (nothing launched)
//     3  the scratch array's address could not be obtained on this device
//     4  a kernel launch failed (cudaGetLastError holds the CUDA error)
//
// The scratch array. `g_digest_scratch` below is 1 MiB of device memory per
// GPU that loads this library, held until the process exits: 131072 chunk
// digests, hence the OFLD_NOALLOC_MAX_BYTES limit of 8 GiB. Host code cannot
// pass the array's name to a kernel (on the host the symbol is only a
// stand-in, not a device address), so the first call in each CUDA context
// (normally: on each device), with that device current, resolves the address
// with cudaGetSymbolAddress, checks the result and keeps it for later calls in
// the same context; make that first call before any stream capture. The
// address is keyed by the context's unique id, so a new context on the same
// device (after cudaDeviceReset, or a non-primary context) resolves it again
// instead of reusing a stale one. Every call shares the array and it keeps the
// last call's contents: calls that overlap on the GPU (different streams, or
// different host threads on the same device) race on it and must be ordered
// by the caller. Nothing in the array needs to start at zero: each call writes
// every digest it reads.
//
// The two kernels are the library's own hash and fold kernels; their output
// is identical to hash_device + fold_digests and to the host oracle.
#include "ofld/hash_noalloc.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "kernels.h"

namespace {

constexpr uint64_t kMaxDigests = (1ull << 20) / sizeof(uint64_t);  // 1 MiB of digests
static_assert(kMaxDigests * 65536ull == OFLD_NOALLOC_MAX_BYTES, "limit matches the array");

static __device__ __align__(256) uint64_t g_digest_scratch[kMaxDigests];

// Driver entry points for the current context's id (no link-time libcuda).
struct CtxApi {
    decltype(&cuCtxGetCurrent) get_current = nullptr;
    decltype(&cuCtxGetId) get_id = nullptr;
};

const CtxApi& ctx_api() {
    static CtxApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            api.get_current = reinterpret_cast<decltype(api.get_current)>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            api.get_id = reinterpret_cast<decltype(api.get_id)>(p);
    });
    return api;
}

// Unique id of the current context (0 when it cannot be read: no caching then).
unsigned long long current_ctx_id() {
    const CtxApi& api = ctx_api();
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!api.get_current || !api.get_id || api.get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (api.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

constexpr int kCacheEntries = 16;
struct CacheEntry {
    unsigned long long ctx_id = 0;
    uint64_t* addr = nullptr;
};
std::mutex g_mu;
CacheEntry g_cache[kCacheEntries];
int g_next = 0;

uint64_t* scratch_address() {
    const unsigned long long id = current_ctx_id();
    std::lock_guard<std::mutex> g(g_mu);
    if (id)
        for (const CacheEntry& e : g_cache)
            if (e.ctx_id == id) return e.addr;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_digest_scratch) != cudaSuccess || !p) return nullptr;
    if (id) {
        g_cache[g_next] = CacheEntry{id, static_cast<uint64_t*>(p)};
        g_next = (g_next + 1) % kCacheEntries;
    }
    return static_cast<uint64_t*>(p);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int ofld_hash_noalloc(const void* src, uint64_t nbytes,
                                                                        uint64_t* out, cudaStream_t stream) {
    if (nbytes > OFLD_NOALLOC_MAX_BYTES) return OFLD_NOALLOC_TOO_LARGE;
    if (!out || (nbytes > 0 && !src)) return OFLD_NOALLOC_NULL_ARG;
    uint64_t* scratch = scratch_address();
    if (!scratch) return OFLD_NOALLOC_NO_SCRATCH;
    const uint64_t nchunks = ofld::kern::digest_count(nbytes);
    if (nbytes > 0 && ofld::kern::hash_device(src, nbytes, scratch, stream, 0) != cudaSuccess)
        return OFLD_NOALLOC_LAUNCH;
    if (ofld::kern::fold_digests(scratch, nchunks, nbytes, out, stream) != cudaSuccess) return OFLD_NOALLOC_LAUNCH;
    return OFLD_NOALLOC_OK;
}
