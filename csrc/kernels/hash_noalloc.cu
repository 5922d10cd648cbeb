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
//     nbytes at most OFLD_NOALLOC_MAX_BYTES (8 GiB)
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
// digests, hence the 8 GiB limit. Host code cannot pass the array's name to a
// kernel (on the host the symbol is only a stand-in, not a device address), so
// the first call on each device, with that device current, resolves the
// address once with cudaGetSymbolAddress and caches it; make that first call
// before any stream capture. Every call shares the array and it keeps the last
// call's contents: calls that overlap on the GPU (different streams, or
// different host threads on the same device) race on it and must be ordered by
// the caller. Nothing in the array needs to start at zero: each call writes
// every digest it reads.
//
// The two kernels are the library's own hash and fold kernels; their output
// is identical to hash_device + fold_digests and to the host oracle.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "kernels.h"

namespace {

constexpr uint64_t kMaxDigests = (1ull << 20) / sizeof(uint64_t);  // 1 MiB of digests
constexpr uint64_t kMaxBytes = kMaxDigests * 65536ull;               // 8 GiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint64_t g_digest_scratch[kMaxDigests];

std::mutex g_mu;
uint64_t* g_scratch_addr[kMaxDevices] = {nullptr};

}  // namespace

extern "C" __attribute__((visibility("default"))) int ofld_hash_noalloc(const void* src, uint64_t nbytes,
                                                                        uint64_t* out, cudaStream_t stream) {
    if (nbytes > kMaxBytes) return 1;
    if (!out || (nbytes > 0 && !src)) return 2;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 3;
    uint64_t* scratch = nullptr;
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_digest_scratch) != cudaSuccess || !p) return 3;
            g_scratch_addr[dev] = static_cast<uint64_t*>(p);
        }
        scratch = g_scratch_addr[dev];
    }
    const uint64_t nchunks = ofld::kern::digest_count(nbytes);
    if (nbytes > 0 && ofld::kern::hash_device(src, nbytes, scratch, stream, 0) != cudaSuccess) return 4;
    if (ofld::kern::fold_digests(scratch, nchunks, nbytes, out, stream) != cudaSuccess) return 4;
    return 0;
}
