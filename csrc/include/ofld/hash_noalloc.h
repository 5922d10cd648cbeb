// Allocation-free content hash of a device buffer (ofld_hash_noalloc).
//
// This entry point has no counterpart in StateSpectre; it is an addition of
// this library, for callers that cannot allocate device memory at the moment
// they need a checksum (see csrc/kernels/hash_noalloc.cu for who they are and
// for the scratch array it uses instead).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

// Largest input: the library's fixed digest array holds 131072 chunk digests
// of 64 KiB each.
#define OFLD_NOALLOC_MAX_BYTES (8ull << 30)

// Return codes of ofld_hash_noalloc.
#define OFLD_NOALLOC_OK 0
#define OFLD_NOALLOC_TOO_LARGE 1   // nbytes > OFLD_NOALLOC_MAX_BYTES; nothing launched
#define OFLD_NOALLOC_NULL_ARG 2    // null src with nbytes > 0, or null out; nothing launched
#define OFLD_NOALLOC_NO_SCRATCH 3  // the scratch array's address is not available in this context
#define OFLD_NOALLOC_LAUNCH 4      // a kernel launch failed (cudaGetLastError holds the error)

#ifdef __cplusplus
extern "C" {
#endif

// ssh128 of nbytes at src (device memory, any alignment) into out[0..1]
// (device memory, {lo, hi}), enqueued on `stream`. Allocates nothing.
int ofld_hash_noalloc(const void* src, uint64_t nbytes, uint64_t* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
