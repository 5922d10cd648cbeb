// Device-side kernel timing without a profiler.
//
// When timing is enabled for a device, every instrumented launch on it takes
// the next record of a ring in host-mapped pinned memory. Each CTA of the
// launch stamps the GPU's global nanosecond timer (%globaltimer) into the
// record at entry (atomic min) and exit (atomic max), so the record spans the
// first CTA start to the last CTA end: the kernel's device time, readable by
// the host with no copy and no event. The launcher fills in the kernel id
// and the bytes the launch moves, so bandwidth follows.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace ofld {
namespace kern {

struct KernelStamp {
    unsigned long long t0;  // earliest CTA entry (ns); ~0 until a CTA starts
    unsigned long long t1;  // latest CTA exit (ns); 0 until a CTA finishes
    uint64_t bytes;         // bytes the launch moves (set by the launcher;
                            // chunk-rounded for batch and K4 launches)
    uint32_t kernel;        // KernelId
    uint32_t seq;           // low bits of the launch's sequence number
};
static_assert(sizeof(KernelStamp) == 32, "KernelStamp is a 32-byte record");

enum KernelId : uint32_t {
    kIdEvict = 1,       // K1 (hash + copy to host)
    kIdHash = 2,        // K1 hash-only pass
    kIdRestore = 3,     // K2
    kIdEvictZ = 4,      // K1 with zbf16 coding
    kIdRestoreZ = 5,    // K2 with zbf16 decoding
    kIdEvictJobs = 6,   // K1 over a batch
    kIdRestoreJobs = 7, // K2 over a batch
    kIdZScan = 8,       // zbf16 pre-pass
    kIdZScanJobs = 9,   // zbf16 pre-pass over a batch
    kIdVerifyPeer = 10, // K3
    kIdPush = 11,       // K4
    kIdEvictBulk = 12,  // K1, bulk-copy form
    kIdRestoreBulk = 13,// K2, bulk-copy form
    kIdEvictZF32 = 14,  // K1 with zf32 coding
    kIdRestoreZF32 = 15,// K2 with zf32 decoding
    kIdZScanF32 = 16,   // zf32 pre-pass
    kIdCount
};
const char* kernel_name(uint32_t id);

struct StampRecord {
    uint64_t seq, bytes, t0, t1;
    uint32_t kernel;
};

// Ring of `capacity` records for launches on `device` (idempotent; a new
// capacity replaces the ring).
cudaError_t timing_enable(int device, uint32_t capacity);
void timing_disable(int device);
bool timing_enabled(int device);
// Record for a launch on the current device, or nullptr when timing is off.
KernelStamp* timing_take(uint32_t kernel, uint64_t bytes);
// Finished records with sequence number >= `since`, oldest first; `*next` is
// the sequence number the next launch will take. Records overwritten by the
// ring before they were read are skipped.
std::vector<StampRecord> timing_read(int device, uint64_t since, uint64_t* next);

#ifdef __CUDACC__
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Placed first in a kernel: stamps entry now and exit when the CTA's thread
// 0 leaves the kernel (on every return path).
struct StampScope {
    KernelStamp* ks;
    __device__ __forceinline__ explicit StampScope(KernelStamp* k) : ks(k) {
        if (ks && threadIdx.x == 0) atomicMin(&ks->t0, global_ns());
    }
    __device__ __forceinline__ ~StampScope() {
        if (ks && threadIdx.x == 0) atomicMax(&ks->t1, global_ns());
    }
};
#endif

}  // namespace kern
}  // namespace ofld
