#include "timing.h"

#include <atomic>
#include <map>
#include <mutex>

namespace ofld {
namespace kern {

namespace {

struct Ring {
    KernelStamp* host = nullptr;  // mapped pinned memory (device pointer is the same under UVA)
    KernelStamp* dev = nullptr;
    uint32_t capacity = 0;
    std::atomic<uint64_t> next{0};
};

std::mutex g_mu;
// Rings stay allocated until exit once created: a launch may still hold a
// record of a ring that timing_disable() detached.
std::map<int, Ring*> g_rings;
std::atomic<int> g_active{0};  // any device enabled (fast path for timing_take)

Ring* ring_of(int device) {
    auto it = g_rings.find(device);
    return it == g_rings.end() ? nullptr : it->second;
}

}  // namespace

const char* kernel_name(uint32_t id) {
    switch (id) {
        case kIdEvict: return "k1_evict";
        case kIdHash: return "k1_hash";
        case kIdRestore: return "k2_restore";
        case kIdEvictZ: return "k1_evict_zbf16";
        case kIdRestoreZ: return "k2_restore_zbf16";
        case kIdEvictJobs: return "k1_evict_jobs";
        case kIdRestoreJobs: return "k2_restore_jobs";
        case kIdZScan: return "zbf16_scan";
        case kIdZScanJobs: return "zbf16_scan_jobs";
        case kIdVerifyPeer: return "k3_verify_peer";
        case kIdPush: return "k4_push";
        case kIdEvictBulk: return "k1_evict_bulk";
        case kIdRestoreBulk: return "k2_restore_bulk";
        case kIdEvictZF32: return "k1_evict_zf32";
        case kIdRestoreZF32: return "k2_restore_zf32";
        case kIdZScanF32: return "zf32_scan";
        default: return "unknown";
    }
}

cudaError_t timing_enable(int device, uint32_t capacity) {
    if (capacity == 0) return cudaErrorInvalidValue;
    std::lock_guard<std::mutex> g(g_mu);
    Ring* r = ring_of(device);
    if (r && r->host && r->capacity == capacity) return cudaSuccess;
    const bool was_on = r && r->capacity;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return e;
    void* p = nullptr;
    e = cudaHostAlloc(&p, sizeof(KernelStamp) * capacity, cudaHostAllocMapped | cudaHostAllocPortable);
    void* d = nullptr;
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(&d, p, 0);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (p) cudaFreeHost(p);
        return e;
    }
    KernelStamp* h = static_cast<KernelStamp*>(p);
    for (uint32_t i = 0; i < capacity; ++i) h[i] = KernelStamp{~0ull, 0ull, 0, 0, 0xFFFFFFFFu};
    Ring* nr = new Ring;
    nr->host = h;
    nr->dev = static_cast<KernelStamp*>(d);
    nr->capacity = capacity;
    if (r) nr->next.store(r->next.load());  // sequence numbers continue
    g_rings[device] = nr;                   // an old ring is left allocated (see above)
    if (!was_on) g_active.fetch_add(1);
    return cudaSuccess;
}

void timing_disable(int device) {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_rings.find(device);
    if (it == g_rings.end() || !it->second->capacity) return;
    Ring* off = new Ring;
    off->next.store(it->second->next.load());
    it->second = off;  // capacity 0: takes return nullptr
    g_active.fetch_sub(1);
}

bool timing_enabled(int device) {
    std::lock_guard<std::mutex> g(g_mu);
    Ring* r = ring_of(device);
    return r && r->capacity;
}

KernelStamp* timing_take(uint32_t kernel, uint64_t bytes) {
    if (g_active.load(std::memory_order_relaxed) <= 0) return nullptr;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    Ring* r;
    {
        std::lock_guard<std::mutex> g(g_mu);
        r = ring_of(dev);
    }
    if (!r || !r->capacity) return nullptr;
    const uint64_t seq = r->next.fetch_add(1);
    const uint32_t i = uint32_t(seq % r->capacity);
    KernelStamp* h = r->host + i;
    h->t0 = ~0ull;
    h->t1 = 0;
    h->bytes = bytes;
    h->kernel = kernel;
    h->seq = uint32_t(seq);
    std::atomic_thread_fence(std::memory_order_seq_cst);  // the record is reset before the launch
    return r->dev + i;
}

std::vector<StampRecord> timing_read(int device, uint64_t since, uint64_t* next) {
    std::vector<StampRecord> out;
    Ring* r;
    {
        std::lock_guard<std::mutex> g(g_mu);
        r = ring_of(device);
    }
    if (!r) {
        if (next) *next = 0;
        return out;
    }
    const uint64_t end = r->next.load();
    if (next) *next = end;
    if (!r->capacity) return out;
    uint64_t s = since;
    if (end > r->capacity && s < end - r->capacity) s = end - r->capacity;
    for (uint64_t q = s; q < end; ++q) {
        const volatile KernelStamp& k = r->host[q % r->capacity];
        const uint64_t t0 = k.t0, t1 = k.t1;
        if (k.seq != uint32_t(q) || t1 == 0 || t0 == ~0ull || t1 < t0) continue;  // unfinished or reused
        out.push_back(StampRecord{q, k.bytes, t0, t1, k.kernel});
    }
    return out;
}

}  // namespace kern
}  // namespace ofld
