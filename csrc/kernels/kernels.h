// Host-side launchers of the sm_100a data-path kernels.
//
//   evict_hash      K1: device -> host-mapped pinned copy, ssh128 chunk digests
//                       computed from the same registers in the same pass.
//   restore_cast    K2: host-mapped pinned -> device copy with optional digest
//                       re-verification and an optional cast (bf16 -> fp8 e4m3
//                       with one fp32 scale per 128 elements, fp32 -> bf16,
//                       bf16 -> fp32).
//   hash_device         ssh128 chunk digests of a device buffer at HBM rate
//                       (the K4 bulk-copy pipeline for aligned buffers).
//   verify_peer     K3: digests of a local buffer plus an exact byte compare
//                       against a peer GPU's replica read over NVLink.
//   quant_fp8_block     standalone 1x128 block quantization (used by the
//                       weight-sync push and tests).
//
// Every launcher takes explicit (pointer, nbytes) and validates alignment and
// bounds on the host before launching; nothing is launched on bad arguments.
// All launches go on the caller's stream; none allocate memory.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace ofld {
namespace kern {

enum class Cast : int {
    kNone = 0,
    kBf16ToFp8Block128 = 1,  // out: fp8 e4m3 bytes (n elems) + fp32 scales (n/128)
    kFp32ToBf16 = 2,
    kBf16ToFp32 = 3,
};

struct LaunchCfg {
    int ctas = 0;        // 0 = launcher default
    int priority = 0;    // informational
};

// Launch counter for every kernel of this library (what bench.py reports as
// gpu_launches). Monotonic per process.
uint64_t launch_count();

// K1. `digests` (may be null) receives ceil(nbytes/64KiB) chunk digests and
// must be device-accessible (device or host-mapped memory).
cudaError_t evict_hash(const void* src_dev, void* dst_mapped, uint64_t nbytes, uint64_t* digests,
                       cudaStream_t stream, int ctas);

// K2. `expect` (may be null): chunk digests to verify against; mismatches are
// counted into *mismatch_dev (device-accessible u32, may be null).
cudaError_t restore_cast(const void* src_mapped, void* dst_dev, uint64_t src_nbytes, Cast cast,
                         float* scales_dev, const uint64_t* expect, uint32_t* mismatch_dev,
                         cudaStream_t stream, int ctas);

cudaError_t hash_device(const void* src_dev, uint64_t nbytes, uint64_t* digests, cudaStream_t stream, int ctas);
// The one-pass hash kernel (per-thread loads, any alignment): hash_device's
// form for unaligned buffers, and an independent second implementation.
cudaError_t hash_onepass(const void* src_dev, uint64_t nbytes, uint64_t* digests, cudaStream_t stream, int ctas);

// Fold chunk digests into the 128-bit object hash on the device (single CTA);
// `out` receives {lo, hi}.
cudaError_t fold_digests(const uint64_t* digests, uint64_t nchunks, uint64_t nbytes, uint64_t* out,
                         cudaStream_t stream);

// K3. Compares local and peer bytes; *mismatch_dev counts differing 16-byte
// vectors. Digests of the local buffer are produced in the same pass.
cudaError_t verify_peer(const void* local_dev, const void* peer_dev, uint64_t nbytes, uint64_t* digests,
                        uint32_t* mismatch_dev, cudaStream_t stream, int ctas);

cudaError_t quant_fp8_block(const void* bf16_src, void* fp8_dst, float* scales, uint64_t nelem,
                            cudaStream_t stream, int ctas);

// zbf16 coding of bf16 objects for host transfers (format: ofld/zbf16.h).
// zscan: per-chunk window base into `ebase` (device-accessible, one byte per
// 64 KiB chunk) and *fail |= 1 when some chunk does not fit coded (then the
// object must move uncoded). evict_z / restore_z: K1 / K2 over a coded run;
// all require zbf16::eligible(nbytes) and 16-byte aligned pointers. restore_z
// supports Cast::kNone, kBf16ToFp8Block128 and kBf16ToFp32.
// `max_coded` (device-accessible, kZScanSlots u32 slots, may be null; the
// caller zeroes it): each CTA stores the largest stored length of the chunks
// it scanned in its own slot (the grid is at most kZScanSlots CTAs then); the
// maximum over the slots is what a strided copy of the coded run must move
// per 64 KiB row.
constexpr int kZScanSlots = 512;
cudaError_t zscan(const void* src_dev, uint64_t nbytes, uint8_t* ebase, uint32_t* fail, cudaStream_t stream,
                  int ctas, uint32_t* max_coded = nullptr);
cudaError_t evict_z(const void* src_dev, void* dst_mapped, uint64_t nbytes, const uint8_t* ebase,
                    uint64_t* digests, cudaStream_t stream, int ctas);
cudaError_t restore_z(const void* src_mapped, void* dst_dev, uint64_t nbytes, Cast cast, float* scales_dev,
                      const uint64_t* expect, uint32_t* mismatch_dev, cudaStream_t stream, int ctas);

// zf32 coding of fp32 objects (format: ofld/zbf16.h, namespace zf32): the
// same three passes over whole 128 KiB rows (zf32::eligible(nbytes), 16-byte
// aligned pointers). zscan_f32 writes one window base per row and, like
// zscan, the per-CTA largest stored length of the rows' coded top halves
// (what a strided copy moves per row beyond the 64 KiB low plane).
// evict_zf32 computes no digests (hash the fp32 bytes with hash_device);
// restore_zf32 has no cast or verification (compare_digests after a
// hash_device of the result verifies).
cudaError_t zscan_f32(const void* src_dev, uint64_t nbytes, uint8_t* ebase, uint32_t* fail, cudaStream_t stream,
                      int ctas, uint32_t* max_coded = nullptr);
cudaError_t evict_zf32(const void* src_dev, void* dst, uint64_t nbytes, const uint8_t* ebase, cudaStream_t stream,
                       int ctas);
cudaError_t restore_zf32(const void* src, void* dst_dev, uint64_t nbytes, cudaStream_t stream, int ctas);
// *mismatch (device-accessible) += the number of i < n with got[i] != expect[i].
cudaError_t compare_digests(const uint64_t* got, const uint64_t* expect, uint64_t n, uint32_t* mismatch,
                            cudaStream_t stream);

// Batched K1/K2: one launch moves every item of a batch (KV-cache blocks).
// Jobs are 64-byte records sorted by chunk_begin (the global index of the
// job's first 64 KiB chunk; total_chunks covers them all), in
// device-accessible memory. src/dst 16-byte aligned, nbytes % 16 == 0.
//   evict:   src = device, dst = host-mapped run; ebase non-null = code the
//            job in zbf16 with those window bases; digests (may be null)
//   restore: src = host-mapped run, dst = device; coded != 0 = zbf16 run
struct XferJob {
    const void* src;
    void* dst;
    uint64_t nbytes;
    uint64_t chunk_begin;
    const uint8_t* ebase;
    uint64_t* digests;
    uint32_t coded;
    uint32_t pad0;
    uint64_t pad1;
};
static_assert(sizeof(XferJob) == 64, "XferJob is a 64-byte record");
// zbf16 pre-pass over a batch: per job, `dst` receives one window base per
// chunk followed, at the next 16-byte boundary, by a u32 fail word (set to 1
// when a chunk does not fit coded; the caller zeroes it). Every src 16-byte
// aligned and zbf16-eligible in size.
cudaError_t zscan_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t stream, int ctas);
cudaError_t evict_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t stream, int ctas);
cudaError_t restore_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t stream, int ctas);

// Number of chunk digests for nbytes.
inline uint64_t digest_count(uint64_t nbytes) { return (nbytes + 65535) / 65536; }

// K4 work item (64 bytes, laid out for a host-packed table). `chunk_begin` is
// the global index of the item's first 64 KiB chunk; items are sorted by it
// and item i owns chunks [chunk_begin_i, chunk_begin_i + ceil(nbytes/64KiB)).
// nbytes is a multiple of 16 (a multiple of 256 for kPushFp8).
//   mode kPushRaw   copy the bytes to `dst`
//        kPushFp8   bf16 source; write fp8 e4m3 bytes to `dst` and one fp32
//                   scale (amax/448) per 128 elements to `dst_scales`
//        kPushHash  digests only, nothing is stored
//   flags kPushDelta  skip the stores of a chunk whose new digest equals the
//                     digest already in the launch's `digests` table (the
//                     table describes what the destination holds)
//         kPushMulticast  `dst` / `dst_scales` are addresses in a multicast
//                     team mapping: stores are `multimem.st`, so the NVSwitch
//                     writes every member's buffer
// Without kPushMulticast, `dst` / `dst_scales` are typically peer-GPU
// pointers (CUDA IPC or VMM mappings).
//        kPushBulk  copy each staged half-chunk to `dst` with one bulk store
//                   (cp.async.bulk shared -> global, no multicast); `dst` is
//                   this GPU's memory or host-mapped pinned memory, never a
//                   peer. The evict / restore bulk forms (evict_bulk,
//                   restore_bulk) are one-item launches of this mode.
//   flags kPushNoHash  skip the ssh128 lane work and the digest write (a
//                     plain copy; only with kPushBulk)
enum : uint32_t { kPushRaw = 0, kPushFp8 = 1, kPushHash = 2, kPushBulk = 3 };
enum : uint32_t { kPushDelta = 1u << 0, kPushMulticast = 1u << 1, kPushNoHash = 1u << 2 };
// launch_flags only: four staged halves per CTA (128 KiB in flight, one CTA
// per SM) instead of two; the bulk forms use it for host-mapped traffic.
enum : uint32_t { kPushDeep = 1u << 8 };
// `digest_base` is the index of the item's first chunk in the launch's digest
// table (equal to chunk_begin for a full table; a subset launch keeps the
// full table's indices so the record of what the destination holds stays put).
struct PushItem {
    const void* src;
    void* dst;
    float* dst_scales;
    uint64_t nbytes;
    uint64_t chunk_begin;
    uint32_t mode;
    uint32_t flags;
    uint64_t digest_base;
    uint64_t reserved;
};
static_assert(sizeof(PushItem) == 64, "PushItem is a 64-byte record");

// Per-launch device state of K4 (all device-accessible memory).
//   digests     [total_chunks] u64, in/out: one ssh128 chunk digest per chunk
//   item_hash   [2*nitems] u64 out (may be null): 128-bit object hash per
//               item, folded by a second small launch on the same stream
//   stats       [2] u64 accumulated (may be null): chunks stored, bytes stored
//   error       u32 (may be null): 0, or the first bounded wait that expired
//               (1 chunk never arrived in shared memory, 2 stage never freed)
struct PushState {
    uint64_t* digests;
    uint64_t* item_hash;
    unsigned long long* stats;
    uint32_t* error;
};

// K4. One persistent grid over every chunk of every item (+ the item-hash
// fold when `item_hash` is set). `launch_flags` & kPushDelta must be set when
// any item carries kPushDelta (it selects the block shape that holds stages
// across the store decision).
cudaError_t push(const PushItem* items_dev, int nitems, uint64_t total_chunks, PushState st, cudaStream_t s,
                 int ctas, uint32_t launch_flags);

// Chunk digests of a device buffer through the K4 pipeline (bulk copies into
// shared memory, three CTAs per SM). src 16-byte aligned, nbytes % 16 == 0.
// `stages` picks the block shape: 2 (three CTAs per SM, 64 KiB staged each),
// 3 (two per SM) or 4 (one per SM, 128 KiB); 0 = the measured default.
cudaError_t hash_stream(const void* src_dev, uint64_t nbytes, uint64_t* digests, uint32_t* error, cudaStream_t s,
                        int ctas, int stages = 0);

// K1 / K2 bulk forms: the bytes cross PCIe as bulk copies issued by one
// thread per CTA (host-mapped source or destination <-> shared memory), with
// the ssh128 chunk digests of the evicted bytes computed from shared memory in
// the same pass (`digests` null: no hash). src, dst 16-byte aligned,
// nbytes % 16 == 0. `error` (device-accessible u32, may be null) receives a
// non-zero code when a bounded wait inside the kernel ran out (the copy is
// then incomplete). ctas = 0: the default for host-mapped traffic.
cudaError_t evict_bulk(const void* src_dev, void* dst_mapped, uint64_t nbytes, uint64_t* digests, uint32_t* error,
                       cudaStream_t s, int ctas);
cudaError_t restore_bulk(const void* src_mapped, void* dst_dev, uint64_t nbytes, uint32_t* error, cudaStream_t s,
                         int ctas);
// Whether the bulk forms take these arguments (alignment and size rules).
inline bool bulk_ok(const void* a, const void* b, uint64_t nbytes) {
    return nbytes > 0 && (nbytes & 15) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(b) & 15) == 0;
}

// Dynamic shared memory of one delta-mode K4 CTA (three 32 KiB half-chunk
// stages + barriers).
size_t push_smem_bytes();
uint64_t push_launch_count();

}  // namespace kern
}  // namespace ofld
