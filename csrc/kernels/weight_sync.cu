// K4: in-box weight-sync push (trainer GPU -> rollout GPU over NVLink), and
// the HBM-rate chunk-digest pass built on the same pipeline.
//
// StateSpectre moves a new model version to rollout engines by staging every
// object on the host and sending it over TCP (reference:
// src/daemon/canonical_rollout.cpp:240-411, python_api/state_spectre/_rollout.py:101-175).
// Inside one B200 node the rollout GPUs are NVLink peers, so the trainer
// pushes the changed tensors of a sealed version directly into the rollout's
// weight buffers:
//
//   * one persistent launch (two or three CTAs per SM) walks a work list of
//     (src, dst) items 64 KiB chunk by chunk, so a version with hundreds of
//     changed tensors is one launch;
//   * in each CTA a producer warp streams 32 KiB half-chunks HBM -> shared
//     memory with 1-D bulk copies (cp.async.bulk, completion on an mbarrier)
//     ahead of the consumers, so loads stay in flight while they hash;
//   * the 256 consumer threads compute the chunk's ssh128 digest from shared
//     memory, compare it with what the destination already holds (delta mode)
//     and store the chunk to the peer: raw bytes, or bf16 quantized to fp8
//     e4m3 with one fp32 scale per 128 elements;
//   * a second small launch folds every item's 128-bit object hash (manifest
//     content hash) from the chunk digests.
//
// Peer memory is only ever the target of plain st.global (or, through a
// multicast team mapping, multimem.st) from registers; the bulk copies read
// this GPU's own memory and carry no multicast qualifier.
// Every mbarrier wait is bounded (about two seconds of SM clock); on expiry the
// kernel records an error code in PushState::error and returns.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <atomic>

#include "kernels.h"
#include "timing.h"
#include "ofld/chunk_hash.h"

namespace ofld {
namespace kern {

namespace {

// Block layout: one consumer group of 256 threads (one ssh128 lane per
// thread) and one producer warp. Each CTA owns its stage ring: every use of a
// stage is consumed by the same in-order group, so a waiter is never more than
// one phase ahead of a barrier and the parity waits cannot alias. (Several
// consumer groups sharing one ring break that: a stage's previous use can
// belong to another group whose copy has not landed, its barrier is then two
// phases behind, the parity test passes early, and the CTA can retire with
// bulk copies still writing its shared memory.) Parallelism per SM comes from
// several resident CTAs instead.
constexpr int kGroupThreads = 256;
constexpr int kGroupWarps = kGroupThreads / 32;
constexpr int kThreads = kGroupThreads + 32;
// A 64 KiB hash chunk is staged as two 32 KiB halves: lane t's vectors
// k*256+t for k < 8 lie in the first half, so the lane state carries over.
constexpr uint32_t kChunk = ssh::kChunkBytes;
constexpr uint32_t kHalf = kChunk / 2;
constexpr int kHalfVecs = ssh::kVecsPerLane / 2;  // 8 vectors per lane per half
constexpr uint32_t kPiece = 16384;               // bytes per bulk copy instruction
constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at 2 GHz

template <int S>
constexpr size_t smem_bytes() {
    return size_t(S) * kHalf + 2 * S * 8 + kGroupWarps * 8 + 16;
}
// S = 2 half-stages: three CTAs per SM (hash-only and non-delta pushes);
// S = 3: two CTAs per SM, one half prefetched while a delta chunk is held;
// S = 4: one CTA per SM with 128 KiB in flight (host-mapped bulk transfers,
// where a few dozen CTAs must cover PCIe latency).
static_assert(3 * (smem_bytes<2>() + 1024) <= 233472, "three S=2 CTAs must fit one SM");
static_assert(2 * (smem_bytes<3>() + 1024) <= 233472, "two S=3 CTAs must fit one SM");
static_assert(smem_bytes<4>() + 1024 <= 233472, "an S=4 CTA must fit one SM");

// Error codes written to PushState::error (first writer wins).
constexpr uint32_t kErrFullTimeout = 1;
constexpr uint32_t kErrEmptyTimeout = 2;
constexpr uint32_t kErrBadItem = 3;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false when the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}

__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk store of a staged half: shared memory -> global (this GPU's memory or
// host-mapped pinned memory), tracked by the issuing thread's bulk groups.
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src_smem),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The stage may be refilled once every issued bulk store finished reading it.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every issued bulk store complete (its writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint4 ld_smem(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ void st_peer(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ void st_peer8(void* p, uint2 v) {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// Stores through a multicast team mapping: one instruction, the NVSwitch
// writes the bytes to every member GPU. The .f32 type only names the 32-bit
// lanes; a store does no arithmetic, so every bit pattern arrives unchanged.
__device__ __forceinline__ void st_multi(void* p, uint4 v) {
    asm volatile("multimem.st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_multi8(void* p, uint2 v) {
    asm volatile("multimem.st.global.v2.f32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

__device__ __forceinline__ void st_multi4(void* p, float v) {
    asm volatile("multimem.st.global.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ void group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "n"(kGroupThreads) : "memory");
}

__device__ __forceinline__ float lo16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_fp8(float a, float b, float c, float d) {
    return uint32_t(__nv_cvt_float_to_fp8(a, __NV_SATFINITE, __NV_E4M3)) |
           (uint32_t(__nv_cvt_float_to_fp8(b, __NV_SATFINITE, __NV_E4M3)) << 8) |
           (uint32_t(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3)) << 16) |
           (uint32_t(__nv_cvt_float_to_fp8(d, __NV_SATFINITE, __NV_E4M3)) << 24);
}

// Items are sorted by chunk_begin and every CTA visits its chunks in
// increasing order, so the owning item only ever advances.
__device__ __forceinline__ void advance_item(const PushItem* items, int nitems, uint64_t c, int& idx) {
    if (!items) return;
    while (idx + 1 < nitems && items[idx + 1].chunk_begin <= c) ++idx;
}

__device__ __forceinline__ uint32_t chunk_len(const PushItem& it, uint64_t c) {
    const uint64_t base = (c - it.chunk_begin) * kChunk;
    return uint32_t(it.nbytes - base < kChunk ? it.nbytes - base : kChunk);
}

// Store one 16-byte source vector (8 bf16 values for fp8) of the chunk at
// byte `base` of the item. Every lane of the warp calls this together (the
// fp8 block amax is a half-warp reduction); `valid` masks the ragged tail.
__device__ __forceinline__ void store_vec(const PushItem& it, uint64_t base, uint32_t vi, uint4 v, bool valid) {
    const bool multi = (it.flags & kPushMulticast) != 0;
    if (it.mode == kPushRaw) {
        uint8_t* p = static_cast<uint8_t*>(it.dst) + base + size_t(vi) * 16;
        if (valid) {
            if (multi)
                st_multi(p, v);
            else
                st_peer(p, v);
        }
        return;
    }
    // 16 consecutive lanes hold one 128-element block (chunk bases are block aligned)
    const float f[8] = {lo16(v.x), hi16(v.x), lo16(v.y), hi16(v.y), lo16(v.z), hi16(v.z), lo16(v.w), hi16(v.w)};
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, valid ? fabsf(f[e]) : 0.f);
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 448.f / amax : 1.f;
    if (valid) {
        const uint64_t elem = base / 2 + uint64_t(vi) * 8;
        const uint2 q = make_uint2(pack_fp8(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv),
                                   pack_fp8(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv));
        const float scale = amax > 0.f ? amax / 448.f : 1.f;
        if (multi) {
            st_multi8(static_cast<uint8_t*>(it.dst) + elem, q);
            if ((threadIdx.x & 15) == 0) st_multi4(it.dst_scales + elem / 128, scale);
        } else {
            st_peer8(static_cast<uint8_t*>(it.dst) + elem, q);
            if ((threadIdx.x & 15) == 0) it.dst_scales[elem / 128] = scale;
        }
    }
}

// Group-level tree fold of the 256 lane digests; the root is valid in the
// group's thread 0.
__device__ __forceinline__ uint64_t chunk_tree(uint64_t d, uint64_t* red, int g, uint32_t lt) {
    const uint32_t lane = lt & 31, warp = lt >> 5;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const uint64_t o = __shfl_down_sync(0xffffffffu, d, s);
        if ((lane & (2 * s - 1)) == 0) d = ssh::fold(d, o);
    }
    if (lane == 0) red[warp] = d;
    group_sync(g);
    uint64_t root = 0;
    if (lt == 0) {
        uint64_t x[kGroupWarps];
#pragma unroll
        for (int i = 0; i < kGroupWarps; ++i) x[i] = red[i];
#pragma unroll
        for (int s = 1; s < kGroupWarps; s <<= 1)
#pragma unroll
            for (int i = 0; i < kGroupWarps; i += 2 * s) x[i] = ssh::fold(x[i], x[i + s]);
        root = x[0];
    }
    return root;
}

// Object fold of one item's chunk digests by one warp: the absorb chain is
// sequential, so the warp prefetches the next 32 digests (L2 loads, written by
// other CTAs before their release fence) while it absorbs the current 32 from
// registers; every lane carries the same state.
__device__ __forceinline__ void fold_item_warp(const PushItem& it, int idx, const PushState& st) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t n = ssh::num_chunks_dev(it.nbytes);
    const uint64_t* d = st.digests + it.digest_base;
    uint64_t lo, hi;
    ssh::object_init(lo, hi);
    uint64_t cur = lane < n ? __ldcg(d + lane) : 0;
    for (uint64_t b = 0; b < n; b += 32) {
        const uint64_t nb = b + 32 + lane;
        const uint64_t next = nb < n ? __ldcg(d + nb) : 0;
        const uint32_t cnt = uint32_t(n - b < 32 ? n - b : 32);
        for (uint32_t j = 0; j < cnt; ++j) ssh::object_absorb(lo, hi, __shfl_sync(0xffffffffu, cur, j));
        cur = next;
    }
    if (lane == 0) {
        const ssh::Object o = ssh::object_finish(lo, hi, it.nbytes);
        st.item_hash[2 * idx] = o.lo;
        st.item_hash[2 * idx + 1] = o.hi;
    }
}

__device__ __forceinline__ void set_error(const PushState& st, uint32_t code) {
    if (st.error) atomicCAS(st.error, 0u, code);
}

template <int S>
__global__ void __launch_bounds__(kThreads, (S == 2 ? 3 : S == 3 ? 2 : 1))
    k_push(const PushItem* __restrict__ items, int nitems, uint64_t total_chunks, PushState st, PushItem one, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    // `items == nullptr`: a single item passed by value (no device table)
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(S) * kHalf);
    uint64_t* empty = full + S;
    uint64_t* red = empty + S;
    // [0] store decision of the current chunk, [1] the group gives up (both
    // written only before a group barrier, so every consumer reads one value)
    volatile int* flags = reinterpret_cast<volatile int*>(red + kGroupWarps);
    const uint32_t stage0 = smem_u32(smem);

    const uint32_t t = threadIdx.x;
    if (t == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGroupWarps);
        }
        flags[0] = 0;
        flags[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (t >= kGroupThreads) {
        // ---- producer warp: one lane issues the bulk copies, two halves per chunk ----
        if (t != kGroupThreads) return;
        int idx = 0;
        uint32_t q = 0;
        for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
            advance_item(items, nitems, c, idx);
            const PushItem it = items ? items[idx] : one;
            const uint64_t off_in_item = (c - it.chunk_begin) * kChunk;
            const uint8_t* src = static_cast<const uint8_t*>(it.src) + off_in_item;
            // Self-check before the copy engine sees the address: an item that
            // does not own chunk c, or a source that is not 16-byte aligned,
            // is recorded and ends the launch without issuing the copy.
            if (c < it.chunk_begin || off_in_item >= it.nbytes || (reinterpret_cast<uintptr_t>(src) & 15) ||
                (it.nbytes & 15) || (it.mode == kPushBulk && (reinterpret_cast<uintptr_t>(it.dst) & 15))) {
                set_error(st, kErrBadItem);
                return;  // the consumers' bounded waits on the stages never filled end the launch
            }
            const uint32_t len = chunk_len(it, c);
            for (uint32_t h = 0; h < 2; ++h, ++q) {
                const int s = int(q % S);
                if (q >= uint32_t(S) && !mbar_wait(&empty[s], ((q / S) - 1) & 1)) {
                    set_error(st, kErrEmptyTimeout);
                    return;
                }
                if (flags[1]) return;
                const uint32_t lo = h * kHalf;
                const uint32_t bytes = len > lo ? (len - lo < kHalf ? len - lo : kHalf) : 0;
                mbar_expect_tx(&full[s], bytes);  // 0 bytes: the phase completes on this arrival
                for (uint32_t off = 0; off < bytes; off += kPiece)
                    bulk_g2s(smem + size_t(s) * kHalf + off, src + lo + off, bytes - off < kPiece ? bytes - off : kPiece,
                             &full[s]);
            }
        }
        return;
    }

    // ---- consumer group ----
    const uint32_t lt = t;
    int idx = 0;
    uint32_t i = 0;
    bool aborted = false, stored_any = false, bulk_any = false;
    for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x, ++i) {
        advance_item(items, nitems, c, idx);
        const PushItem it = items ? items[idx] : one;
        const uint64_t base = (c - it.chunk_begin) * kChunk;
        const uint32_t len = chunk_len(it, c);
        const uint32_t nvec = len / 16;  // the launcher guarantees nbytes % 16 == 0
        const bool bulk = it.mode == kPushBulk;
        const bool nohash = bulk && (it.flags & kPushNoHash) != 0;
        const bool delta = !bulk && (it.flags & kPushDelta) != 0;
        // stores need no digest: issue from the same registers
        const bool store_now = !delta && it.mode != kPushHash && !bulk;
        const bool hold = delta && it.mode != kPushHash;  // stages kept until the store decision
        // the destination's digest of this chunk, loaded now and used after the hash
        const uint64_t dgi = it.digest_base + (c - it.chunk_begin);
        const uint64_t old_dg = (delta && lt == 0) ? st.digests[dgi] : 0;
        ssh::Lane L = ssh::lane_init(lt);
        for (uint32_t h = 0; h < 2; ++h) {
            const uint32_t q = 2 * i + h;
            const int s = int(q % S);
            if (!mbar_wait(&full[s], (q / S) & 1)) {
                set_error(st, kErrFullTimeout);
                flags[1] = 1;
            }
            group_sync(0);
            if (flags[1]) {
                aborted = true;
                break;
            }
            const uint32_t sb = stage0 + uint32_t(s) * kHalf;
            if (bulk && lt == 0) {
                // one thread hands the staged half to the bulk-copy unit; the
                // group hashes the same shared memory meanwhile
                const uint32_t lo = h * kHalf;
                const uint32_t bytes = len > lo ? (len - lo < kHalf ? len - lo : kHalf) : 0;
                if (bytes) {
                    fence_proxy_async_smem();
                    bulk_s2g(static_cast<uint8_t*>(it.dst) + base + lo, sb, bytes);
                    bulk_commit();
                    bulk_any = true;
                }
            }
            if (nohash) {
            } else if (len == kChunk) {
#pragma unroll
                for (int kk = 0; kk < kHalfVecs; ++kk) {
                    const uint4 v = ld_smem(sb + (uint32_t(kk) * kGroupThreads + lt) * 16);
                    ssh::lane_update(L, v.x, v.y, v.z, v.w);
                    if (store_now) store_vec(it, base, (h * kHalfVecs + kk) * kGroupThreads + lt, v, true);
                }
            } else {
#pragma unroll
                for (int kk = 0; kk < kHalfVecs; ++kk) {
                    const uint32_t vi = (h * kHalfVecs + kk) * kGroupThreads + lt;
                    const bool valid = vi < nvec;
                    const uint4 v = valid ? ld_smem(sb + (uint32_t(kk) * kGroupThreads + lt) * 16)
                                          : make_uint4(0, 0, 0, 0);
                    if (valid) ssh::lane_update(L, v.x, v.y, v.z, v.w);
                    if (store_now) store_vec(it, base, vi, v, valid);
                }
            }
            if (!hold) {
                if (bulk && lt == 0) bulk_wait_read_all();  // the stage's bulk store has read it
                __syncwarp();
                if ((lt & 31) == 0) mbar_arrive(&empty[s]);
            }
        }
        if (aborted) break;
        stored_any |= store_now;
        const uint64_t root = nohash ? 0 : chunk_tree(ssh::lane_digest(L, lt), red, 0, lt);
        if (lt == 0) {
            const uint64_t dg = nohash ? 0 : ssh::chunk_finish(root, len);
            const bool same = delta && old_dg == dg;
            if (!nohash) st.digests[dgi] = dg;
            const bool stored = it.mode != kPushHash && !same;
            flags[0] = hold && stored;
            if (stored && st.stats) {
                atomicAdd(&st.stats[0], 1ull);
                atomicAdd(&st.stats[1], (unsigned long long)len);
            }
        }
        group_sync(0);
        if (hold) {
            const bool do_store = flags[0] != 0;
            stored_any |= do_store;
            for (uint32_t h = 0; h < 2; ++h) {
                const uint32_t q = 2 * i + h;
                const int s = int(q % S);
                if (do_store) {
                    const uint32_t sb = stage0 + uint32_t(s) * kHalf;
#pragma unroll
                    for (int kk = 0; kk < kHalfVecs; ++kk) {
                        const uint32_t vi = (h * kHalfVecs + kk) * kGroupThreads + lt;
                        const bool valid = vi < nvec;
                        const uint4 v = valid ? ld_smem(sb + (uint32_t(kk) * kGroupThreads + lt) * 16)
                                              : make_uint4(0, 0, 0, 0);
                        store_vec(it, base, vi, v, valid);
                    }
                }
                __syncwarp();
                if ((lt & 31) == 0) mbar_arrive(&empty[s]);
            }
        }
    }
    // Peer stores are posted writes: make them visible system-wide before the
    // grid completes, so a host-side signal after the stream sync is safe.
    if (stored_any) __threadfence_system();
    // Bulk stores read this CTA's shared memory and write asynchronously:
    // wait for all of them before the CTA retires.
    if (bulk_any) {
        bulk_wait_all();
        __threadfence_system();
    }
    // Do not leave with bulk copies still writing this CTA's shared memory:
    // after an abort give the stages the producer may have filled a bounded
    // chance to complete.
    if (aborted && lt == 0) {
        const uint32_t q0 = 2 * i;
        for (uint32_t q = q0; q < q0 + S; ++q) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[q % S], (q / S) & 1) && clock64() - t0 < kWaitCycles / 8) {
            }
        }
    }
}

// Item hashes: one warp per item folds the chunk digests the push kernel
// wrote (stream order makes them visible; no fences in the push itself).
__global__ void __launch_bounds__(256) k_fold_items(const PushItem* __restrict__ items, int nitems, PushState st,
                                                    PushItem one) {
    const int idx = int(blockIdx.x) * 8 + int(threadIdx.x >> 5);
    if (idx >= nitems) return;
    const PushItem it = items ? items[idx] : one;
    fold_item_warp(it, idx, st);
}

std::atomic<uint64_t> g_push_launches{0};

}  // namespace

size_t push_smem_bytes() { return smem_bytes<3>(); }

namespace {
template <int S>
cudaError_t launch_stages(const PushItem* items_dev, int nitems, uint64_t total_chunks, const PushState& st,
                          const PushItem& one, cudaStream_t s, int ctas, uint32_t stamp_id = kIdPush) {
    static thread_local int configured_device = -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (configured_device != dev) {
        e = cudaFuncSetAttribute(k_push<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_bytes<S>()));
        if (e != cudaSuccess) return e;
        configured_device = dev;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int g = ctas > 0 ? ctas : sms * (S == 2 ? 3 : S == 3 ? 2 : 1);  // persistent: every resident slot
    if (uint64_t(g) > total_chunks) g = int(total_chunks);
    // bytes: one-item launches move exactly the item; tables are chunk-rounded
    KernelStamp* ks = timing_take(stamp_id, items_dev ? total_chunks * kChunk : one.nbytes);
    k_push<S><<<g, kThreads, smem_bytes<S>(), s>>>(items_dev, nitems, total_chunks, st, one, ks);
    g_push_launches.fetch_add(1, std::memory_order_relaxed);
    e = cudaGetLastError();
    if (e != cudaSuccess || !st.item_hash) return e;
    k_fold_items<<<(nitems + 7) / 8, 256, 0, s>>>(items_dev, nitems, st, one);
    g_push_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}
}  // namespace

cudaError_t push(const PushItem* items_dev, int nitems, uint64_t total_chunks, PushState st, cudaStream_t s,
                 int ctas, uint32_t launch_flags) {
    if (nitems <= 0 || total_chunks == 0) return cudaSuccess;
    if (!items_dev || !st.digests) return cudaErrorInvalidValue;
    if (launch_flags & kPushDelta) return launch_stages<3>(items_dev, nitems, total_chunks, st, PushItem{}, s, ctas);
    return launch_stages<2>(items_dev, nitems, total_chunks, st, PushItem{}, s, ctas);
}

// Block shape of the standalone hash (see hash_stream).
constexpr int kHashStages = 3;

cudaError_t hash_stream(const void* src_dev, uint64_t nbytes, uint64_t* digests, uint32_t* error, cudaStream_t s,
                        int ctas, int stages) {
    if (nbytes == 0) return cudaSuccess;
    if (!src_dev || !digests || (reinterpret_cast<uintptr_t>(src_dev) & 15) || (nbytes & 15))
        return cudaErrorInvalidValue;
    PushItem one{};
    one.src = src_dev;
    one.nbytes = nbytes;
    one.mode = kPushHash;
    PushState st{digests, nullptr, nullptr, error};
    const uint64_t nch = ssh::num_chunks(nbytes);
    if (stages == 0) stages = kHashStages;
    if (stages == 4) return launch_stages<4>(nullptr, 1, nch, st, one, s, ctas, kIdHash);
    if (stages == 3) return launch_stages<3>(nullptr, 1, nch, st, one, s, ctas, kIdHash);
    if (stages == 2) return launch_stages<2>(nullptr, 1, nch, st, one, s, ctas, kIdHash);
    return cudaErrorInvalidValue;
}

// Default grid of the bulk forms: PCIe Gen5 x16 carries ~55 GB/s with about
// 2 us of read latency, so ~110 KB must be in flight; 24 CTAs of 128 KiB keep
// 3 MiB in flight and leave the other SMs to concurrent work.
constexpr int kBulkCtas = 24;

cudaError_t evict_bulk(const void* src_dev, void* dst_mapped, uint64_t nbytes, uint64_t* digests, uint32_t* error,
                       cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src_dev || !dst_mapped || !bulk_ok(src_dev, dst_mapped, nbytes)) return cudaErrorInvalidValue;
    PushItem one{};
    one.src = src_dev;
    one.dst = dst_mapped;
    one.nbytes = nbytes;
    one.mode = kPushBulk;
    one.flags = digests ? 0u : kPushNoHash;
    PushState st{digests, nullptr, nullptr, error};
    return launch_stages<4>(nullptr, 1, ssh::num_chunks(nbytes), st, one, s, ctas > 0 ? ctas : kBulkCtas,
                            kIdEvictBulk);
}

cudaError_t restore_bulk(const void* src_mapped, void* dst_dev, uint64_t nbytes, uint32_t* error, cudaStream_t s,
                         int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src_mapped || !dst_dev || !bulk_ok(src_mapped, dst_dev, nbytes)) return cudaErrorInvalidValue;
    PushItem one{};
    one.src = src_mapped;
    one.dst = dst_dev;
    one.nbytes = nbytes;
    one.mode = kPushBulk;
    one.flags = kPushNoHash;
    PushState st{nullptr, nullptr, nullptr, error};
    return launch_stages<4>(nullptr, 1, ssh::num_chunks(nbytes), st, one, s, ctas > 0 ? ctas : kBulkCtas,
                            kIdRestoreBulk);
}

uint64_t push_launch_count() { return g_push_launches.load(std::memory_order_relaxed); }

}  // namespace kern
}  // namespace ofld
