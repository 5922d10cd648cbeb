// K4: in-box weight-sync push (trainer GPU -> rollout GPU over NVLink).
//
// StateSpectre moves a new model version to rollout engines by staging every
// object on the host and sending it over TCP (reference:
// src/daemon/canonical_rollout.cpp:240-411, python_api/state_spectre/_rollout.py:101-175).
// Inside one B200 node the rollout GPUs are NVLink peers, so the trainer
// pushes the changed tensors of a sealed version directly into the rollout's
// weight buffers:
//
//   * one persistent launch walks a work list of (src, dst) items, 64 KiB
//     chunk by chunk (binary search of the chunk's item), so a version with
//     hundreds of changed tensors is one launch;
//   * each chunk is loaded from local HBM once; the same registers feed the
//     ssh128 lane state (the digests verify that the pushed bytes are the
//     sealed version's) and the stores to the peer: raw bytes, or bf16
//     quantized to fp8 e4m3 with one fp32 scale per 128 elements;
//   * stores to the peer are plain st.global on a peer pointer (CUDA IPC
//     mapping over NVLink); no TMA and no multicast load touches peer memory.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <atomic>

#include "kernels.h"
#include "ofld/chunk_hash.h"

namespace ofld {
namespace kern {

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kChunk = ssh::kChunkBytes;
constexpr int kVecs = ssh::kVecsPerLane;

__device__ __forceinline__ uint4 ld_local(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_peer(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ void st_peer8(void* p, uint2 v) {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

__device__ __forceinline__ float lo16(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi16(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_fp8(float a, float b, float c, float d) {
    return uint32_t(__nv_cvt_float_to_fp8(a, __NV_SATFINITE, __NV_E4M3)) |
           (uint32_t(__nv_cvt_float_to_fp8(b, __NV_SATFINITE, __NV_E4M3)) << 8) |
           (uint32_t(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3)) << 16) |
           (uint32_t(__nv_cvt_float_to_fp8(d, __NV_SATFINITE, __NV_E4M3)) << 24);
}

__device__ __forceinline__ uint64_t chunk_tree(uint64_t d, uint64_t* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        uint64_t o = __shfl_down_sync(0xffffffffu, d, s);
        if ((lane & (2 * s - 1)) == 0) d = ssh::fold(d, o);
    }
    if (lane == 0) red[warp] = d;
    __syncthreads();
    uint64_t root = 0;
    if (threadIdx.x == 0) {
        uint64_t x[kThreads / 32];
#pragma unroll
        for (int i = 0; i < kThreads / 32; ++i) x[i] = red[i];
#pragma unroll
        for (int s = 1; s < kThreads / 32; s <<= 1)
#pragma unroll
            for (int i = 0; i < kThreads / 32; i += 2 * s) x[i] = ssh::fold(x[i], x[i + s]);
        root = x[0];
    }
    __syncthreads();
    return root;
}

// Object fold of one item's chunk digests, run by the CTA that finishes the
// item's last chunk (detected with a device-scope counter; no CTA waits on
// another).
__device__ __forceinline__ void fold_item(const PushItem& it, int idx, const PushState& st) {
    const uint64_t n = ssh::num_chunks_dev(it.nbytes);
    uint64_t lo, hi;
    ssh::object_init(lo, hi);
    const volatile uint64_t* d = st.digests + it.chunk_begin;
    for (uint64_t i = 0; i < n; ++i) ssh::object_absorb(lo, hi, d[i]);
    ssh::Object o = ssh::object_finish(lo, hi, it.nbytes);
    st.item_hash[2 * idx] = o.lo;
    st.item_hash[2 * idx + 1] = o.hi;
}

__global__ void __launch_bounds__(kThreads, 2)
    k_push(const PushItem* __restrict__ items, int nitems, uint64_t total_chunks, PushState st) {
    __shared__ uint64_t red[kThreads / 32];
    __shared__ int s_store, s_last;
    const uint32_t t = threadIdx.x;
    for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
        // item owning chunk c: last item with chunk_begin <= c
        int lo = 0, hi = nitems - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (items[mid].chunk_begin <= c) lo = mid;
            else hi = mid - 1;
        }
        const int idx = lo;
        const PushItem it = items[idx];
        const uint64_t base = (c - it.chunk_begin) * kChunk;
        const uint32_t len = uint32_t(it.nbytes - base < kChunk ? it.nbytes - base : kChunk);
        const uint32_t nvec = len / 16;  // the launcher guarantees nbytes % 16 == 0
        const uint8_t* src = static_cast<const uint8_t*>(it.src) + base;
        uint4 v[kVecs];
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            v[k] = vi < nvec ? ld_local(src + uint64_t(vi) * 16) : make_uint4(0, 0, 0, 0);
        }
        ssh::Lane L = ssh::lane_init(t);
#pragma unroll
        for (int k = 0; k < kVecs; ++k)
            if (uint32_t(k) * kThreads + t < nvec) ssh::lane_update(L, v[k].x, v[k].y, v[k].z, v[k].w);
        const uint64_t root = chunk_tree(ssh::lane_digest(L, t), red);
        if (t == 0) {
            const uint64_t dg = ssh::chunk_finish(root, len);
            const bool same = (it.flags & kPushDelta) && st.digests[c] == dg;
            st.digests[c] = dg;
            s_store = it.mode != kPushHash && !same;
            if (s_store && st.stats) {
                atomicAdd(&st.stats[0], 1ull);
                atomicAdd(&st.stats[1], (unsigned long long)len);
            }
        }
        __syncthreads();
        if (s_store) {
            if (it.mode == kPushRaw) {
                uint8_t* dst = static_cast<uint8_t*>(it.dst) + base;
#pragma unroll
                for (int k = 0; k < kVecs; ++k) {
                    const uint32_t vi = uint32_t(k) * kThreads + t;
                    if (vi < nvec) st_peer(dst + uint64_t(vi) * 16, v[k]);
                }
            } else {
                // 16 consecutive lanes hold one 128-element block (chunk bases are block aligned)
#pragma unroll
                for (int k = 0; k < kVecs; ++k) {
                    const uint32_t vi = uint32_t(k) * kThreads + t;
                    const bool valid = vi < nvec;
                    float f[8] = {lo16(v[k].x), hi16(v[k].x), lo16(v[k].y), hi16(v[k].y),
                                  lo16(v[k].z), hi16(v[k].z), lo16(v[k].w), hi16(v[k].w)};
                    float amax = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, valid ? fabsf(f[i]) : 0.f);
#pragma unroll
                    for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                    const float inv = amax > 0.f ? 448.f / amax : 1.f;
                    if (valid) {
                        const uint64_t elem = base / 2 + uint64_t(vi) * 8;
                        uint2 q = make_uint2(pack_fp8(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv),
                                             pack_fp8(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv));
                        st_peer8(static_cast<uint8_t*>(it.dst) + elem, q);
                        if ((t & 15) == 0) it.dst_scales[elem / 128] = amax > 0.f ? amax / 448.f : 1.f;
                    }
                }
            }
        }
        if (st.item_hash) {
            // Last finisher of the item folds its digests.
            if (t == 0) {
                __threadfence();
                const uint32_t need = uint32_t(ssh::num_chunks_dev(it.nbytes));
                const uint32_t prev = atomicAdd(&st.item_done[idx], 1u);
                s_last = prev + 1 == need;
                if (s_last) {
                    __threadfence();
                    fold_item(it, idx, st);
                    st.item_done[idx] = 0;
                }
            }
        }
        __syncthreads();  // s_store / s_last / red reuse by the next chunk
    }
}

std::atomic<uint64_t> g_push_launches{0};

}  // namespace

cudaError_t push(const PushItem* items_dev, int nitems, uint64_t total_chunks, PushState st, cudaStream_t s,
                 int ctas) {
    if (nitems <= 0 || total_chunks == 0) return cudaSuccess;
    if (!items_dev || !st.digests || (st.item_hash && !st.item_done)) return cudaErrorInvalidValue;
    int g = ctas > 0 ? ctas : 148 * 2;
    if (uint64_t(g) > total_chunks) g = int(total_chunks);
    k_push<<<g, kThreads, 0, s>>>(items_dev, nitems, total_chunks, st);
    g_push_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

uint64_t push_launch_count() { return g_push_launches.load(std::memory_order_relaxed); }

}  // namespace kern
}  // namespace ofld
