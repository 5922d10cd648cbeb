// sm_100a data-path kernels of the offload runtime.
//
// StateSpectre moves every byte with cudaMemcpyAsync on the copy engines and
// hashes on the host, byte-serially (reference: src/agent/agent.cpp:57-68,
// 825-829, 992-996). Here the SMs move the bytes so the content hash, digest
// verification and dtype casts happen in the same pass over the data:
//
//   * One CTA of 256 threads owns one 64 KiB chunk at a time; thread t is hash
//     lane t and touches 16-byte vectors t, t+256, ... (16 per chunk). Each
//     thread issues all 16 of its loads before consuming any, so a CTA keeps
//     64 KiB in flight: enough memory-level parallelism to cover PCIe read
//     latency for host-mapped sources with a few dozen CTAs.
//   * Loads use the non-coherent read-only path without L1 allocation; stores
//     to host memory are streaming (.cs): every byte is touched once.
//   * The 256 lane digests reduce with warp shuffles and one shared-memory
//     step into the chunk digest (the ssh128 tree, ofld/chunk_hash.h).
//   * Grids are persistent and sized by the caller (a few dozen CTAs) so a
//     concurrent GEMM keeps most SMs.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <set>

#include "kernels.h"
#include "timing.h"
#include "ofld/chunk_hash.h"
#include "ofld/zbf16.h"

namespace ofld {
namespace kern {

namespace {

std::atomic<uint64_t> g_launches{0};

constexpr int kThreads = 256;  // == ssh::kLanes
constexpr uint32_t kChunk = ssh::kChunkBytes;
constexpr int kVecs = ssh::kVecsPerLane;  // 16
static_assert(kThreads == int(ssh::kLanes), "one thread per hash lane");

__host__ __device__ __forceinline__ uint64_t round_up_dev(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ uint4 ld_once(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 ld_bytes(const uint8_t* p, uint32_t n) {
    uint32_t w[4] = {0, 0, 0, 0};
    for (uint32_t i = 0; i < n; ++i) w[i >> 2] |= uint32_t(p[i]) << (8 * (i & 3));
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void st_bytes(uint8_t* p, uint4 v, uint32_t n) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    for (uint32_t i = 0; i < n; ++i) p[i] = uint8_t(w[i >> 2] >> (8 * (i & 3)));
}

template <bool ALIGNED>
__device__ __forceinline__ uint4 load_vec(const uint8_t* p, uint32_t n) {
    if (ALIGNED && n == 16) return ld_once(p);
    return ld_bytes(p, n);
}

template <bool ALIGNED>
__device__ __forceinline__ void store_vec(uint8_t* p, uint4 v, uint32_t n) {
    if (ALIGNED && n == 16)
        st_stream(p, v);
    else
        st_bytes(p, v, n);
}

// Reduce lane digests to the chunk digest (valid in thread 0). Implements the
// ssh128 tree: at distance s, entry i (multiple of 2s) = fold(x[i], x[i+s]).
__device__ __forceinline__ uint64_t tree_fold(uint64_t d, uint64_t* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        uint64_t other = __shfl_down_sync(0xffffffffu, d, s);
        if (((lane & (2 * s - 1)) == 0)) d = ssh::fold(d, other);
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

// K1 and the device hash. STORE=false hashes without copying.
template <bool ALIGNED, bool HASH, bool STORE>
__global__ void __launch_bounds__(kThreads, 2)
    k_evict(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t nbytes,
            uint64_t* __restrict__ digests, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    __shared__ uint64_t red[kThreads / 32];
    const uint32_t t = threadIdx.x;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        const uint32_t nvec = (len + 15) / 16;
        uint4 v[kVecs];
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            const uint32_t n = vi < nvec ? min(16u, len - vi * 16) : 0u;
            v[k] = n ? load_vec<ALIGNED>(src + base + uint64_t(vi) * 16, n) : make_uint4(0, 0, 0, 0);
        }
        ssh::Lane L = ssh::lane_init(t);
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            if (vi < nvec) {
                if (HASH) ssh::lane_update(L, v[k].x, v[k].y, v[k].z, v[k].w);
                if (STORE) store_vec<ALIGNED>(dst + base + uint64_t(vi) * 16, v[k], min(16u, len - vi * 16));
            }
        }
        if (HASH) {
            uint64_t root = tree_fold(ssh::lane_digest(L, t), red);
            if (t == 0) digests[c] = ssh::chunk_finish(root, len);
        }
    }
}

// ---- K2: restore with optional verify and cast -----------------------------

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t fp8x4(float a, float b, float c, float d) {
    uint32_t r = 0;
    r |= uint32_t(__nv_cvt_float_to_fp8(a, __NV_SATFINITE, __NV_E4M3));
    r |= uint32_t(__nv_cvt_float_to_fp8(b, __NV_SATFINITE, __NV_E4M3)) << 8;
    r |= uint32_t(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3)) << 16;
    r |= uint32_t(__nv_cvt_float_to_fp8(d, __NV_SATFINITE, __NV_E4M3)) << 24;
    return r;
}

// Quantize 8 bf16 values (one 16-byte vector) of a 128-element block whose 16
// vectors sit in 16 consecutive lanes. Returns the 8 fp8 bytes; lane 0 of the
// group stores the block scale.
__device__ __forceinline__ uint2 quant8(uint4 v, bool valid, float* scale_out) {
    float f[8] = {bf16_lo(v.x), bf16_hi(v.x), bf16_lo(v.y), bf16_hi(v.y),
                  bf16_lo(v.z), bf16_hi(v.z), bf16_lo(v.w), bf16_hi(v.w)};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, valid ? fabsf(f[i]) : 0.f);
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 448.f / amax : 1.f;
    *scale_out = amax > 0.f ? amax / 448.f : 1.f;
    return make_uint2(fp8x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv),
                      fp8x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv));
}

template <bool ALIGNED, bool VERIFY, int CAST>
__global__ void __launch_bounds__(kThreads, 2)
    k_restore(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t nbytes,
              float* __restrict__ scales, const uint64_t* __restrict__ expect, uint32_t* mismatch, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    __shared__ uint64_t red[kThreads / 32];
    const uint32_t t = threadIdx.x;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        const uint32_t nvec = (len + 15) / 16;
        uint4 v[kVecs];
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            const uint32_t n = vi < nvec ? min(16u, len - vi * 16) : 0u;
            v[k] = n ? load_vec<ALIGNED>(src + base + uint64_t(vi) * 16, n) : make_uint4(0, 0, 0, 0);
        }
        ssh::Lane L = ssh::lane_init(t);
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            const bool valid = vi < nvec;
            if (VERIFY && valid) ssh::lane_update(L, v[k].x, v[k].y, v[k].z, v[k].w);
            const uint64_t gv = base / 16 + vi;  // global vector index
            if (CAST == int(Cast::kNone)) {
                if (valid) store_vec<ALIGNED>(dst + gv * 16, v[k], min(16u, len - vi * 16));
            } else if (CAST == int(Cast::kBf16ToFp8Block128)) {
                float s;
                uint2 q = quant8(v[k], valid, &s);  // all lanes take part in the shuffle
                if (valid) {
                    *reinterpret_cast<uint2*>(dst + gv * 8) = q;
                    if ((t & 15) == 0) scales[gv / 16] = s;
                }
            } else if (CAST == int(Cast::kFp32ToBf16)) {
                if (valid) {
                    uint2 o = make_uint2(pack_bf16x2(__uint_as_float(v[k].x), __uint_as_float(v[k].y)),
                                         pack_bf16x2(__uint_as_float(v[k].z), __uint_as_float(v[k].w)));
                    *reinterpret_cast<uint2*>(dst + gv * 8) = o;
                }
            } else if (CAST == int(Cast::kBf16ToFp32)) {
                if (valid) {
                    uint4 a = make_uint4(__float_as_uint(bf16_lo(v[k].x)), __float_as_uint(bf16_hi(v[k].x)),
                                         __float_as_uint(bf16_lo(v[k].y)), __float_as_uint(bf16_hi(v[k].y)));
                    uint4 b = make_uint4(__float_as_uint(bf16_lo(v[k].z)), __float_as_uint(bf16_hi(v[k].z)),
                                         __float_as_uint(bf16_lo(v[k].w)), __float_as_uint(bf16_hi(v[k].w)));
                    *reinterpret_cast<uint4*>(dst + gv * 32) = a;
                    *reinterpret_cast<uint4*>(dst + gv * 32 + 16) = b;
                }
            }
        }
        if (VERIFY) {
            uint64_t root = tree_fold(ssh::lane_digest(L, t), red);
            if (t == 0 && ssh::chunk_finish(root, len) != expect[c]) atomicAdd(mismatch, 1u);
        }
    }
}

// ---- zbf16 coding (pre-pass, K1 with coding, K2 with decoding) -----------

// Exclusive prefix sum over the 256 threads of the block; *total = the sum.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t x, uint32_t* sm, uint32_t* total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= uint32_t(o)) inc += y;
    }
    if (lane == 31) sm[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < kThreads / 32 ? sm[lane] : 0;
#pragma unroll
        for (int o = 1; o < kThreads / 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= uint32_t(o)) w += y;
        }
        if (lane < kThreads / 32) sm[lane] = w;
    }
    __syncthreads();
    const uint32_t warp_off = warp ? sm[warp - 1] : 0;
    *total = sm[kThreads / 32 - 1];
    __syncthreads();  // sm is reused by the next call
    return warp_off + inc - x;
}

__device__ __forceinline__ uint32_t half_of(const uint4& v, int j) {
    const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
    return (j & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Vector vi of a coded chunk's bf16 elements. bf16 objects: the 16 bytes at
// src + 16 vi. zf32 rows: the top halves of the eight fp32 values at
// src + 32 vi, in element order, with their low halves in *lo.
template <bool F32>
__device__ __forceinline__ uint4 ld_zvec(const uint8_t* __restrict__ src, uint32_t vi, uint4* lo) {
    if (!F32) return ld_once(src + uint64_t(vi) * 16);
    const uint4 a = ld_once(src + uint64_t(vi) * 32), b = ld_once(src + uint64_t(vi) * 32 + 16);
    *lo = make_uint4(__byte_perm(a.x, a.y, 0x5410), __byte_perm(a.z, a.w, 0x5410), __byte_perm(b.x, b.y, 0x5410),
                     __byte_perm(b.z, b.w, 0x5410));
    return make_uint4(__byte_perm(a.x, a.y, 0x7632), __byte_perm(a.z, a.w, 0x7632), __byte_perm(b.x, b.y, 0x7632),
                      __byte_perm(b.z, b.w, 0x7632));
}

// Pre-pass over one chunk: the largest exponent (window base = emax - 14)
// and whether the coded chunk fits in its raw length; a chunk that does not
// fit sets *fail and the object is then moved uncoded. Two register passes
// per chunk, so the pass runs at HBM rate. Every thread of the block calls
// this; `red` is reused on return.
// `stored` (may be null; thread 0's value counts) receives the chunk's stored length.
// F32: `src` is a zf32 row and the chunk is its top halves (len = kChunk).
template <bool F32 = false>
__device__ __forceinline__ void zscan_chunk(const uint8_t* __restrict__ src, uint32_t len, uint8_t* eb_out,
                                            uint32_t* fail, uint32_t* red, uint32_t* stored = nullptr) {
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t nvec = len / 16;
    uint4 v[kVecs];
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
        const uint32_t vi = uint32_t(k) * kThreads + t;
        uint4 lo;
        v[k] = vi < nvec ? ld_zvec<F32>(src, vi, &lo) : make_uint4(0, 0, 0, 0);
    }
    // bf16 bit patterns with the sign cleared order like their magnitudes
    uint32_t m = 0;
    auto hmax = [](uint32_t w) { return max(w & 0x7FFFu, (w >> 16) & 0x7FFFu); };
#pragma unroll
    for (int k = 0; k < kVecs; ++k)
        m = max(m, max(max(hmax(v[k].x), hmax(v[k].y)), max(hmax(v[k].z), hmax(v[k].w))));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    uint32_t mm = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) mm = max(mm, red[w]);
    const uint32_t eb = zbf16::window_base(zbf16::exponent(uint16_t(mm)));
    // mode-1 escapes in the low half, values in the window's lowest 8 binades
    // in the high half (each at most 32768 per chunk: no carry between halves)
    uint32_t cnt = 0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
        const uint32_t vi = uint32_t(k) * kThreads + t;
        if (vi < nvec)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t e = zbf16::exponent(uint16_t(half_of(v[k], j)));
                cnt += (zbf16::code_of(e, eb) == zbf16::kEscape ? 1u : 0u) + (zbf16::in_low8(e, eb) ? 0x10000u : 0u);
            }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    __syncthreads();  // everyone has read red[] (the max)
    if (lane == 0) red[warp] = cnt;
    __syncthreads();
    if (t == 0) {
        uint32_t tot = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) tot += red[w];
        *eb_out = uint8_t(eb);
        uint32_t clen = 0;
        zbf16::choose_mode(len, eb, tot & 0xFFFFu, tot >> 16, &clen);
        if (clen > len) atomicOr(fail, 1u);
        if (stored) *stored = clen;
    }
    __syncthreads();  // red[] is reused by the next chunk
}

// F32: `nbytes` is the fp32 object's size (whole zf32 rows); chunk c is the
// top halves of row c.
template <bool F32>
__global__ void __launch_bounds__(kThreads, F32 ? 2 : 3)
    k_zscan(const uint8_t* __restrict__ src, uint64_t nbytes, uint8_t* __restrict__ ebase_out, uint32_t* fail,
            uint32_t* max_coded, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    __shared__ uint32_t red[kThreads / 32];
    const uint64_t nchunks = F32 ? nbytes / zf32::kRow : (nbytes + kChunk - 1) / kChunk;
    uint32_t cta_max = 0;  // thread 0: largest stored length of this CTA's chunks
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = F32 ? kChunk : uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        if (!F32 && zbf16::raw_by_rule(c, nchunks, len)) {
            if (threadIdx.x == 0) {
                ebase_out[c] = 0;
                cta_max = max(cta_max, len);  // stored raw
            }
            continue;  // uniform per chunk
        }
        uint32_t clen = 0;
        zscan_chunk<F32>(src + (F32 ? c * zf32::kRow : base), len, ebase_out + c, fail, red, &clen);
        cta_max = max(cta_max, clen);
    }
    // One plain store per CTA into its own slot (the slots may be host-mapped
    // memory: per-chunk atomics there would each cross PCIe); the host reduces.
    if (max_coded && threadIdx.x == 0) max_coded[blockIdx.x] = cta_max;
}

// Shared-memory stage of one coded chunk: PCIe moves it with full 16-byte
// vector accesses (512 bytes per warp instruction), like the uncoded path;
// the planes' 8- and 4-byte pieces are only ever touched in shared memory.
constexpr uint32_t kZStage = zbf16::kChunk;

// One chunk of K1 with coding: hash the raw bytes, code the chunk into shared
// memory (or keep it raw) and stream it to the host-mapped destination with
// 16-byte vector stores. `src`/`dst` point at the chunk; 16-byte aligned,
// len % 16 == 0. Every thread of the block calls this.
// F32: `src`/`dst` are a zf32 row: the low halves go to dst, the coded top
// halves to dst + kChunk; no digests (the caller hashes the fp32 bytes).
template <bool F32 = false>
__device__ __forceinline__ void evict_chunk_z(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                              uint32_t len, bool raw, uint32_t eb, uint64_t* digest_out,
                                              uint64_t* red, uint32_t* sc, uint8_t* zbuf) {
    const uint32_t t = threadIdx.x;
    const uint32_t nvec = len / 16;
    uint4 v[kVecs];
    if (F32) {
        // groups of four vectors: eight 16-byte loads in flight, then the
        // four low-half vectors leave (bounded registers: the top halves of
        // all sixteen stay for the coding below)
#pragma unroll
        for (int k0 = 0; k0 < kVecs; k0 += 4) {
            uint4 a[4], b[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint64_t off = uint64_t(uint32_t(k0 + q) * kThreads + t) * 32;
                a[q] = ld_once(src + off);
                b[q] = ld_once(src + off + 16);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t vi = uint32_t(k0 + q) * kThreads + t;
                v[k0 + q] = make_uint4(__byte_perm(a[q].x, a[q].y, 0x7632), __byte_perm(a[q].z, a[q].w, 0x7632),
                                       __byte_perm(b[q].x, b[q].y, 0x7632), __byte_perm(b[q].z, b[q].w, 0x7632));
                st_stream(dst + uint64_t(vi) * 16,
                          make_uint4(__byte_perm(a[q].x, a[q].y, 0x5410), __byte_perm(a[q].z, a[q].w, 0x5410),
                                     __byte_perm(b[q].x, b[q].y, 0x5410), __byte_perm(b[q].z, b[q].w, 0x5410)));
            }
        }
        dst += kChunk;
    } else {
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            v[k] = vi < nvec ? ld_once(src + uint64_t(vi) * 16) : make_uint4(0, 0, 0, 0);
        }
    }
    ssh::Lane L = ssh::lane_init(t);
    // mode-1 escapes (low half) and values in the lowest 8 binades of the
    // mode-1 window (high half); one scan of the pair gives both modes' offsets
    uint32_t cnt = 0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
        const uint32_t vi = uint32_t(k) * kThreads + t;
        if (vi < nvec) {
            if (!F32) ssh::lane_update(L, v[k].x, v[k].y, v[k].z, v[k].w);
            if (raw) {
                st_stream(dst + uint64_t(vi) * 16, v[k]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t e = zbf16::exponent(uint16_t(half_of(v[k], j)));
                    cnt += (zbf16::code_of(e, eb) == zbf16::kEscape ? 1u : 0u) + (zbf16::in_low8(e, eb) ? 0x10000u : 0u);
                }
            }
        }
    }
    if (!raw) {  // uniform per chunk
        uint32_t tot;
        const uint32_t offp = block_excl_scan(cnt, sc, &tot);
        const uint32_t n = len / 2;
        uint32_t comp = 0;
        const bool m2 = zbf16::choose_mode(len, eb, tot & 0xFFFFu, tot >> 16, &comp) == 2;
        const uint32_t base = m2 ? eb + zbf16::kBase3Offset : eb;
        const uint32_t plane = m2 ? (n / 8) * 3 : n / 2;
        uint32_t off = m2 ? (offp & 0xFFFFu) + (offp >> 16) : (offp & 0xFFFFu);
        if (t == 0)
            *reinterpret_cast<uint4*>(zbuf) = make_uint4(uint32_t(zbf16::kTag) | ((m2 ? 2u : 1u) << 16) | (base << 24),
                                                         comp - (zbf16::kHeader + n + plane), len, comp);
        uint8_t* esc = zbuf + zbf16::kHeader + n + plane;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            if (vi >= nvec) continue;
            uint32_t lo0 = 0, lo1 = 0, codes = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint16_t h = uint16_t(half_of(v[k], j));
                const uint32_t e = zbf16::exponent(h);
                const uint32_t lb = zbf16::low_byte(h);
                if (j < 4) lo0 |= lb << (8 * j);
                else lo1 |= lb << (8 * (j - 4));
                if (m2) {
                    const uint32_t cd = zbf16::code3_of(e, base);
                    codes |= cd << (3 * j);
                    if (cd == zbf16::kEscape3) esc[off++] = uint8_t(e);
                } else {
                    const uint32_t cd = zbf16::code_of(e, base);
                    codes |= cd << (4 * j);
                    if (cd == zbf16::kEscape) esc[off++] = uint8_t(e);
                }
            }
            *reinterpret_cast<uint2*>(zbuf + zbf16::kHeader + vi * 8) = make_uint2(lo0, lo1);
            if (m2) {
                uint8_t* c3 = zbuf + zbf16::kHeader + n + vi * 3;
                c3[0] = uint8_t(codes);
                c3[1] = uint8_t(codes >> 8);
                c3[2] = uint8_t(codes >> 16);
            } else {
                *reinterpret_cast<uint32_t*>(zbuf + zbf16::kHeader + n + vi * 4) = codes;
            }
        }
        __syncthreads();
        const uint32_t nout = (comp + 15) / 16;  // <= len / 16: coded chunks fit their raw length
        for (uint32_t i = t; i < nout; i += kThreads)
            st_stream(dst + uint64_t(i) * 16, *reinterpret_cast<const uint4*>(zbuf + i * 16));
    }
    if (F32) {
        __syncthreads();  // orders zbuf reuse
        return;
    }
    uint64_t root = tree_fold(ssh::lane_digest(L, t), red);  // also orders zbuf reuse
    if (t == 0 && digest_out) *digest_out = ssh::chunk_finish(root, len);
}

// K1 with coding over one object. Requires 16-byte aligned src/dst and
// nbytes % 16 == 0 (zbf16::eligible).
// F32: a zf32 object (nbytes a whole number of rows), no digests.
template <bool F32>
__global__ void __launch_bounds__(kThreads, 2)
    k_evict_z(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t nbytes,
              const uint8_t* __restrict__ ebase, uint64_t* __restrict__ digests, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    extern __shared__ __align__(16) uint8_t zbuf[];
    __shared__ uint64_t red[kThreads / 32];
    __shared__ uint32_t sc[kThreads / 32];
    if (F32) {
        const uint64_t nrows = nbytes / zf32::kRow;
        // == kChunk, but computed: with the length a compile-time constant the
        // coder's specialised form needs far more than its 128 registers
        const uint32_t len = nrows ? uint32_t(nbytes / nrows / 2) : kChunk;
        for (uint64_t c = blockIdx.x; c < nrows; c += gridDim.x)
            evict_chunk_z<true>(src + c * zf32::kRow, dst + c * zf32::kRow, len, false, uint32_t(ebase[c]), nullptr,
                                red, sc, zbuf);
        return;
    }
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        const bool raw = zbf16::raw_by_rule(c, nchunks, len);
        const uint32_t eb = raw ? 0u : uint32_t(ebase[c]);
        evict_chunk_z(src + base, dst + base, len, raw, eb, digests ? digests + c : nullptr, red, sc, zbuf);
    }
}

// Items of a batch are sorted by first chunk and every CTA visits its chunks
// in increasing order, so the owning job only ever advances.
__device__ __forceinline__ void advance_job(const XferJob* jobs, int n, uint64_t c, int& idx) {
    while (idx + 1 < n && jobs[idx + 1].chunk_begin <= c) ++idx;
}

// The pre-pass over a batch: job `src`/`nbytes`/`chunk_begin` as for K1;
// `dst` is the job's scan buffer (one window base per chunk, then the fail
// word at the next 16-byte boundary).
__global__ void __launch_bounds__(kThreads, 3)
    k_zscan_jobs(const XferJob* __restrict__ jobs, int njobs, uint64_t total_chunks, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    __shared__ uint32_t red[kThreads / 32];
    int idx = 0;
    for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
        advance_job(jobs, njobs, c, idx);
        const XferJob j = jobs[idx];
        const uint64_t lc = c - j.chunk_begin, nch = (j.nbytes + kChunk - 1) / kChunk;
        const uint64_t base = lc * kChunk;
        const uint32_t len = uint32_t(j.nbytes - base < kChunk ? j.nbytes - base : kChunk);
        uint8_t* eb = static_cast<uint8_t*>(j.dst);
        if (zbf16::raw_by_rule(lc, nch, len)) {
            if (threadIdx.x == 0) eb[lc] = 0;
            continue;  // uniform per chunk
        }
        zscan_chunk(static_cast<const uint8_t*>(j.src) + base, len, eb + lc,
                    reinterpret_cast<uint32_t*>(eb + (nch + 15) / 16 * 16), red);
    }
}

// K1 over a batch: one grid walks every chunk of every job (raw or coded per
// job), so many small tensors (KV-cache blocks) cost one launch.
__global__ void __launch_bounds__(kThreads, 2)
    k_evict_jobs(const XferJob* __restrict__ jobs, int njobs, uint64_t total_chunks, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    extern __shared__ __align__(16) uint8_t zbuf[];
    __shared__ uint64_t red[kThreads / 32];
    __shared__ uint32_t sc[kThreads / 32];
    int idx = 0;
    for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
        advance_job(jobs, njobs, c, idx);
        const XferJob j = jobs[idx];
        const uint64_t lc = c - j.chunk_begin, nch = (j.nbytes + kChunk - 1) / kChunk;
        const uint64_t base = lc * kChunk;
        const uint32_t len = uint32_t(j.nbytes - base < kChunk ? j.nbytes - base : kChunk);
        const bool raw = !j.ebase || zbf16::raw_by_rule(lc, nch, len);
        const uint32_t eb = raw ? 0u : uint32_t(j.ebase[lc]);
        evict_chunk_z(static_cast<const uint8_t*>(j.src) + base, static_cast<uint8_t*>(j.dst) + base, len, raw, eb,
                      j.digests ? j.digests + lc : nullptr, red, sc, zbuf);
    }
}

// Loads [lo, hi) of a host-mapped chunk into the stage with 16-byte vectors,
// up to 13 in flight per thread (one full coded chunk plus 1 KiB of escapes).
__device__ __forceinline__ void stage_in(const uint8_t* in, uint8_t* zbuf, uint32_t lo, uint32_t hi) {
    constexpr int kPer = 13;
    const uint32_t t = threadIdx.x;
    const uint32_t v0 = lo / 16, v1 = (hi + 15) / 16;
    for (uint32_t b = v0; b < v1; b += kPer * kThreads) {
        uint4 r[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t i = b + uint32_t(k) * kThreads + t;
            r[k] = i < v1 ? ld_once(in + uint64_t(i) * 16) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t i = b + uint32_t(k) * kThreads + t;
            if (i < v1) *reinterpret_cast<uint4*>(zbuf + i * 16) = r[k];
        }
    }
}

// One chunk of K2 with decoding, into registers: thread t receives vectors
// k*256 + t (zeros past the end). Coded chunks come into shared memory with
// 16-byte loads (header, planes and, speculatively, 1 KiB of escapes in one
// round trip; the rest of the escapes in a second one when present); raw
// chunks load straight into registers. Every thread of the block calls this.
__device__ __forceinline__ void load_chunk_z(const uint8_t* __restrict__ in, uint32_t len, bool raw,
                                             uint32_t* sc, uint8_t* zbuf, uint4 (&v)[kVecs]) {
    const uint32_t t = threadIdx.x;
    const uint32_t nvec = len / 16;
    if (raw) {
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            v[k] = vi < nvec ? ld_once(in + uint64_t(vi) * 16) : make_uint4(0, 0, 0, 0);
        }
        return;
    }
    const uint32_t n = len / 2;
    // stage the header, both planes and 1 KiB of escapes in one round trip
    // (sized for mode 1, whose code plane is the larger)
    const uint32_t fixed1 = zbf16::kHeader + n + n / 2;
    const uint32_t spec = min(len, fixed1 + 1024u);
    stage_in(in, zbuf, 0, spec);
    __syncthreads();
    const uint4 hd = *reinterpret_cast<const uint4*>(zbuf);
    const uint32_t comp = min(hd.w, len);
    if (comp > spec) {  // uniform: every thread read the same header
        stage_in(in, zbuf, spec / 16 * 16, comp);
        __syncthreads();
    }
    const bool m2 = ((hd.x >> 16) & 0xFFu) == 2u;
    const uint32_t fixed = m2 ? zbf16::kHeader + n + (n / 8) * 3 : fixed1;
    const uint32_t eb = hd.x >> 24;  // the stored mode's base
    uint2 lo[kVecs];
    uint32_t cd[kVecs];
    uint32_t cnt = 0;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
        const uint32_t vi = uint32_t(k) * kThreads + t;
        if (vi < nvec) {
            lo[k] = *reinterpret_cast<const uint2*>(zbuf + zbf16::kHeader + vi * 8);
            if (m2) {  // widen the 3-bit codes to mode 1's nibbles (escape 7 -> 15)
                const uint8_t* c3 = zbuf + zbf16::kHeader + n + vi * 3;
                const uint32_t w = uint32_t(c3[0]) | (uint32_t(c3[1]) << 8) | (uint32_t(c3[2]) << 16);
                uint32_t c4 = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t c = (w >> (3 * j)) & 7u;
                    c4 |= (c == zbf16::kEscape3 ? zbf16::kEscape : c) << (4 * j);
                }
                cd[k] = c4;
            } else {
                cd[k] = *reinterpret_cast<const uint32_t*>(zbuf + zbf16::kHeader + n + vi * 4);
            }
        } else {
            lo[k] = make_uint2(0, 0);
            cd[k] = 0;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) cnt += ((cd[k] >> (4 * j)) & 15u) == zbf16::kEscape;
    }
    uint32_t total;
    uint32_t off = block_excl_scan(cnt, sc, &total);
    const uint8_t* esc = zbuf + fixed;
#pragma unroll
    for (int k = 0; k < kVecs; ++k) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t code = (cd[k] >> (4 * j)) & 15u;
            const uint32_t lb = ((j < 4 ? lo[k].x : lo[k].y) >> (8 * (j & 3))) & 0xFFu;
            uint32_t e = eb + code;
            if (code == zbf16::kEscape) e = esc[off++];  // only valid vectors carry escapes
            const uint32_t h = zbf16::rebuild(uint8_t(lb), e);
            if (j & 1) w[j >> 1] |= h << 16;
            else w[j >> 1] = h;
        }
        v[k] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    __syncthreads();  // the stage is refilled by the next chunk
}

// zf32 decode (K2 over a zf32 object, no cast or verification): the top
// halves decode into registers, the low halves load from the row's low
// plane, and each vector leaves as eight interleaved fp32 values.
__global__ void __launch_bounds__(kThreads, 2)
    k_restore_zf32(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t nbytes, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    extern __shared__ __align__(16) uint8_t zbuf[];
    __shared__ uint32_t sc[kThreads / 32];
    const uint32_t t = threadIdx.x;
    const uint64_t nrows = nbytes / zf32::kRow;
    const uint32_t len = nrows ? uint32_t(nbytes / nrows / 2) : kChunk;  // == kChunk, computed (registers)
    for (uint64_t c = blockIdx.x; c < nrows; c += gridDim.x) {
        const uint8_t* row = src + c * zf32::kRow;
        uint8_t* out = dst + c * zf32::kRow;
        uint4 v[kVecs];
        load_chunk_z(row + zf32::kLowPlane, len, false, sc, zbuf, v);
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;  // < kChunk / 16: rows are full
            const uint4 lo = ld_once(row + uint64_t(vi) * 16);
            const uint4 a = make_uint4(__byte_perm(lo.x, v[k].x, 0x5410), __byte_perm(lo.x, v[k].x, 0x7632),
                                       __byte_perm(lo.y, v[k].y, 0x5410), __byte_perm(lo.y, v[k].y, 0x7632));
            const uint4 b = make_uint4(__byte_perm(lo.z, v[k].z, 0x5410), __byte_perm(lo.z, v[k].z, 0x7632),
                                       __byte_perm(lo.w, v[k].w, 0x5410), __byte_perm(lo.w, v[k].w, 0x7632));
            // write-back stores: a warp instruction covers every other 16 bytes
            // of its 1 KiB, and L2 must hold the line until the second
            // instruction fills the gaps (an evict-first store made the HBM
            // writes partial-sector read-modify-writes)
            *reinterpret_cast<uint4*>(out + uint64_t(vi) * 32) = a;
            *reinterpret_cast<uint4*>(out + uint64_t(vi) * 32 + 16) = b;
        }
    }
}

// K2 with decoding over one object: decode into registers, then continue as
// K2 (verify, cast, store).
template <bool VERIFY, int CAST>
__global__ void __launch_bounds__(kThreads, 2)
    k_restore_z(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint64_t nbytes,
                float* __restrict__ scales, const uint64_t* __restrict__ expect, uint32_t* mismatch, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    extern __shared__ __align__(16) uint8_t zbuf[];
    __shared__ uint64_t red[kThreads / 32];
    __shared__ uint32_t sc[kThreads / 32];
    const uint32_t t = threadIdx.x;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        const uint32_t nvec = len / 16;
        uint4 v[kVecs];
        load_chunk_z(src + base, len, zbf16::raw_by_rule(c, nchunks, len), sc, zbuf, v);
        ssh::Lane L = ssh::lane_init(t);
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            const bool valid = vi < nvec;
            if (VERIFY && valid) ssh::lane_update(L, v[k].x, v[k].y, v[k].z, v[k].w);
            const uint64_t gv = base / 16 + vi;
            if (CAST == int(Cast::kNone)) {
                if (valid) store_vec<true>(dst + gv * 16, v[k], 16u);
            } else if (CAST == int(Cast::kBf16ToFp8Block128)) {
                float s;
                uint2 q = quant8(v[k], valid, &s);
                if (valid) {
                    *reinterpret_cast<uint2*>(dst + gv * 8) = q;
                    if ((t & 15) == 0) scales[gv / 16] = s;
                }
            } else if (CAST == int(Cast::kBf16ToFp32)) {
                if (valid) {
                    uint4 a = make_uint4(__float_as_uint(bf16_lo(v[k].x)), __float_as_uint(bf16_hi(v[k].x)),
                                         __float_as_uint(bf16_lo(v[k].y)), __float_as_uint(bf16_hi(v[k].y)));
                    uint4 b = make_uint4(__float_as_uint(bf16_lo(v[k].z)), __float_as_uint(bf16_hi(v[k].z)),
                                         __float_as_uint(bf16_lo(v[k].w)), __float_as_uint(bf16_hi(v[k].w)));
                    *reinterpret_cast<uint4*>(dst + gv * 32) = a;
                    *reinterpret_cast<uint4*>(dst + gv * 32 + 16) = b;
                }
            }
        }
        if (VERIFY) {
            uint64_t root = tree_fold(ssh::lane_digest(L, t), red);
            if (t == 0 && ssh::chunk_finish(root, len) != expect[c]) atomicAdd(mismatch, 1u);
        }
    }
}

// K2 over a batch (no cast, no verification): one grid for every chunk of
// every job, raw or coded per job.
__global__ void __launch_bounds__(kThreads, 2)
    k_restore_jobs(const XferJob* __restrict__ jobs, int njobs, uint64_t total_chunks, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    extern __shared__ __align__(16) uint8_t zbuf[];
    __shared__ uint32_t sc[kThreads / 32];
    const uint32_t t = threadIdx.x;
    int idx = 0;
    for (uint64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
        advance_job(jobs, njobs, c, idx);
        const XferJob j = jobs[idx];
        const uint64_t lc = c - j.chunk_begin, nch = (j.nbytes + kChunk - 1) / kChunk;
        const uint64_t base = lc * kChunk;
        const uint32_t len = uint32_t(j.nbytes - base < kChunk ? j.nbytes - base : kChunk);
        const bool raw = !j.coded || zbf16::raw_by_rule(lc, nch, len);
        uint4 v[kVecs];
        load_chunk_z(static_cast<const uint8_t*>(j.src) + base, len, raw, sc, zbuf, v);
        uint8_t* out = static_cast<uint8_t*>(j.dst) + base;
#pragma unroll
        for (int k = 0; k < kVecs; ++k) {
            const uint32_t vi = uint32_t(k) * kThreads + t;
            if (vi < len / 16) store_vec<true>(out + uint64_t(vi) * 16, v[k], 16u);
        }
    }
}

// ---- K3: local hash + exact compare against a peer replica ----------------
__global__ void __launch_bounds__(kThreads, 2)
    k_verify_peer(const uint8_t* __restrict__ local, const uint8_t* __restrict__ peer, uint64_t nbytes,
                  uint64_t* __restrict__ digests, uint32_t* mismatch, KernelStamp* ks) {
    StampScope stamp_scope_(ks);
    __shared__ uint64_t red[kThreads / 32];
    const uint32_t t = threadIdx.x;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        const uint32_t nvec = (len + 15) / 16;
        uint4 a[kVecs / 2], b[kVecs / 2];
        ssh::Lane L = ssh::lane_init(t);
        uint32_t bad = 0;
        // Two halves of 8 vectors each keep 16 loads (8 local + 8 peer) in flight.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int k = 0; k < kVecs / 2; ++k) {
                const uint32_t vi = uint32_t(h * (kVecs / 2) + k) * kThreads + t;
                const uint32_t n = vi < nvec ? min(16u, len - vi * 16) : 0u;
                a[k] = n ? load_vec<true>(local + base + uint64_t(vi) * 16, n) : make_uint4(0, 0, 0, 0);
                b[k] = n ? load_vec<true>(peer + base + uint64_t(vi) * 16, n) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k = 0; k < kVecs / 2; ++k) {
                const uint32_t vi = uint32_t(h * (kVecs / 2) + k) * kThreads + t;
                if (vi < nvec) {
                    ssh::lane_update(L, a[k].x, a[k].y, a[k].z, a[k].w);
                    bad += (a[k].x != b[k].x) | (a[k].y != b[k].y) | (a[k].z != b[k].z) | (a[k].w != b[k].w);
                }
            }
        }
        uint64_t root = tree_fold(ssh::lane_digest(L, t), red);
        if (t == 0 && digests) digests[c] = ssh::chunk_finish(root, len);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
        if ((t & 31) == 0 && bad) atomicAdd(mismatch, bad);
    }
}

__global__ void k_fold(const uint64_t* __restrict__ d, uint64_t n, uint64_t nbytes, uint64_t* out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    uint64_t lo, hi;
    ssh::object_init(lo, hi);
    for (uint64_t i = 0; i < n; ++i) ssh::object_absorb(lo, hi, d[i]);
    ssh::Object o = ssh::object_finish(lo, hi, nbytes);
    out[0] = o.lo;
    out[1] = o.hi;
}

// Standalone 1x128 quantization: one half-warp per 128-element block.
__global__ void __launch_bounds__(kThreads) k_quant_fp8(const uint4* __restrict__ src, uint2* __restrict__ dst,
                                                          float* __restrict__ scales, uint64_t nelem) {
    const uint64_t nvec = (nelem + 7) / 8;
    const uint64_t nblocks = (nelem + 127) / 128;
    const uint64_t stride = uint64_t(gridDim.x) * kThreads;
    // Iterate whole blocks so every half-warp stays converged for its shuffle.
    for (uint64_t vi = uint64_t(blockIdx.x) * kThreads + threadIdx.x; vi < round_up_dev(nblocks * 16, 32);
         vi += stride) {
        const bool valid = vi < nvec;
        uint4 v = valid ? ld_once(src + vi) : make_uint4(0, 0, 0, 0);
        if (valid && (vi + 1) * 8 > nelem) {  // zero elements past the end
            uint32_t keep = uint32_t(nelem - vi * 8);
            uint32_t w[4] = {v.x, v.y, v.z, v.w};
            for (uint32_t e = keep; e < 8; ++e) w[e / 2] &= (e & 1) ? 0x0000ffffu : 0xffff0000u;
            v = make_uint4(w[0], w[1], w[2], w[3]);
        }
        float s;
        uint2 q = quant8(v, valid, &s);
        if (valid) {
            dst[vi] = q;
            if ((threadIdx.x & 15) == 0) scales[vi / 16] = s;
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Opt a coded-path kernel into the 64 KiB dynamic shared-memory stage, once
// per (kernel, device) per process.
cudaError_t allow_stage(const void* fn, int id) {
    static std::mutex mu;
    static std::set<std::pair<int, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(mu);
    if (done.count({id, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kZStage));
    if (e == cudaSuccess) done.insert({id, dev});
    return e;
}

int grid_for(uint64_t nbytes, int ctas, int dflt) {
    uint64_t chunks = (nbytes + kChunk - 1) / kChunk;
    int g = ctas > 0 ? ctas : dflt;
    if (uint64_t(g) > chunks) g = int(chunks);
    return g < 1 ? 1 : g;
}

}  // namespace



uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed) + push_launch_count(); }

cudaError_t evict_hash(const void* src, void* dst, uint64_t nbytes, uint64_t* digests, cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src || !dst) return cudaErrorInvalidValue;
    const int g = grid_for(nbytes, ctas, 48);
    const bool al = aligned16(src) && aligned16(dst);
    KernelStamp* ks = timing_take(kIdEvict, nbytes);
    auto S = static_cast<const uint8_t*>(src);
    auto D = static_cast<uint8_t*>(dst);
    if (digests) {
        if (al) k_evict<true, true, true><<<g, kThreads, 0, s>>>(S, D, nbytes, digests, ks);
        else k_evict<false, true, true><<<g, kThreads, 0, s>>>(S, D, nbytes, digests, ks);
    } else {
        if (al) k_evict<true, false, true><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, ks);
        else k_evict<false, false, true><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, ks);
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

// Aligned buffers go through the K4 bulk-copy pipeline (bulk copies into
// shared memory keep more bytes in flight per SM than per-thread loads);
// others take the one-pass kernel.
cudaError_t hash_device(const void* src, uint64_t nbytes, uint64_t* digests, cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src || !digests) return cudaErrorInvalidValue;
    if (aligned16(src) && (nbytes & 15) == 0) return hash_stream(src, nbytes, digests, nullptr, s, ctas, 0);
    return hash_onepass(src, nbytes, digests, s, ctas);
}

cudaError_t hash_onepass(const void* src, uint64_t nbytes, uint64_t* digests, cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src || !digests) return cudaErrorInvalidValue;
    const int g = grid_for(nbytes, ctas, 148 * 4);
    auto S = static_cast<const uint8_t*>(src);
    KernelStamp* ks = timing_take(kIdHash, nbytes);
    if (aligned16(src)) k_evict<true, true, false><<<g, kThreads, 0, s>>>(S, nullptr, nbytes, digests, ks);
    else k_evict<false, true, false><<<g, kThreads, 0, s>>>(S, nullptr, nbytes, digests, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t restore_cast(const void* src, void* dst, uint64_t nbytes, Cast cast, float* scales,
                         const uint64_t* expect, uint32_t* mismatch, cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!src || !dst) return cudaErrorInvalidValue;
    if (expect && !mismatch) return cudaErrorInvalidValue;
    const int g = grid_for(nbytes, ctas, 96);
    auto S = static_cast<const uint8_t*>(src);
    auto D = static_cast<uint8_t*>(dst);
    const bool verify = expect != nullptr;
    KernelStamp* ks = timing_take(kIdRestore, nbytes);
    if (cast == Cast::kNone) {
        const bool al = aligned16(src) && aligned16(dst);
        if (al && verify) k_restore<true, true, 0><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
        else if (al) k_restore<true, false, 0><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
        else if (verify) k_restore<false, true, 0><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
        else k_restore<false, false, 0><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
    } else {
        // Casts need element-aligned whole vectors.
        if (!aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7) || nbytes % 16) return cudaErrorInvalidValue;
        if (cast == Cast::kBf16ToFp8Block128) {
            if (!scales) return cudaErrorInvalidValue;
            if (verify) k_restore<true, true, 1><<<g, kThreads, 0, s>>>(S, D, nbytes, scales, expect, mismatch, ks);
            else k_restore<true, false, 1><<<g, kThreads, 0, s>>>(S, D, nbytes, scales, nullptr, nullptr, ks);
        } else if (cast == Cast::kFp32ToBf16) {
            if (verify) k_restore<true, true, 2><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
            else k_restore<true, false, 2><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
        } else if (cast == Cast::kBf16ToFp32) {
            if (reinterpret_cast<uintptr_t>(dst) & 15) return cudaErrorInvalidValue;
            if (verify) k_restore<true, true, 3><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
            else k_restore<true, false, 3><<<g, kThreads, 0, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
        } else {
            return cudaErrorInvalidValue;
        }
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t zscan(const void* src, uint64_t nbytes, uint8_t* ebase, uint32_t* fail, cudaStream_t s, int ctas,
                  uint32_t* max_coded) {
    if (max_coded) ctas = ctas > 0 ? std::min(ctas, kZScanSlots) : kZScanSlots;
    if (!zbf16::eligible(nbytes) || !aligned16(src) || !ebase || !fail) return cudaErrorInvalidValue;
    int sms = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    int g = ctas > 0 ? ctas : sms * 3;
    if (uint64_t(g) > nchunks) g = int(nchunks);
    KernelStamp* ks = timing_take(kIdZScan, nbytes);
    k_zscan<false><<<g, kThreads, 0, s>>>(static_cast<const uint8_t*>(src), nbytes, ebase, fail, max_coded, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t zscan_f32(const void* src, uint64_t nbytes, uint8_t* ebase, uint32_t* fail, cudaStream_t s, int ctas,
                      uint32_t* max_coded) {
    if (max_coded) ctas = ctas > 0 ? std::min(ctas, kZScanSlots) : kZScanSlots;
    if (!zf32::eligible(nbytes) || !aligned16(src) || !ebase || !fail) return cudaErrorInvalidValue;
    int sms = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t nrows = zf32::rows(nbytes);
    int g = ctas > 0 ? ctas : sms * 3;
    if (uint64_t(g) > nrows) g = int(nrows);
    KernelStamp* ks = timing_take(kIdZScanF32, nbytes);
    k_zscan<true><<<g, kThreads, 0, s>>>(static_cast<const uint8_t*>(src), nbytes, ebase, fail, max_coded, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t zscan_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t s, int ctas) {
    if (!jobs || njobs <= 0) return cudaErrorInvalidValue;
    if (total_chunks == 0) return cudaSuccess;
    int sms = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int g = ctas > 0 ? ctas : sms * 3;
    if (uint64_t(g) > total_chunks) g = int(total_chunks);
    KernelStamp* ks = timing_take(kIdZScanJobs, total_chunks * kChunk);
    k_zscan_jobs<<<g, kThreads, 0, s>>>(jobs, njobs, total_chunks, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t evict_z(const void* src, void* dst, uint64_t nbytes, const uint8_t* ebase, uint64_t* digests,
                    cudaStream_t s, int ctas) {
    if (!zbf16::eligible(nbytes) || !aligned16(src) || !aligned16(dst) || !ebase) return cudaErrorInvalidValue;
    cudaError_t e = allow_stage(reinterpret_cast<const void*>(&k_evict_z<false>), 0);
    if (e != cudaSuccess) return e;
    // 96 CTAs: PCIe saturates with 48 at full clock, but a training step at
    // the power cap lowers SM clocks and these latency-bound CTAs need the
    // margin (KV blocks under an 8192^2 GEMM loop: 58.8 -> 66.1 GB/s).
    const int g = grid_for(nbytes, ctas, 96);
    KernelStamp* ks = timing_take(kIdEvictZ, nbytes);
    k_evict_z<false><<<g, kThreads, kZStage, s>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), nbytes,
                                           ebase, digests, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t evict_zf32(const void* src, void* dst, uint64_t nbytes, const uint8_t* ebase, cudaStream_t s, int ctas) {
    if (!zf32::eligible(nbytes) || !aligned16(src) || !aligned16(dst) || !ebase) return cudaErrorInvalidValue;
    cudaError_t e = allow_stage(reinterpret_cast<const void*>(&k_evict_z<true>), 12);
    if (e != cudaSuccess) return e;
    const int g = grid_for(nbytes / 2, ctas, 96);  // one CTA iteration per row
    KernelStamp* ks = timing_take(kIdEvictZF32, nbytes);
    k_evict_z<true><<<g, kThreads, kZStage, s>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), nbytes,
                                                 ebase, nullptr, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t restore_zf32(const void* src, void* dst, uint64_t nbytes, cudaStream_t s, int ctas) {
    if (!zf32::eligible(nbytes) || !aligned16(src) || !aligned16(dst)) return cudaErrorInvalidValue;
    cudaError_t e = allow_stage(reinterpret_cast<const void*>(&k_restore_zf32), 13);
    if (e != cudaSuccess) return e;
    const int g = grid_for(nbytes / 2, ctas, 96);
    KernelStamp* ks = timing_take(kIdRestoreZF32, nbytes);
    k_restore_zf32<<<g, kThreads, kZStage, s>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), nbytes,
                                                ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

__global__ void k_compare_digests(const uint64_t* __restrict__ got, const uint64_t* __restrict__ expect, uint64_t n,
                                  uint32_t* mismatch) {
    uint32_t bad = 0;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x)
        bad += got[i] != expect[i];
    if (bad) atomicAdd(mismatch, bad);
}

cudaError_t compare_digests(const uint64_t* got, const uint64_t* expect, uint64_t n, uint32_t* mismatch,
                            cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    if (!got || !expect || !mismatch) return cudaErrorInvalidValue;
    const int g = int(std::min<uint64_t>((n + 255) / 256, 148));
    k_compare_digests<<<g, 256, 0, s>>>(got, expect, n, mismatch);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t restore_z(const void* src, void* dst, uint64_t nbytes, Cast cast, float* scales, const uint64_t* expect,
                      uint32_t* mismatch, cudaStream_t s, int ctas) {
    if (!zbf16::eligible(nbytes) || !aligned16(src) || !aligned16(dst)) return cudaErrorInvalidValue;
    if (expect && !mismatch) return cudaErrorInvalidValue;
    const int g = grid_for(nbytes, ctas, 96);
    auto S = static_cast<const uint8_t*>(src);
    auto D = static_cast<uint8_t*>(dst);
    const bool v = expect != nullptr;
    const void* fn = nullptr;
    int id = 0;
    switch (cast) {
        case Cast::kNone: fn = v ? (const void*)&k_restore_z<true, 0> : (const void*)&k_restore_z<false, 0>; id = v ? 1 : 2; break;
        case Cast::kBf16ToFp8Block128:
            if (!scales) return cudaErrorInvalidValue;
            fn = v ? (const void*)&k_restore_z<true, 1> : (const void*)&k_restore_z<false, 1>;
            id = v ? 3 : 4;
            break;
        case Cast::kBf16ToFp32: fn = v ? (const void*)&k_restore_z<true, 3> : (const void*)&k_restore_z<false, 3>; id = v ? 5 : 6; break;
        default: return cudaErrorInvalidValue;  // coded objects are bf16
    }
    cudaError_t e = allow_stage(fn, id);
    if (e != cudaSuccess) return e;
    KernelStamp* ks = timing_take(kIdRestoreZ, nbytes);
    switch (cast) {
        case Cast::kNone:
            if (v) k_restore_z<true, 0><<<g, kThreads, kZStage, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
            else k_restore_z<false, 0><<<g, kThreads, kZStage, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
            break;
        case Cast::kBf16ToFp8Block128:
            if (v) k_restore_z<true, 1><<<g, kThreads, kZStage, s>>>(S, D, nbytes, scales, expect, mismatch, ks);
            else k_restore_z<false, 1><<<g, kThreads, kZStage, s>>>(S, D, nbytes, scales, nullptr, nullptr, ks);
            break;
        default:
            if (v) k_restore_z<true, 3><<<g, kThreads, kZStage, s>>>(S, D, nbytes, nullptr, expect, mismatch, ks);
            else k_restore_z<false, 3><<<g, kThreads, kZStage, s>>>(S, D, nbytes, nullptr, nullptr, nullptr, ks);
            break;
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t evict_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t s, int ctas) {
    if (njobs <= 0 || total_chunks == 0) return cudaSuccess;
    if (!jobs) return cudaErrorInvalidValue;
    cudaError_t e = allow_stage(reinterpret_cast<const void*>(&k_evict_jobs), 10);
    if (e != cudaSuccess) return e;
    int g = ctas > 0 ? ctas : 96;  // as evict_z
    if (uint64_t(g) > total_chunks) g = int(total_chunks);
    KernelStamp* ks = timing_take(kIdEvictJobs, total_chunks * kChunk);
    k_evict_jobs<<<g, kThreads, kZStage, s>>>(jobs, njobs, total_chunks, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t restore_jobs(const XferJob* jobs, int njobs, uint64_t total_chunks, cudaStream_t s, int ctas) {
    if (njobs <= 0 || total_chunks == 0) return cudaSuccess;
    if (!jobs) return cudaErrorInvalidValue;
    cudaError_t e = allow_stage(reinterpret_cast<const void*>(&k_restore_jobs), 11);
    if (e != cudaSuccess) return e;
    int g = ctas > 0 ? ctas : 96;
    if (uint64_t(g) > total_chunks) g = int(total_chunks);
    KernelStamp* ks = timing_take(kIdRestoreJobs, total_chunks * kChunk);
    k_restore_jobs<<<g, kThreads, kZStage, s>>>(jobs, njobs, total_chunks, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t fold_digests(const uint64_t* digests, uint64_t n, uint64_t nbytes, uint64_t* out, cudaStream_t s) {
    if (!out || (n && !digests)) return cudaErrorInvalidValue;
    k_fold<<<1, 32, 0, s>>>(digests, n, nbytes, out);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t verify_peer(const void* local, const void* peer, uint64_t nbytes, uint64_t* digests, uint32_t* mismatch,
                        cudaStream_t s, int ctas) {
    if (nbytes == 0) return cudaSuccess;
    if (!local || !peer || !mismatch) return cudaErrorInvalidValue;
    if (!aligned16(local) || !aligned16(peer) || nbytes % 16) return cudaErrorInvalidValue;
    const int g = grid_for(nbytes, ctas, 148 * 2);
    KernelStamp* ks = timing_take(kIdVerifyPeer, nbytes);
    k_verify_peer<<<g, kThreads, 0, s>>>(static_cast<const uint8_t*>(local), static_cast<const uint8_t*>(peer),
                                         nbytes, digests, mismatch, ks);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

cudaError_t quant_fp8_block(const void* src, void* dst, float* scales, uint64_t nelem, cudaStream_t s, int ctas) {
    if (nelem == 0) return cudaSuccess;
    if (!src || !dst || !scales || !aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7))
        return cudaErrorInvalidValue;
    uint64_t nvec = (nelem + 7) / 8;
    int g = ctas > 0 ? ctas : int(std::min<uint64_t>((nvec + kThreads - 1) / kThreads, 148 * 8));
    k_quant_fp8<<<g < 1 ? 1 : g, kThreads, 0, s>>>(static_cast<const uint4*>(src), static_cast<uint2*>(dst), scales,
                                                    nelem);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace ofld
