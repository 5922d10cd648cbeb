// "ssh128": the chunk-parallel 128-bit content hash of this runtime.
//
// Why a new hash: StateSpectre hashes objects with two byte-serial FNV-1a
// streams on the host (reference: src/daemon/canonical.cpp:84-95,
// src/agent/agent.cpp:57-68), which cannot run at GPU memory bandwidth. ssh128
// is defined so a GPU computes it in the same pass that moves the bytes, and a
// CPU computes the identical value (this header is the host oracle; the CUDA
// kernels include the same functions).
//
// Definition (all integers little-endian; arithmetic modulo 2^32 on u32 and
// 2^64 on u64; rotl = rotate left):
//   Constants (xxHash32 primes, Y. Collet, xxHash specification):
//     P1 = 2654435761, P2 = 2246822519, P3 = 3266489917, P4 = 668265263,
//     P5 = 374761393; G = 0x9E3779B97F4A7C15 (64-bit golden ratio).
//   fmix64(k) (MurmurHash3 finalizer, A. Appleby): k ^= k >> 33;
//     k *= 0xff51afd7ed558ccd; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53; k ^= k >> 33.
//   fold(a, b) = fmix64(a ^ (b * G)).
//   avalanche32(h) (xxHash32): h ^= h >> 15; h *= P2; h ^= h >> 13; h *= P3;
//     h ^= h >> 16.
//   * Bytes are split into chunks of 64 KiB; the last chunk may be short.
//   * A chunk is a sequence of 16-byte vectors of four u32 words w0..w3 (the
//     final vector zero-padded to 16 bytes). Vector v belongs to lane
//     (v mod 256); lane t sees vectors t, t+256, ..., at most 16 of them, in
//     that order. Lanes past the chunk's last vector see none.
//   * Lane t starts from seed = t * P5 + 0x9E3779B9 with accumulators
//     (a0, a1, a2, a3) = (seed + P1 + P2, seed + P2, seed, seed - P1) and, per
//     vector, applies the xxHash32 round to each word:
//     ai = rotl32(ai + wi * P2, 13) * P1.
//   * Lane digest (u64) = hi << 32 | lo, with
//     lo = avalanche32((rotl32(a0,1) + rotl32(a1,7) + rotl32(a2,12) + rotl32(a3,18)) ^ (t * P3)),
//     hi = avalanche32((rotl32(a0,3) ^ rotl32(a1,11) ^ rotl32(a2,17) ^ rotl32(a3,25)) + P4 + t).
//   * The 256 lane digests x[0..255] are reduced by a binary tree: for
//     s = 1, 2, 4, ..., 128, every i that is a multiple of 2s becomes
//     fold(x[i], x[i + s]); the root is x[0].
//     Chunk digest = fold(root, chunk length in bytes).
//   * Object hash of n bytes with chunk digests d0, d1, ...: start from
//     lo = 0xcbf29ce484222325, hi = 0x6a09e667f3bcc909; for each digest d in
//     order: lo = (lo ^ d) * 0x100000001b3; hi = rotl64(hi ^ d, 29) * G +
//     0x94d049bb133111eb. Result (fmix64(lo ^ n), fmix64(hi + n)); (0, 0) is
//     reserved for "no hash" and maps to (1, 0).
#pragma once

#include <cstdint>
#include <cstring>
#include <vector>

#ifdef __CUDACC__
#define SSH_HD __host__ __device__ __forceinline__
#else
#define SSH_HD inline
#endif

namespace ofld {
namespace ssh {

constexpr uint32_t kChunkBytes = 64u * 1024u;
constexpr uint32_t kLanes = 256;
constexpr uint32_t kVecBytes = 16;
constexpr uint32_t kVecsPerChunk = kChunkBytes / kVecBytes;    // 4096
constexpr uint32_t kVecsPerLane = kVecsPerChunk / kLanes;      // 16

constexpr uint32_t P1 = 2654435761u;
constexpr uint32_t P2 = 2246822519u;
constexpr uint32_t P3 = 3266489917u;
constexpr uint32_t P4 = 668265263u;
constexpr uint32_t P5 = 374761393u;
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

SSH_HD uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
SSH_HD uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

SSH_HD uint64_t fmix64(uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

SSH_HD uint64_t fold(uint64_t a, uint64_t b) { return fmix64(a ^ (b * kGolden)); }

struct Lane {
    uint32_t a0, a1, a2, a3;
};

SSH_HD Lane lane_init(uint32_t t) {
    uint32_t seed = t * P5 + 0x9E3779B9u;
    return Lane{seed + P1 + P2, seed + P2, seed, seed - P1};
}

SSH_HD uint32_t round32(uint32_t acc, uint32_t w) { return rotl32(acc + w * P2, 13) * P1; }

SSH_HD void lane_update(Lane& L, uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
    L.a0 = round32(L.a0, w0);
    L.a1 = round32(L.a1, w1);
    L.a2 = round32(L.a2, w2);
    L.a3 = round32(L.a3, w3);
}

SSH_HD uint32_t avalanche32(uint32_t h) {
    h ^= h >> 15;
    h *= P2;
    h ^= h >> 13;
    h *= P3;
    h ^= h >> 16;
    return h;
}

SSH_HD uint64_t lane_digest(const Lane& L, uint32_t t) {
    uint32_t lo = rotl32(L.a0, 1) + rotl32(L.a1, 7) + rotl32(L.a2, 12) + rotl32(L.a3, 18);
    lo = avalanche32(lo ^ (t * P3));
    uint32_t hi = rotl32(L.a0, 3) ^ rotl32(L.a1, 11) ^ rotl32(L.a2, 17) ^ rotl32(L.a3, 25);
    hi = avalanche32(hi + P4 + t);
    return (uint64_t(hi) << 32) | lo;
}

SSH_HD uint64_t chunk_finish(uint64_t root, uint32_t chunk_len) { return fold(root, chunk_len); }

struct Object {
    uint64_t lo, hi;
};

SSH_HD void object_init(uint64_t& lo, uint64_t& hi) {
    lo = 0xcbf29ce484222325ull;
    hi = 0x6a09e667f3bcc909ull;
}
SSH_HD void object_absorb(uint64_t& lo, uint64_t& hi, uint64_t d) {
    lo = (lo ^ d) * 0x100000001b3ull;
    hi = rotl64(hi ^ d, 29) * kGolden + 0x94d049bb133111ebull;
}
SSH_HD Object object_finish(uint64_t lo, uint64_t hi, uint64_t nbytes) {
    Object o{fmix64(lo ^ nbytes), fmix64(hi + nbytes)};
    if (o.lo == 0 && o.hi == 0) o.lo = 1;
    return o;
}

inline uint64_t num_chunks(uint64_t nbytes) { return (nbytes + kChunkBytes - 1) / kChunkBytes; }
SSH_HD uint64_t num_chunks_dev(uint64_t nbytes) { return (nbytes + kChunkBytes - 1) / kChunkBytes; }

// ---- host reference implementation -------------------------------------

// Digest of one chunk of `len` (<= kChunkBytes) bytes.
inline uint64_t host_chunk_digest(const uint8_t* p, uint32_t len) {
    uint64_t d[kLanes];
    uint32_t nvec = (len + kVecBytes - 1) / kVecBytes;
    for (uint32_t t = 0; t < kLanes; ++t) {
        Lane L = lane_init(t);
        for (uint32_t k = 0; k < kVecsPerLane; ++k) {
            uint32_t v = k * kLanes + t;
            if (v >= nvec) break;
            uint32_t w[4] = {0, 0, 0, 0};
            uint32_t off = v * kVecBytes;
            uint32_t take = len - off < kVecBytes ? len - off : kVecBytes;
            std::memcpy(w, p + off, take);
            lane_update(L, w[0], w[1], w[2], w[3]);
        }
        d[t] = lane_digest(L, t);
    }
    for (uint32_t s = 1; s < kLanes; s <<= 1)
        for (uint32_t i = 0; i < kLanes; i += 2 * s) d[i] = fold(d[i], d[i + s]);
    return chunk_finish(d[0], len);
}

inline void host_chunk_digests(const void* data, uint64_t nbytes, uint64_t* out) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    uint64_t n = num_chunks(nbytes);
    for (uint64_t c = 0; c < n; ++c) {
        uint64_t off = c * kChunkBytes;
        uint32_t len = uint32_t(nbytes - off < kChunkBytes ? nbytes - off : kChunkBytes);
        out[c] = host_chunk_digest(p + off, len);
    }
}

inline Object fold_digests(const uint64_t* d, uint64_t count, uint64_t nbytes) {
    uint64_t lo, hi;
    object_init(lo, hi);
    for (uint64_t i = 0; i < count; ++i) object_absorb(lo, hi, d[i]);
    return object_finish(lo, hi, nbytes);
}

inline Object host_hash(const void* data, uint64_t nbytes) {
    std::vector<uint64_t> d(num_chunks(nbytes));
    host_chunk_digests(data, nbytes, d.data());
    return fold_digests(d.data(), d.size(), nbytes);
}

}  // namespace ssh

// 64-bit FNV-1a over bytes: job-id derivation and the Python key hashes use
// this exact function (reference: python_api/state_spectre/__init__.py:89-102).
inline uint64_t fnv1a64(const void* data, size_t n, uint64_t seed = 1469598103934665603ull) {
    const uint8_t* b = static_cast<const uint8_t*>(data);
    uint64_t h = seed;
    for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

// Two seeded byte-serial FNV-1a streams: the interoperable 128-bit hash that
// StateSpectre ranks send on commit (reference: src/daemon/canonical.cpp:84-95).
// Used for job-id derivation and accepted as hash algorithm "fnv2" by the agent.
inline void fnv2_hash(const void* data, uint64_t n, uint64_t* lo, uint64_t* hi) {
    const uint8_t* b = static_cast<const uint8_t*>(data);
    uint64_t h1 = 1469598103934665603ull, h2 = 1099511628211ull;
    for (uint64_t i = 0; i < n; ++i) {
        h1 = (h1 ^ b[i]) * 1099511628211ull;
        h2 = (h2 ^ b[i]) * 1099511628211ull;
        h2 = (h2 << 1) | (h2 >> 63);
    }
    *lo = h1;
    *hi = h2;
}

}  // namespace ofld
