// zbf16: lossless chunk coding of bf16 tensors for host transfers.
//
// PCIe (and the host memory behind it) is the bottleneck of evict/restore, so
// bf16 data crosses it coded: a bf16 value is sign(1) exponent(8) mantissa(7);
// sign and mantissa are near-random, but the exponents of weights,
// activations and KV caches cluster in a few binades. Per 64 KiB chunk
// (the same chunking as the ssh128 hash):
//
//   offset 0           header (16 bytes, below)
//   16                 low plane: one byte per element, (sign << 7) | mantissa
//   16 + n             code plane: one 4-bit code per element (element 2j in
//                      the low nibble of byte j): code = exponent - ebase when
//                      that is 0..14, else 15 (escape)
//   16 + n + n/2       escape bytes: the raw exponent of every escaped
//                      element, ordered by hash lane t = 0..255, then by the
//                      lane's vectors k*256 + t (k = 0..15), then by element
//                      within the 16-byte vector
//
// with n = len / 2 elements. The window is anchored at the top: ebase =
// max(emax - 14, 0) for the chunk's largest exponent emax, so only values
// more than 14 binades below the chunk's largest escape (for N(0, s) data a
// few per chunk). That is mode 1 (header mode byte 1, 12 bits per value).
//
// Mode 2 (header mode byte 2, 11 bits per value): the code plane holds 3-bit
// codes, 3 bytes per 16-byte source vector (the vector's 8 codes as one
// little-endian 24-bit value, element j in bits 3j..3j+2), and the window is
// the top 7 binades: base = ebase + 8 (mode 1's base plus 8, stored in the
// header), code = exponent - base when that is 0..6, else 7 (escape):
//
//   16                 low plane (n bytes, as in mode 1)
//   16 + n             code plane (3 * n / 8 bytes)
//   16 + n + 3n/8      escape bytes, in the same lane order as mode 1
//
// A chunk is stored in mode 2 when mode 1's base is above 0 and mode 2 is
// strictly shorter (it is for Gaussian-like data: the eighth binade below the
// top holds fewer than 1/8 of the values); ties and base 0 stay mode 1. The
// GPU pre-pass, the GPU coder and this reference apply the same rule, so the
// coded bytes are identical. A coded chunk must fit in its own raw length (so every byte of an object stays inside [0, nbytes)
// of its pinned run and tiers that copy nbytes keep it intact). A final
// chunk shorter than kRawTail bytes is stored raw (decided from nbytes
// alone). An object is coded only when every other chunk fits; the format is
// a property of the pinned run (OFLD_FLAG_FORMAT_ZBF16 on its slot entries).
//
// Typical ratio for N(0, s) bf16 data: 0.75 + escapes (a few per chunk).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <vector>

#include "ofld/chunk_hash.h"  // SSH_HD

namespace ofld {
namespace zbf16 {

constexpr uint32_t kChunk = 65536;
constexpr uint32_t kHeader = 16;
constexpr uint32_t kWindow = 15;
constexpr uint32_t kEscape = 15;
constexpr uint32_t kRawTail = 4096;  // a final chunk shorter than this is stored raw
constexpr uint32_t kLanes = 256;
constexpr uint32_t kVecsPerLane = 16;
constexpr uint16_t kTag = 0x425A;  // "ZB"

struct Header {
    uint16_t tag;
    uint8_t mode;  // 1 = coded
    uint8_t ebase;
    uint32_t n_esc;
    uint32_t src_len;
    uint32_t comp_len;
};
static_assert(sizeof(Header) == kHeader, "16-byte chunk header");

SSH_HD uint32_t exponent(uint16_t h) { return (h >> 7) & 0xFFu; }
SSH_HD uint8_t low_byte(uint16_t h) { return uint8_t(((h >> 8) & 0x80u) | (h & 0x7Fu)); }
SSH_HD uint32_t code_of(uint32_t e, uint32_t ebase) {
    const uint32_t d = e - ebase;  // wraps below ebase
    return d < kWindow ? d : kEscape;
}
SSH_HD uint16_t rebuild(uint8_t low, uint32_t e) {
    return uint16_t((uint32_t(low & 0x80u) << 8) | ((e & 0xFFu) << 7) | (low & 0x7Fu));
}
SSH_HD uint32_t coded_len(uint32_t len, uint32_t n_esc) {
    const uint32_t n = len / 2;
    return kHeader + n + n / 2 + n_esc;
}
// ---- mode 2: 3-bit codes over the top 7 binades -----------------------------
constexpr uint32_t kWindow3 = 7;
constexpr uint32_t kEscape3 = 7;
constexpr uint32_t kBase3Offset = 8;  // mode 2 base = mode 1 base + 8
SSH_HD uint32_t code3_of(uint32_t e, uint32_t base3) {
    const uint32_t d = e - base3;  // wraps below base3
    return d < kWindow3 ? d : kEscape3;
}
SSH_HD uint32_t coded_len3(uint32_t len, uint32_t n_esc3) {
    const uint32_t n = len / 2;
    return kHeader + n + (n / 8) * 3 + n_esc3;
}
// Mode 2 escapes from the mode-1 statistics of a chunk: the mode-1 escapes
// (below base or above base + 14, never above for a top-anchored base) plus
// the values in the lowest 8 binades of the mode-1 window.
SSH_HD uint32_t escapes3(uint32_t esc1, uint32_t low8) { return esc1 + low8; }
// Whether an element falls in the lowest 8 binades of the mode-1 window.
SSH_HD bool in_low8(uint32_t e, uint32_t ebase) { return e - ebase < kBase3Offset; }
// The stored mode and length of a chunk (the shared selection rule).
SSH_HD uint32_t choose_mode(uint32_t len, uint32_t ebase, uint32_t esc1, uint32_t low8, uint32_t* stored) {
    const uint32_t l1 = coded_len(len, esc1);
    const uint32_t l2 = coded_len3(len, escapes3(esc1, low8));
    if (ebase > 0 && l2 < l1) {
        *stored = l2;
        return 2;
    }
    *stored = l1;
    return 1;
}
// Whether chunk c (of `nchunks`, raw length len) is stored raw by rule.
SSH_HD bool raw_by_rule(uint64_t c, uint64_t nchunks, uint32_t len) { return c + 1 == nchunks && len < kRawTail; }
// Objects that can be coded at all: 16-byte multiple, at least one chunk.
SSH_HD bool eligible(uint64_t nbytes) { return nbytes >= kRawTail && nbytes % 16 == 0; }

// ---- host reference implementation (tests, tools) -------------------------

SSH_HD uint32_t window_base(uint32_t emax) { return emax >= kWindow - 1 ? emax - (kWindow - 1) : 0; }

// Elements of a chunk in escape order: lane t, vector k*256+t, element j.
template <class F>
inline void for_each_in_lane_order(uint32_t len, F&& f) {
    const uint32_t nvec = len / 16;
    for (uint32_t t = 0; t < kLanes; ++t)
        for (uint32_t k = 0; k < kVecsPerLane; ++k) {
            const uint32_t vi = k * kLanes + t;
            if (vi >= nvec) continue;
            for (uint32_t j = 0; j < 8; ++j) f(vi * 8 + j);
        }
}

// Code one chunk (len % 16 == 0). Returns the coded length, or 0 when the
// chunk does not fit in `len` bytes.
inline uint32_t encode_chunk(const uint8_t* src, uint32_t len, uint8_t* out) {
    const uint32_t n = len / 2;
    std::vector<uint16_t> h(n);
    std::memcpy(h.data(), src, len);
    uint32_t emax = 0;
    for (uint32_t i = 0; i < n; ++i) emax = exponent(h[i]) > emax ? exponent(h[i]) : emax;
    const uint32_t ebase = window_base(emax);
    uint32_t esc1 = 0, low8 = 0;
    for (uint32_t i = 0; i < n; ++i) {
        esc1 += code_of(exponent(h[i]), ebase) == kEscape;
        low8 += in_low8(exponent(h[i]), ebase);
    }
    uint32_t total = 0;
    const uint32_t mode = choose_mode(len, ebase, esc1, low8, &total);
    if (total > len) return 0;
    const uint32_t base = mode == 2 ? ebase + kBase3Offset : ebase;
    auto code = [&](uint32_t e) { return mode == 2 ? code3_of(e, base) : code_of(e, base); };
    const uint32_t escape = mode == 2 ? kEscape3 : kEscape;
    const uint32_t plane = mode == 2 ? (n / 8) * 3 : n / 2;
    Header hd{kTag, uint8_t(mode), uint8_t(base), total - (kHeader + n + plane), len, total};
    std::memcpy(out, &hd, kHeader);
    uint8_t* low = out + kHeader;
    uint8_t* codes = low + n;
    uint8_t* esc = codes + plane;
    std::memset(codes, 0, plane);
    for (uint32_t i = 0; i < n; ++i) {
        low[i] = low_byte(h[i]);
        const uint32_t cd = code(exponent(h[i]));
        if (mode == 2) {
            const uint32_t bit = (i / 8) * 24 + (i % 8) * 3;  // vector i/8, element i%8
            for (uint32_t b = 0; b < 3; ++b)
                codes[(bit + b) / 8] |= uint8_t(((cd >> b) & 1u) << ((bit + b) % 8));
        } else {
            codes[i / 2] |= uint8_t(cd << (4 * (i & 1)));
        }
    }
    uint32_t k = 0;
    for_each_in_lane_order(len, [&](uint32_t i) {
        if (code(exponent(h[i])) == escape) esc[k++] = uint8_t(exponent(h[i]));
    });
    return total;
}

// Decode one coded chunk into `len` bytes; false on a malformed chunk.
inline bool decode_chunk(const uint8_t* in, uint32_t len, uint8_t* out) {
    Header hd;
    std::memcpy(&hd, in, kHeader);
    if (hd.tag != kTag || (hd.mode != 1 && hd.mode != 2) || hd.src_len != len || hd.comp_len > len ||
        hd.comp_len != (hd.mode == 2 ? coded_len3(len, hd.n_esc) : coded_len(len, hd.n_esc)))
        return false;
    const uint32_t n = len / 2;
    const bool m2 = hd.mode == 2;
    const uint8_t* low = in + kHeader;
    const uint8_t* codes = low + n;
    const uint8_t* esc = codes + (m2 ? (n / 8) * 3 : n / 2);
    const uint32_t escape = m2 ? kEscape3 : kEscape;
    auto code_at = [&](uint32_t i) -> uint32_t {
        if (!m2) return (codes[i / 2] >> (4 * (i & 1))) & 15u;
        const uint32_t bit = (i / 8) * 24 + (i % 8) * 3;
        uint32_t c = 0;
        for (uint32_t b = 0; b < 3; ++b) c |= ((codes[(bit + b) / 8] >> ((bit + b) % 8)) & 1u) << b;
        return c;
    };
    std::vector<uint16_t> h(n);
    for (uint32_t i = 0; i < n; ++i) h[i] = rebuild(low[i], hd.ebase + code_at(i));  // escapes patched below
    uint32_t k = 0;
    bool ok = true;
    for_each_in_lane_order(len, [&](uint32_t i) {
        const uint32_t c = code_at(i);
        if (c == escape) {
            if (k >= hd.n_esc) {
                ok = false;
                return;
            }
            h[i] = rebuild(low[i], esc[k++]);
        }
    });
    if (!ok || k != hd.n_esc) return false;
    std::memcpy(out, h.data(), len);
    return true;
}

// The same decoding without the lane-order walk over every element and
// without allocation (the daemon decodes coded canonical objects on export):
// passes in element order rebuild every value from its window code and find
// the escaped elements; a counting pass over the 256 lanes then maps each to
// its escape byte. `keys` is caller scratch reused across calls.
inline bool decode_chunk_fast(const uint8_t* in, uint32_t len, uint8_t* out, std::vector<uint32_t>& keys) {
    Header hd;
    std::memcpy(&hd, in, kHeader);
    if (hd.tag != kTag || (hd.mode != 1 && hd.mode != 2) || hd.src_len != len || hd.comp_len > len || len % 16 ||
        hd.comp_len != (hd.mode == 2 ? coded_len3(len, hd.n_esc) : coded_len(len, hd.n_esc)))
        return false;
    const uint32_t n = len / 2;
    const bool m2 = hd.mode == 2;
    const uint8_t* low = in + kHeader;
    const uint8_t* codes = low + n;
    const uint8_t* esc = codes + (m2 ? (n / 8) * 3 : n / 2);
    const uint32_t ebase = hd.ebase;
    keys.clear();
    uint16_t* dst = reinterpret_cast<uint16_t*>(out);  // out is 2-byte aligned in every caller
    // Three simple passes the compiler vectorizes: every value's exponent
    // (window base + code) into a byte array, the rebuild of every value from
    // its low byte and exponent, and a memchr scan for the escape marker
    // (base + the all-ones code; its byte value cannot be a window exponent).
    uint8_t e8[kChunk / 2];
    const uint8_t eb = uint8_t(hd.ebase);
    if (!m2) {
        for (uint32_t j = 0; j < n / 2; ++j) {
            e8[2 * j] = uint8_t(eb + (codes[j] & 15u));
            e8[2 * j + 1] = uint8_t(eb + (codes[j] >> 4));
        }
    } else {
        for (uint32_t v = 0; v < n / 8; ++v) {
            const uint32_t w =
                uint32_t(codes[3 * v]) | (uint32_t(codes[3 * v + 1]) << 8) | (uint32_t(codes[3 * v + 2]) << 16);
            for (uint32_t j = 0; j < 8; ++j) e8[8 * v + j] = uint8_t(eb + ((w >> (3 * j)) & 7u));
        }
    }
    for (uint32_t i = 0; i < n; ++i)
        dst[i] = uint16_t((uint32_t(low[i] & 0x80u) << 8) | (uint32_t(e8[i]) << 7) | (low[i] & 0x7Fu));
    const uint8_t mark = uint8_t(eb + (m2 ? kEscape3 : kEscape));
    for (const uint8_t* q = e8; (q = static_cast<const uint8_t*>(std::memchr(q, mark, size_t(e8 + n - q)))) != nullptr;
         ++q) {
        if (keys.size() >= hd.n_esc) return false;
        keys.push_back(uint32_t(q - e8));
    }
    if (keys.size() != hd.n_esc) return false;
    // Escape order is lane-major (lane t = vector index mod 256, then the
    // lane's vectors, then elements); the scan above found them vector-major,
    // which within one lane is already that order. A counting pass over the
    // lanes gives each lane's first escape byte.
    uint32_t start[kLanes] = {};
    for (uint32_t i : keys) ++start[(i >> 3) & (kLanes - 1)];
    uint32_t acc = 0;
    for (uint32_t l = 0; l < kLanes; ++l) {
        const uint32_t c = start[l];
        start[l] = acc;
        acc += c;
    }
    for (uint32_t i : keys) {
        const uint32_t k = start[(i >> 3) & (kLanes - 1)]++;
        dst[i] = rebuild(low[i], esc[k]);
    }
    return true;
}

// Decode bytes [off, off + n) of a coded object of `nbytes` (format bits of
// OFLD_FLAG_FORMAT_*: 1 = zbf16, 2 = zf32) whose coded run is `in` (the run's
// bytes at the same offsets). `off` must be a multiple of the format's block
// (64 KiB zbf16 chunks, 128 KiB zf32 rows); n may end mid-object only at a
// block boundary or at nbytes. False on a malformed block.
enum class Coding : uint32_t { kZbf16 = 1, kZf32 = 2 };
inline bool decode_range(Coding fmt, const uint8_t* in, uint64_t nbytes, uint64_t off, uint64_t n, uint8_t* out,
                         std::vector<uint32_t>& keys) {
    const uint64_t block = fmt == Coding::kZf32 ? 2ull * kChunk : kChunk;
    if (off % block || off + n > nbytes || ((off + n) % block && off + n != nbytes)) return false;
    if (fmt == Coding::kZbf16) {
        const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
        for (uint64_t base = off; base < off + n; base += kChunk) {
            const uint64_t c = base / kChunk;
            const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
            if (raw_by_rule(c, nchunks, len)) {
                std::memcpy(out + (base - off), in + (base - off), len);
            } else if (!decode_chunk_fast(in + (base - off), len, out + (base - off), keys)) {
                return false;
            }
        }
        return true;
    }
    std::vector<uint8_t> hi(kChunk);
    for (uint64_t base = off; base < off + n; base += block) {
        const uint8_t* row = in + (base - off);
        uint8_t* dst = out + (base - off);
        if (!decode_chunk_fast(row + kChunk, kChunk, hi.data(), keys)) return false;
        for (uint32_t i = 0; i < kChunk / 2; ++i) {  // value i = top half i << 16 | low half i
            uint16_t h, l;
            std::memcpy(&h, hi.data() + 2 * i, 2);
            std::memcpy(&l, row + 2 * i, 2);
            const uint32_t w = (uint32_t(h) << 16) | l;
            std::memcpy(dst + 4 * i, &w, 4);
        }
    }
    return true;
}

// Whole objects at the 64 KiB stride. encode_object returns false (and
// leaves `out` unspecified) when the object is not codable.
inline bool encode_object(const uint8_t* src, uint64_t nbytes, uint8_t* out) {
    if (!eligible(nbytes)) return false;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = 0; c < nchunks; ++c) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        if (raw_by_rule(c, nchunks, len)) {
            std::memcpy(out + base, src + base, len);
            continue;
        }
        if (!encode_chunk(src + base, len, out + base)) return false;
    }
    return true;
}

inline bool decode_object(const uint8_t* in, uint64_t nbytes, uint8_t* out) {
    if (!eligible(nbytes)) return false;
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    for (uint64_t c = 0; c < nchunks; ++c) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        if (raw_by_rule(c, nchunks, len)) {
            std::memcpy(out + base, in + base, len);
            continue;
        }
        if (!decode_chunk(in + base, len, out + base)) return false;
    }
    return true;
}

// Bytes that actually carry data (what crosses PCIe), for statistics.
inline uint64_t coded_bytes(const uint8_t* in, uint64_t nbytes) {
    const uint64_t nchunks = (nbytes + kChunk - 1) / kChunk;
    uint64_t total = 0;
    for (uint64_t c = 0; c < nchunks; ++c) {
        const uint64_t base = c * kChunk;
        const uint32_t len = uint32_t(nbytes - base < kChunk ? nbytes - base : kChunk);
        if (raw_by_rule(c, nchunks, len)) {
            total += len;
        } else {
            Header hd;
            std::memcpy(&hd, in + base, kHeader);
            total += hd.comp_len;
        }
    }
    return total;
}

}  // namespace zbf16

// zf32: lossless coding of fp32 tensors for host transfers, built on zbf16.
//
// An fp32 value is the bf16 value of its top 16 bits (sign, exponent,
// 7 mantissa bits) followed by 16 low mantissa bits. The top halves carry
// the exponents and code like bf16 data; the low halves are near-random and
// travel as they are. Per 128 KiB row of the object (32768 values):
//
//   row + 0            low plane: the low 16 bits of every value, in order
//                      (64 KiB)
//   row + 65536        the zbf16 coded chunk (mode 1 or 2, header first) of
//                      the row's top halves, a 64 KiB bf16 chunk whose
//                      element i is the top half of value i
//
// A row occupies its own 128 KiB of the run, so every byte of an object stays
// inside [0, nbytes). Objects must be a whole number of rows (nbytes %
// 131072 == 0); an object is coded only when every row's top-half chunk
// codes (fits in 64 KiB). Typical ratio for N(0, s) fp32 data: 0.5 + 0.5 x
// the zbf16 ratio of the top halves (about 0.85). The format is a property
// of the pinned run (OFLD_FLAG_FORMAT_ZF32 on its slot entries).
namespace zf32 {

constexpr uint32_t kRow = 2 * zbf16::kChunk;
constexpr uint32_t kLowPlane = zbf16::kChunk;  // offset of the coded chunk in a row

SSH_HD bool eligible(uint64_t nbytes) { return nbytes >= kRow && nbytes % kRow == 0; }
SSH_HD uint64_t rows(uint64_t nbytes) { return nbytes / kRow; }

// Split one row of fp32 values into its top halves (`hi`, kChunk bytes) and
// low halves (`lo`, kChunk bytes).
inline void split_row(const uint8_t* src, uint8_t* hi, uint8_t* lo) {
    for (uint32_t i = 0; i < kRow / 4; ++i) {
        uint32_t w;
        std::memcpy(&w, src + 4 * i, 4);
        const uint16_t h = uint16_t(w >> 16), l = uint16_t(w & 0xFFFFu);
        std::memcpy(hi + 2 * i, &h, 2);
        std::memcpy(lo + 2 * i, &l, 2);
    }
}

inline void join_row(const uint8_t* hi, const uint8_t* lo, uint8_t* out) {
    for (uint32_t i = 0; i < kRow / 4; ++i) {
        uint16_t h, l;
        std::memcpy(&h, hi + 2 * i, 2);
        std::memcpy(&l, lo + 2 * i, 2);
        const uint32_t w = (uint32_t(h) << 16) | l;
        std::memcpy(out + 4 * i, &w, 4);
    }
}

// Whole objects. encode_object returns false (and leaves `out` unspecified)
// when the object is not codable.
inline bool encode_object(const uint8_t* src, uint64_t nbytes, uint8_t* out) {
    if (!eligible(nbytes)) return false;
    std::vector<uint8_t> hi(zbf16::kChunk);
    for (uint64_t r = 0; r < rows(nbytes); ++r) {
        const uint64_t base = r * kRow;
        split_row(src + base, hi.data(), out + base);
        if (!zbf16::encode_chunk(hi.data(), zbf16::kChunk, out + base + kLowPlane)) return false;
    }
    return true;
}

inline bool decode_object(const uint8_t* in, uint64_t nbytes, uint8_t* out) {
    if (!eligible(nbytes)) return false;
    std::vector<uint8_t> hi(zbf16::kChunk);
    for (uint64_t r = 0; r < rows(nbytes); ++r) {
        const uint64_t base = r * kRow;
        if (!zbf16::decode_chunk(in + base + kLowPlane, zbf16::kChunk, hi.data())) return false;
        join_row(hi.data(), in + base, out + base);
    }
    return true;
}

// Bytes that actually carry data (what crosses PCIe), for statistics.
inline uint64_t coded_bytes(const uint8_t* in, uint64_t nbytes) {
    uint64_t total = 0;
    for (uint64_t r = 0; r < rows(nbytes); ++r) {
        zbf16::Header hd;
        std::memcpy(&hd, in + r * kRow + kLowPlane, zbf16::kHeader);
        total += kLowPlane + hd.comp_len;
    }
    return total;
}

}  // namespace zf32
}  // namespace ofld
