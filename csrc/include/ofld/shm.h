// Layout of the shared control region and the per-rank completion rings.
//
// Control region (one memfd, mapped by the daemon and every rank):
//   [header][arena descriptors][slot entries][completion rings]
// each section cache-line aligned and the total page aligned. The ring area
// holds one single-producer/single-consumer ring per rank session; ring
// geometry is published in header.reserved[0..11] as (max_ranks, stride,
// capacity). This layout is the interoperable format of record
// (reference: src/common/control_layout.h:42-84,
// src/common/completion_ring.h:33-121) so a rank built against either
// implementation can attach to the other's control region.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>

#include "ofld/abi/offload_abi.h"

namespace ofld {

inline constexpr uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

struct ControlLayout {
    uint64_t arena_desc_offset = 0;
    uint64_t slot_entries_offset = 0;
    uint64_t ring_offset = 0;
    uint64_t ring_bytes = 0;
    uint64_t total_bytes = 0;
    uint32_t num_arenas = 0;
    uint32_t num_slots = 0;
};

inline ControlLayout control_layout(uint32_t num_arenas, uint32_t num_slots, uint64_t ring_bytes) {
    ControlLayout L;
    L.num_arenas = num_arenas;
    L.num_slots = num_slots;
    L.ring_bytes = ring_bytes;
    uint64_t off = round_up(sizeof(ofld_slot_table_header_t), OFLD_CACHELINE);
    L.arena_desc_offset = off;
    off = round_up(off + uint64_t(num_arenas) * sizeof(ofld_arena_desc_t), OFLD_CACHELINE);
    L.slot_entries_offset = off;
    off = round_up(off + uint64_t(num_slots) * sizeof(ofld_slot_entry_t), OFLD_CACHELINE);
    L.ring_offset = off;
    L.total_bytes = round_up(off + ring_bytes, 4096);
    return L;
}

inline ofld_slot_table_header_t* header_of(void* base) {
    return static_cast<ofld_slot_table_header_t*>(base);
}
inline ofld_arena_desc_t* arena_descs_of(void* base) {
    auto* h = header_of(base);
    return reinterpret_cast<ofld_arena_desc_t*>(static_cast<char*>(base) + h->arena_desc_offset);
}
inline ofld_slot_entry_t* slots_of(void* base) {
    auto* h = header_of(base);
    return reinterpret_cast<ofld_slot_entry_t*>(static_cast<char*>(base) + h->slot_entries_offset);
}

// One rank's completion ring: header followed by `capacity` entries. head is
// advanced by the daemon (consumer), tail by the rank (producer); each on its
// own cache line. Indices are free-running u64; capacity is a power of two.
struct alignas(OFLD_CACHELINE) RingHeader {
    uint32_t capacity;
    uint32_t owner_rank;  // 0xFFFFFFFF = unassigned
    uint64_t rank_epoch;  // 0 = ring inactive
    alignas(OFLD_CACHELINE) std::atomic<uint64_t> head;
    alignas(OFLD_CACHELINE) std::atomic<uint64_t> tail;
};
static_assert(sizeof(RingHeader) == 192, "ring header layout is frozen");

struct RingGeometry {
    uint32_t max_ranks;
    uint32_t stride;
    uint32_t capacity;
    uint32_t pad;
};
static_assert(sizeof(RingGeometry) <= sizeof(((ofld_slot_table_header_t*)nullptr)->reserved),
              "ring geometry must fit the header's reserved bytes");

inline uint64_t ring_stride_bytes(uint32_t capacity) {
    return round_up(sizeof(RingHeader) + uint64_t(capacity) * sizeof(ofld_completion_entry_t),
                    OFLD_CACHELINE);
}
inline RingGeometry* ring_geometry(ofld_slot_table_header_t* h) {
    return reinterpret_cast<RingGeometry*>(h->reserved);
}
inline ofld_completion_entry_t* ring_entries(RingHeader* r) {
    return reinterpret_cast<ofld_completion_entry_t*>(reinterpret_cast<char*>(r) + sizeof(RingHeader));
}
inline RingHeader* ring_at(void* base, uint32_t index) {
    auto* h = header_of(base);
    const RingGeometry* g = ring_geometry(h);
    if (g->max_ranks == 0 || index >= g->max_ranks) return nullptr;
    return reinterpret_cast<RingHeader*>(static_cast<char*>(base) + h->control_ring_offset +
                                         uint64_t(index) * g->stride);
}

// Producer side (rank). False when the ring is full.
inline bool ring_push(RingHeader* r, const ofld_completion_entry_t& e) {
    uint64_t t = r->tail.load(std::memory_order_relaxed);
    if (t - r->head.load(std::memory_order_acquire) >= r->capacity) return false;
    ring_entries(r)[t & (r->capacity - 1)] = e;
    r->tail.store(t + 1, std::memory_order_release);
    return true;
}
// Consumer side (daemon). False when empty. The header sits in memory the
// producing rank maps writable, so the consumer indexes with the capacity it
// laid the ring out with, and a tail more than a ring ahead of the head
// (never written by a correct producer) discards the ring's contents rather
// than reading entries that were never published.
inline bool ring_pop(RingHeader* r, uint64_t capacity, ofld_completion_entry_t* out) {
    uint64_t h = r->head.load(std::memory_order_relaxed);
    const uint64_t t = r->tail.load(std::memory_order_acquire);
    if (h == t) return false;
    if (t - h > capacity) {
        r->head.store(t, std::memory_order_release);
        return false;
    }
    *out = ring_entries(r)[h & (capacity - 1)];
    r->head.store(h + 1, std::memory_order_release);
    return true;
}
inline bool ring_pop(RingHeader* r, ofld_completion_entry_t* out) { return ring_pop(r, r->capacity, out); }

}  // namespace ofld
