/*
 * Shared-memory ABI of the offload runtime (version 1).
 *
 * Every struct here lives in memory shared between the daemon and every rank
 * process (memfd mappings passed over AF_UNIX). The layout is frozen: sizes,
 * offsets and enum values are the on-shm format of record and must stay
 * interoperable with ranks built from StateSpectre's abi/offload_abi.h
 * (reference: abi/offload_abi.h:25-150). The static_asserts at the bottom pin
 * every offset so an accidental edit fails the build instead of corrupting a
 * live control region.
 *
 * Rule: shared memory never holds process-local pointers; a location is
 * (arena_id, arena_offset) and each process adds its own mapping base.
 *
 * Atomic fields use std::atomic<T> in C++ and _Atomic T in C; both have the
 * plain integer's size, alignment and representation for the lock-free widths
 * used here.
 */
#ifndef OFLD_ABI_OFFLOAD_ABI_H_
#define OFLD_ABI_OFFLOAD_ABI_H_

#include <stdint.h>

#ifdef __cplusplus
#include <atomic>
#define OFLD_ATOMIC(T) std::atomic<T>
#else
#include <stdatomic.h>
#define OFLD_ATOMIC(T) _Atomic T
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define OFLD_MAGIC 0x4F464C44u /* "OFLD" little-endian */
#define OFLD_ABI_VERSION 1u
#define OFLD_CACHELINE 64u

typedef uint64_t ofld_tensor_id_t;
typedef uint64_t ofld_version_t;
typedef uint64_t ofld_lease_id_t;
typedef uint32_t ofld_slot_id_t;
typedef uint64_t ofld_arena_id_t;

/* Slot lifecycle. D2H side: FREE -> RESERVED_D2H -> D2H_IN_FLIGHT ->
 * PINNED_VALID -> DRAIN_IN_FLIGHT -> COLD_VALID. H2D side: PINNED_VALID ->
 * H2D_IN_FLIGHT -> PINNED_VALID | FREE; cold readback goes through
 * READBACK_IN_FLIGHT. */
typedef enum ofld_slot_state_e {
    OFLD_SLOT_FREE = 0,
    OFLD_SLOT_RESERVED_D2H = 1,
    OFLD_SLOT_D2H_IN_FLIGHT = 2,
    OFLD_SLOT_PINNED_VALID = 3,
    OFLD_SLOT_DRAIN_IN_FLIGHT = 4,
    OFLD_SLOT_COLD_VALID = 5,
    OFLD_SLOT_RESERVED_H2D = 6,
    OFLD_SLOT_READBACK_IN_FLIGHT = 7,
    OFLD_SLOT_H2D_IN_FLIGHT = 8,
    OFLD_SLOT_GPU_VALID = 9,
    OFLD_SLOT_ERROR = 255
} ofld_slot_state_t;

typedef enum ofld_location_kind_e {
    OFLD_LOC_NONE = 0,
    OFLD_LOC_GPU = 1,
    OFLD_LOC_PINNED = 2,
    OFLD_LOC_PAGEABLE = 3,
    OFLD_LOC_NVME = 4,
    OFLD_LOC_DELETED = 5,
    OFLD_LOC_ERROR = 255
} ofld_location_kind_t;

typedef enum ofld_arena_kind_e {
    OFLD_ARENA_DATA_PINNED = 1,
    OFLD_ARENA_CONTROL = 2,
    OFLD_ARENA_OVERFLOW = 3
} ofld_arena_kind_t;

/* Request flags. Bits 0-5 are the interoperable set; bits >= 16 are
 * extensions of this runtime that older daemons store and ignore. */
#define OFLD_FLAG_NONE 0ull
#define OFLD_FLAG_ALLOW_OVERFLOW (1ull << 0)
#define OFLD_FLAG_ALLOW_REMOTE_NUMA (1ull << 1)
#define OFLD_FLAG_BORROWABLE (1ull << 2)
#define OFLD_FLAG_DESTRUCTIVE (1ull << 3)
#define OFLD_FLAG_VIEW_COMPACT (1ull << 4)
#define OFLD_FLAG_UNSAFE_AUTOGRAD (1ull << 5)
/* Extension: the grant moves the run straight to D2H_IN_FLIGHT (saves the
 * MarkD2HSubmitted round trip). */
#define OFLD_FLAG_SUBMIT_ON_GRANT (1ull << 16)
/* Extension: a ready prefetch moves the run straight to H2D_IN_FLIGHT. */
#define OFLD_FLAG_SUBMIT_ON_READY (1ull << 17)
/* Extension: the run holds the object in zbf16 chunk coding (ofld/zbf16.h).
 * Set by the rank at reservation, stamped on the run's slot entries, kept
 * across drains and readbacks; readers decode. */
#define OFLD_FLAG_FORMAT_ZBF16 (1ull << 18)
/* Extension: the run holds an fp32 object in zf32 coding (ofld/zbf16.h),
 * carried like OFLD_FLAG_FORMAT_ZBF16. */
#define OFLD_FLAG_FORMAT_ZF32 (1ull << 19)
#define OFLD_FLAG_FORMAT_MASK (OFLD_FLAG_FORMAT_ZBF16 | OFLD_FLAG_FORMAT_ZF32)

typedef struct ofld_arena_desc_s {
    ofld_arena_id_t arena_id;
    uint64_t base_offset;
    uint64_t size;
    uint32_t numa_node;
    uint32_t kind;
    uint32_t registration_granularity;
    uint32_t allocation_granularity;
    uint32_t preferred_gpu;
    uint64_t flags;
    uint8_t reserved[24];
} ofld_arena_desc_t;

typedef struct ofld_slot_entry_s {
    OFLD_ATOMIC(uint32_t) state;
    ofld_slot_id_t slot_id;
    uint32_t numa_node;
    uint32_t gpu_preferred;

    ofld_arena_id_t arena_id;
    uint64_t arena_offset;
    uint64_t capacity;
    uint64_t nbytes;

    ofld_tensor_id_t tensor_id;
    ofld_version_t version;
    ofld_lease_id_t lease_id;
    uint64_t owner_rank;

    uint64_t owner_pid;
    uint64_t rank_epoch;
    uint64_t flags;
    uint64_t cold_ref;

    uint64_t checksum;
    uint64_t last_touch_ns;
    uint64_t submit_seq;
    uint64_t complete_seq;

    uint8_t reserved[64];
} __attribute__((aligned(OFLD_CACHELINE))) ofld_slot_entry_t;

typedef struct ofld_slot_table_header_s {
    uint32_t magic;
    uint32_t abi_version;
    uint32_t num_slots;
    uint32_t num_arenas;

    uint64_t generation;
    uint64_t daemon_pid;
    uint64_t daemon_epoch;
    OFLD_ATOMIC(uint64_t) heartbeat_ns;

    uint64_t flags;
    uint64_t arena_desc_offset;
    uint64_t slot_entries_offset;
    uint64_t control_ring_offset;

    uint8_t reserved[64];
} __attribute__((aligned(OFLD_CACHELINE))) ofld_slot_table_header_t;

typedef struct ofld_completion_entry_s {
    ofld_lease_id_t lease_id;
    ofld_tensor_id_t tensor_id;
    ofld_version_t version;
    ofld_slot_id_t slot_id;
    uint32_t event_type;
    uint64_t timestamp_ns;
} ofld_completion_entry_t;

#ifdef __cplusplus
}  /* extern "C" */

#include <cstddef>
static_assert(sizeof(ofld_arena_desc_t) == 80, "arena desc size is frozen");
static_assert(offsetof(ofld_arena_desc_t, numa_node) == 24, "arena desc layout");
static_assert(offsetof(ofld_arena_desc_t, flags) == 48, "arena desc layout");
static_assert(sizeof(ofld_slot_entry_t) == 256, "slot entry size is frozen");
static_assert(offsetof(ofld_slot_entry_t, arena_id) == 16, "slot entry layout");
static_assert(offsetof(ofld_slot_entry_t, tensor_id) == 48, "slot entry layout");
static_assert(offsetof(ofld_slot_entry_t, owner_pid) == 80, "slot entry layout");
static_assert(offsetof(ofld_slot_entry_t, checksum) == 112, "slot entry layout");
static_assert(offsetof(ofld_slot_entry_t, reserved) == 144, "slot entry layout");
static_assert(sizeof(ofld_slot_table_header_t) == 192, "header size is frozen");
static_assert(offsetof(ofld_slot_table_header_t, generation) == 16, "header layout");
static_assert(offsetof(ofld_slot_table_header_t, heartbeat_ns) == 40, "header layout");
static_assert(offsetof(ofld_slot_table_header_t, control_ring_offset) == 72, "header layout");
static_assert(offsetof(ofld_slot_table_header_t, reserved) == 80, "header layout");
static_assert(sizeof(ofld_completion_entry_t) == 40, "completion entry size is frozen");
#endif

#endif /* OFLD_ABI_OFFLOAD_ABI_H_ */
