// Rank agent: the per-process side of the offload runtime.
//
// Connects to offloadd, maps the shared arenas and control region, registers
// the arenas with CUDA once (host-mapped, so kernels address them directly),
// and moves tensor bytes with the sm_100a kernels (kernels.h): K1 for evict
// (copy + content hash in one pass), K2 for restore (copy + optional verify
// and cast). A progress thread retires asynchronous transfers and publishes
// completions through the shared completion ring; a heartbeat thread keeps
// the session alive. Host mode (device < 0) serves CPU tensors with memcpy
// and the host hash, so every control-plane path also runs without a GPU.
//
// Public API mirrors StateSpectre's OffloadAgent (reference:
// src/agent/agent.h:112-217); the header carries no CUDA or torch types.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "ofld/protocol.h"

namespace ofld {

using StreamHandle = uintptr_t;
constexpr StreamHandle kInternalStream = ~StreamHandle(0);
using DoneCallback = std::function<void()>;

struct AgentOptions {
    std::string socket_path = "/tmp/state_spectre.sock";
    int device = 0;  // CUDA device index; -1 = host mode
    uint32_t rank_id = 0, local_rank = 0, world_rank = 0;
    int numa_node = -1;  // -1: from the GPU's PCI affinity
    bool eager_register = false;
    uint64_t heartbeat_ms = 1000;
    uint64_t progress_poll_us = 50;
    uint64_t prefetch_poll_us = 200;
    std::string engine = "kernel";  // "kernel" (SM copies) | "copy_engine" (cudaMemcpyAsync)
    // How kernel mode moves the bytes it does not code (fp32, fp8, integer
    // and small or unaligned tensors, bf16 data that does not code):
    //   "copy_engine"  cudaMemcpyAsync, with the ssh128 chunk digests of an
    //                  evict computed at HBM rate on a side stream meanwhile
    //                  (default: SM-initiated PCIe traffic tops out ~7 % below
    //                  the copy engine on B200, in every instruction form);
    //   "bulk"         kern::evict_bulk / restore_bulk (bulk copies through
    //                  shared memory; aligned, size % 16 == 0);
    //   "sm"           per-thread K1 / K2.
    // Restores that verify digests or cast always run K2. In restore_batch,
    // "copy_engine" moves each uncoded item with its own copy and the other
    // forms put uncoded items into the group's job kernel with the coded ones;
    // evict_batch always uses the job kernel (one launch per group computes
    // every item's digests; per-item copies with digest kernels beside a
    // training step were 35 % slower for 4 MiB blocks).
    std::string uncoded = "copy_engine";
    // How a zbf16-coded run comes back: "copy_engine" (the copy engine moves
    // each chunk's stored bytes as one strided copy into device staging, in
    // pieces, while K2 decodes the previous piece from HBM; about 8 % more
    // host-read bandwidth than SM loads) or "sm" (K2 decodes straight from
    // host memory). The first needs the run's largest stored chunk, known to
    // the session that evicted it; restores that verify or cast use K2.
    std::string coded_restore = "copy_engine";
    // How a zbf16 evict leaves the GPU: "copy_engine" (K1 codes into device
    // staging at HBM rate, digests from the same pass, and the copy engine
    // moves each chunk's stored bytes, piece by piece, as strided copies) or
    // "sm" (K1 codes straight into the host-mapped run).
    std::string coded_evict = "copy_engine";
    int evict_ctas = 0, restore_ctas = 0, hash_ctas = 0;
    // CTAs of the staged (HBM to HBM) coding and decoding passes of the
    // copy-engine coded paths; 0 = auto.
    int stage_ctas = 0;
    // Staging ring of those paths: buffers (2..8) and 64 KiB chunks per
    // buffer; 0 = auto (2 x 512 chunks, 64 MiB of HBM).
    int stage_depth = 0;
    int stage_piece_chunks = 0;
    bool hash_on_evict = true;
    // Uncoded copy-engine evicts of at most this many bytes hash their pinned
    // copy on the host once the copy is done, instead of launching the digest
    // kernel on a side stream: beside a training step a tiny kernel waits for
    // SM room longer than the host takes to hash a few KB. 0 = always on the GPU.
    uint64_t host_hash_max_bytes = 16384;
    bool use_ring = true;
    bool fast_submit = true;     // reserve+submit and ready+submit in one round trip
    bool keep_digests = true;    // remember chunk digests for verify-on-restore
    bool zero_canonical_hash = false;  // commit hash 0 in trusted mode (manifest parity)
    int stream_priority = 0;     // internal stream priority (0 = default)
    // zbf16 coding of bf16 evictions (ofld/zbf16.h): fewer bytes over PCIe
    // and host memory. Applies to evict() calls that pass fmt_hint = kFmtBf16,
    // on objects of at least compress_min_bytes, in kernel-engine mode.
    bool compress = true;
    // The same coding for canonical objects of bf16 tensors (sealed versions,
    // DP dedup owners): offloadd records the run's coding and decodes it when
    // it exports the object, so TCP / FILE receivers get the raw bytes.
    bool compress_canonical = true;
    // Talk to StateSpectre's own offloadd: only its opcodes 1-30. Batches run
    // as one call per item, discard releases the tensor's lease, runs are not
    // coded (it keeps no run formats), reservations carry no submit flags and
    // completions go by RPC (it applies ring entries on its own schedule).
    // Calls that need this repository's daemon (carry-forward, job stats,
    // peer buffers) raise instead of waiting for an answer that never comes.
    bool v1_only = false;
    uint64_t compress_min_bytes = 4ull << 20;
    // evict_batch/restore_batch reserve and launch in groups of about this
    // many bytes: one daemon round trip and one kernel launch per group, the
    // round trip of the next group overlapping the copy of this one.
    uint64_t batch_group_bytes = 256ull << 20;
    // Device-side kernel timing (%globaltimer stamps into a host-mapped ring,
    // read with Agent::kernel_timings / statespectre_b200.Off.kernel_timings).
    bool kernel_timing = false;
    // Threads that register an arena with CUDA concurrently (pieces of at
    // least 1 GiB), when the GPU addresses registered memory by host pointer.
    // One by default: on B200 hosts measured 140 ms/GiB with one thread and
    // 159 ms/GiB with eight (the driver serializes the pinning).
    int registration_threads = 1;
    // How long evict() and evict_batch() keep retrying a reservation the
    // daemon answers as blocked (pinned window full, nothing drainable yet)
    // before failing.
    uint64_t blocked_wait_ms = 10000;
};

// evict() data hints.
constexpr uint32_t kFmtUnknown = 0;
constexpr uint32_t kFmtBf16 = 1;
constexpr uint32_t kFmtF32 = 2;  // fp32 payload: zf32 coding when it pays
// torch's ScalarType code of bfloat16, as canonical keys carry it
constexpr uint32_t kScalarBf16 = 15;

struct EvictTicket {
    bool ok = false;
    std::string message;
    uint64_t tensor_id = 0, version = 0, nbytes = 0, lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t hash_lo = 0, hash_hi = 0;  // valid once the copy completed (wait=true)
    bool coded = false;                  // moved in zbf16 coding
};

struct RestoreOptions {
    int cast = 0;               // kern::Cast
    uint64_t scales_ptr = 0;    // device fp32 scales for fp8 casts
    bool verify = false;        // re-hash while copying and compare with the evict-time digests
    bool keep_pinned = false;   // keep the pinned copy resident after H2D
};

struct RestoreOutcome {
    bool ok = false;
    std::string message;
    uint32_t mismatched_chunks = 0;
};

struct CanonicalOutcome {
    bool ok = false;
    std::string message;
    uint32_t action = 0;
    uint64_t object_id = 0;
    bool did_d2h = false;
    uint64_t hash_lo = 0, hash_hi = 0;
};

// One item of canonical_evict_batch.
struct CanonicalItem {
    uint64_t ptr = 0, nbytes = 0;
    RequestCanonicalEvictRequest req;
    DoneCallback on_invalidate;
};

struct AgentStats {
    uint32_t rank_id = 0;
    int gpu_id = -1, numa_node = 0;
    uint64_t registered_pinned_bytes = 0, inflight_d2h_bytes = 0, inflight_h2d_bytes = 0;
    uint64_t evict_count = 0, restore_count = 0, d2h_completed = 0, h2d_completed = 0;
    uint64_t rank_epoch = 0, num_slots = 0;
    uint64_t d2h_bytes = 0, h2d_bytes = 0, kernel_launches = 0, rpc_count = 0;
    uint64_t d2h_ns = 0, h2d_ns = 0;  // summed device time of completed copies (wait paths)
    uint64_t registration_ns = 0;     // host time spent registering arenas with CUDA
    uint64_t coded_canonical = 0;     // canonical objects that crossed PCIe zbf16-coded
};

struct BatchItem {
    uint64_t ptr = 0, nbytes = 0, tensor_id = 0, version = 0;
    uint32_t fmt_hint = 0;  // evict_batch: kFmtBf16 allows zbf16 coding
};

class Agent {
 public:
    explicit Agent(const AgentOptions& opt);
    ~Agent();
    Agent(const Agent&) = delete;
    Agent& operator=(const Agent&) = delete;

    // ---- v1 offload ----
    // Copy nbytes at `ptr` (device pointer, or host pointer in host mode) into
    // a pinned slot. `on_done` runs once the copy is complete (from the
    // progress thread, or inline when wait=true).
    EvictTicket evict(uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive, uint64_t tensor_id,
                      uint64_t version, const std::string& name, DoneCallback on_done, bool wait,
                      uint32_t fmt_hint = kFmtUnknown);
    // Many tensors with one reservation round trip (KV-cache blocks). All or
    // nothing per item; returns one ticket per item.
    std::vector<EvictTicket> evict_batch(const std::vector<BatchItem>& items, StreamHandle stream, bool wait);
    RestoreOutcome restore(uint64_t tensor_id, uint64_t version, uint64_t ptr, uint64_t nbytes, StreamHandle stream,
                           bool wait, const RestoreOptions& ro);
    std::vector<RestoreOutcome> restore_batch(const std::vector<BatchItem>& items, StreamHandle stream, bool wait);
    bool is_offloaded(uint64_t tensor_id, uint64_t version) const;
    void wait_offloaded(uint64_t tensor_id, uint64_t version);
    bool is_restored(uint64_t tensor_id, uint64_t version) const;
    void wait_restored(uint64_t tensor_id, uint64_t version);
    // Object hash recorded at evict time (0,0 when not hashed).
    bool tensor_hash(uint64_t tensor_id, uint64_t version, uint64_t* lo, uint64_t* hi) const;
    std::string location(uint64_t tensor_id, uint64_t version);
    void discard(uint64_t tensor_id, uint64_t version);
    // One round trip for many tensors; items still in a transfer are retried
    // together (bounded), like discard().
    void discard_batch(const std::vector<std::pair<uint64_t, uint64_t>>& items);
    void assert_no_inflight() const;
    void synchronize();

    // ---- canonical model state ----
    RegisterJobResponse register_job(const RegisterJobRequest& r);
    CanonicalOutcome canonical_evict(uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                                     const RequestCanonicalEvictRequest& req, DoneCallback on_invalidate, bool wait);
    // Many canonical evicts: all round trips and copies are issued before the
    // first completion is awaited (bounded by max_inflight_bytes, 0 = none).
    std::vector<CanonicalOutcome> canonical_evict_batch(const std::vector<CanonicalItem>& items, StreamHandle stream,
                                                        bool destructive, uint64_t max_inflight_bytes = 0);
    RestoreOutcome canonical_restore(uint64_t object_id, uint64_t ptr, uint64_t nbytes, StreamHandle stream,
                                     bool wait, const RestoreOptions& ro);
    SealModelVersionResponse seal(const SealModelVersionRequest& r);
    GetLatestSealedVersionResponse latest(const GetLatestSealedVersionRequest& r);
    GetManifestResponse manifest(const GetManifestRequest& r);
    PullTensorResponse pull(const PullTensorRequest& r);
    DropCanonicalVersionResponse drop_version(const DropCanonicalVersionRequest& r);
    // Objects of a new version that share the storage of an older version's
    // unchanged objects (rank id / epoch are filled in).
    CarryForwardResponse carry_forward(const CarryForwardRequest& r);
    ReleaseCanonicalResponse release(const ReleaseCanonicalRequest& r);
    ExportManifestResponse export_manifest(const ExportManifestRequest& r);
    GetJobStatsResponse job_stats(const GetJobStatsRequest& r);
    GetStatsResponse daemon_stats();
    StatusResponse publish_peer_buffer(const PeerBufferDesc& d, int fd);
    LookupPeerBufferResponse lookup_peer_buffer(const std::string& key, uint32_t wait_ms, int* fd_out);

    // ---- device utilities (GPU mode) ----
    // ssh128 of a device (or host, in host mode) buffer.
    void hash_buffer(uint64_t ptr, uint64_t nbytes, StreamHandle stream, uint64_t* lo, uint64_t* hi);
    uint64_t map_arena(uint64_t arena_id, uint64_t offset) const;  // host pointer of (arena, offset)

    AgentStats stats() const;
    std::string summary_string() const;
    int device() const;
    int numa_node() const;
    uint32_t rank_id() const;
    uint64_t rank_epoch() const;

    // Test hook: stop heartbeating (simulates a hung rank without killing it).
    void pause_heartbeat(bool paused);

    struct Impl;

 private:
    struct CanonPending;
    void canonical_request(CanonPending& c, uint64_t ptr, uint64_t nbytes, StreamHandle stream, bool destructive,
                           const RequestCanonicalEvictRequest& req, DoneCallback on_invalidate);
    void canonical_scan(std::vector<CanonPending*>& cs);
    void canonical_launch(CanonPending& c);
    void canonical_end(CanonPending& c);
    std::unique_ptr<Impl> d_;
};

}  // namespace ofld
