// Daemon/agent counters, bandwidth percentiles and the JSONL event trace.
//
// Counter names are the exported metric names (GetStats keys, Prometheus
// series) and match StateSpectre's set so existing dashboards keep working
// (reference: src/common/metrics.h:19-81, metrics.cpp:10-68). Counters added
// by this runtime are appended after the shared set.
#pragma once

#include <array>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

namespace ofld {

#define OFLD_METRICS(X)                                                        \
    X(kD2HBytes, "d2h_bytes")                                                  \
    X(kH2DBytes, "h2d_bytes")                                                  \
    X(kPinnedToPageableBytes, "pinned_to_pageable_bytes")                      \
    X(kPageableToPinnedBytes, "pageable_to_pinned_bytes")                      \
    X(kNvmeWriteBytes, "nvme_write_bytes")                                     \
    X(kNvmeReadBytes, "nvme_read_bytes")                                       \
    X(kUsedPinnedBytes, "used_pinned_bytes")                                   \
    X(kInflightD2HBytes, "inflight_d2h_bytes")                                 \
    X(kInflightH2DBytes, "inflight_h2d_bytes")                                 \
    X(kDrainingBytes, "draining_bytes")                                        \
    X(kPageableResidentBytes, "pageable_resident_bytes")                       \
    X(kNvmeResidentBytes, "nvme_resident_bytes")                               \
    X(kOffloadRequests, "offload_requests")                                    \
    X(kLeasesGranted, "leases_granted")                                        \
    X(kBlockedReservations, "blocked_reservation_count")                       \
    X(kRemoteNumaAllocs, "remote_numa_alloc_count")                            \
    X(kDrainsEnqueued, "drains_enqueued")                                      \
    X(kDrainsCompleted, "drains_completed")                                    \
    X(kPrefetchRequests, "prefetch_requests")                                  \
    X(kReadbacksStarted, "readbacks_started")                                  \
    X(kReadbacksCompleted, "readbacks_completed")                              \
    X(kInvalidTransitionRejected, "invalid_transition_rejected")               \
    X(kStaleVersionRejected, "stale_version_completion_rejected")              \
    X(kEpochMismatchRejected, "rank_epoch_mismatch_rejected")                  \
    X(kSlotOverlapPrevented, "slot_overlap_prevented")                         \
    X(kLeaseOwnerMismatchRejected, "lease_owner_mismatch_rejected")            \
    X(kChecksumMismatch, "checksum_mismatch")                                  \
    X(kIoFailure, "io_failure")                                                \
    X(kRankSessionsInvalidated, "rank_sessions_invalidated")                   \
    X(kJobsRegistered, "jobs_registered_total")                                \
    X(kCanonicalObjectsCreated, "canonical_objects_created_total")             \
    X(kCanonicalAttachExisting, "canonical_attach_existing_total")             \
    X(kCanonicalAttachWait, "canonical_attach_wait_total")                     \
    X(kCanonicalDuplicateCandidate, "canonical_duplicate_candidate_total")     \
    X(kCanonicalDedupBytesSaved, "canonical_dedup_bytes_saved")                \
    X(kCanonicalD2HBytesAvoided, "canonical_d2h_bytes_avoided")                \
    X(kCanonicalHashMismatch, "canonical_hash_mismatch_total")                 \
    X(kCanonicalStaleVersionReject, "canonical_stale_version_reject_total")    \
    X(kCanonicalRestoreServed, "canonical_restore_served_total")               \
    X(kCanonicalObjectsDropped, "canonical_objects_dropped_total")             \
    X(kQuotaRejections, "quota_rejections")                                    \
    X(kManifestSealed, "manifest_sealed_total")                                \
    X(kManifestSealFailed, "manifest_seal_failed_total")                       \
    X(kRolloutGetManifest, "rollout_get_manifest_total")                       \
    X(kRolloutPullTensor, "rollout_pull_tensor_total")                         \
    X(kRolloutPullBytes, "rollout_pull_bytes_total")                           \
    X(kRolloutStaleManifestReject, "rollout_stale_manifest_reject_total")      \
    X(kExportInflightBytes, "export_inflight_bytes")                           \
    X(kExportStagingBytes, "export_staging_bytes")                             \
    X(kExportFromPinned, "export_from_pinned_total")                           \
    X(kExportFromPageable, "export_from_pageable_total")                       \
    X(kExportFromNvme, "export_from_nvme_total")                               \
    X(kExportTransportErrors, "export_transport_errors_total")                 \
    /* ---- additions of this runtime ---- */                                  \
    X(kColdBytesReclaimed, "cold_bytes_reclaimed_total")                       \
    X(kPressureDrainsNormal, "pressure_drains_normal_total")                   \
    X(kPressureDrainsPriority, "pressure_drains_priority_total")               \
    X(kPressureDrainsAggressive, "pressure_drains_aggressive_total")           \
    X(kBatchOffloadItems, "batch_offload_items_total")                         \
    X(kBatchPrefetchItems, "batch_prefetch_items_total")                       \
    X(kPeerBuffersPublished, "peer_buffers_published_total")                   \
    X(kRingCompletionsApplied, "ring_completions_applied_total")                 \
    X(kVersionsPersisted, "versions_persisted_total")                          \
    X(kPersistedBytes, "persisted_bytes_total")                                \
    X(kVersionsRecovered, "versions_recovered_total")                          \
    X(kCanonicalP2PVerified, "canonical_p2p_verified_total")                   \
    X(kExportDecodedBytes, "export_decoded_bytes_total")                       \
    X(kPageableRoomRejected, "pageable_room_rejected_total")

enum class M : int {
#define OFLD_ENUM(id, name) id,
    OFLD_METRICS(OFLD_ENUM)
#undef OFLD_ENUM
        kCount
};

const char* metric_name(M m);

class Metrics {
 public:
    static Metrics& get();
    void add(M m, uint64_t v) { c_[int(m)].fetch_add(v, std::memory_order_relaxed); }
    void inc(M m) { add(m, 1); }
    void sub(M m, uint64_t v) {
        // Saturating subtraction: a gauge never wraps below zero.
        uint64_t cur = c_[int(m)].load(std::memory_order_relaxed);
        while (!c_[int(m)].compare_exchange_weak(cur, cur >= v ? cur - v : 0,
                                                 std::memory_order_relaxed)) {
        }
    }
    uint64_t value(M m) const { return c_[int(m)].load(std::memory_order_relaxed); }
    void record_mbps(double mbps);
    double mbps_percentile(double p) const;
    // name/value pairs of every counter, then bandwidth_mbps_p50/p90/p99.
    std::vector<std::pair<std::string, uint64_t>> snapshot() const;
    void reset();

 private:
    Metrics();
    std::array<std::atomic<uint64_t>, size_t(M::kCount)> c_;
    mutable std::mutex bw_mu_;
    std::vector<double> bw_ring_;
    size_t bw_next_ = 0;
};

// JSONL trace: one {"ts_ns",...,"event"} object per line, flushed per event.
// Enabled by offloadd --trace PATH or OFLD_TRACE.
class Trace {
 public:
    static Trace& get();
    void open(const std::string& path);
    void close();
    bool on() const { return fp_.load(std::memory_order_acquire) != nullptr; }
    void event(const char* name, uint32_t rank, uint32_t gpu, uint64_t tensor_id, uint64_t version,
               uint64_t lease_id, uint32_t slot_id, uint64_t nbytes);

 private:
    std::mutex mu_;
    std::atomic<FILE*> fp_{nullptr};
};

}  // namespace ofld
