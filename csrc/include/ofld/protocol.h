// Control-plane messages of the offload runtime.
//
// Each message is a plain struct plus one `fields(V&, T&)` overload that lists
// its members in wire order. The same list drives encoding, decoding and the
// Python schema mirror (statespectre_b200/_wire.py), so field order is written
// down exactly once per language. Field order and types follow StateSpectre's
// protocol (reference: src/common/protocol.h:84-321, protocol_v2.h:29-326,
// wire.cpp:66-412, wire_v2.cpp:11-438) so frames are byte-compatible with it.
//
// Opcodes 1-13 (v1) and 20-30 (canonical v2) keep the reference numbering.
// Opcodes >= 40 are additive extensions of this runtime.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "ofld/abi/offload_abi.h"

namespace ofld {

constexpr uint32_t kRpcMagic = 0x4F465250u;  // "OFRP"
constexpr uint32_t kRpcWireVersion = 1u;

enum class Op : uint16_t {
    kInvalid = 0,
    kRegisterRank = 1,
    kHeartbeat = 2,
    kRequestOffload = 3,
    kMarkD2HSubmitted = 4,
    kMarkD2HComplete = 5,
    kRequestPrefetch = 6,
    kMarkH2DSubmitted = 7,
    kMarkH2DComplete = 8,
    kReleaseLease = 9,
    kQueryLocation = 10,
    kBatchComplete = 11,
    kShutdown = 12,
    kGetStats = 13,
    kRegisterJob = 20,
    kRequestCanonicalEvict = 21,
    kCommitCanonicalObject = 22,
    kSealModelVersion = 23,
    kGetLatestSealedVersion = 24,
    kGetManifest = 25,
    kPullTensor = 26,
    kRequestCanonicalRestore = 27,
    kReleaseCanonicalRestore = 28,
    kDropCanonicalVersion = 29,
    kReleaseCanonical = 30,
    // ---- extensions ----
    kBatchRequestOffload = 40,   // many reservations in one round trip
    kBatchRequestPrefetch = 41,  // many prefetches in one round trip
    kPublishPeerBuffer = 42,     // rank publishes a GPU buffer handle (fd via SCM_RIGHTS)
    kLookupPeerBuffer = 43,      // rank fetches a peer's buffer handle
    kGetJobStats = 44,           // per-job accounting export
    kExportManifest = 45,        // write a sealed manifest in ABI record format
    kDiscardTensor = 46,         // drop a tensor's pinned and cold copies by identity
    kCarryForward = 47,          // new-version objects that share an older version's storage
    kGetAgentOptions = 48,       // tuning the daemon config forwards to rank agents (kernels:, nvlink:)
    kBatchDiscardTensor = 49,    // DiscardTensor for many (tensor, version) pairs in one round trip
    kSetRunFormat = 50,          // record the coding (OFLD_FLAG_FORMAT_*) of a reserved run's bytes
};

const char* op_name(Op op);

enum class EventType : uint32_t {
    kNone = 0,
    kD2HComplete = 1,
    kH2DComplete = 2,
    kReadbackDone = 3,
    kDrainDone = 4,
    kError = 5,
};

// --------------------------------------------------------------------------
// v1 messages
// --------------------------------------------------------------------------
struct ArenaFd {
    uint64_t arena_id = 0;
    uint32_t numa_node = 0;
    uint32_t kind = 0;
    uint64_t size = 0;
    uint64_t base_offset = 0;
    uint32_t preferred_gpu = 0;
    uint64_t flags = 0;
    uint32_t fd_index = 0;
    uint32_t registration_granularity = 0;
    uint32_t allocation_granularity = 0;
};
template <class V> void fields(V& v, ArenaFd& m) {
    v(m.arena_id, m.numa_node, m.kind, m.size, m.base_offset, m.preferred_gpu, m.flags,
      m.fd_index, m.registration_granularity, m.allocation_granularity);
}

// RegisterRankRequest.capabilities bits.
constexpr uint64_t kCapMultiSession = 1ull << 0;  // process may hold several rank sessions

struct RegisterRankRequest {
    uint32_t rank_id = 0, local_rank = 0, world_rank = 0, gpu_id = 0, numa_node = 0;
    uint64_t pid = 0, capabilities = 0;
};
template <class V> void fields(V& v, RegisterRankRequest& m) {
    v(m.rank_id, m.local_rank, m.world_rank, m.gpu_id, m.numa_node, m.pid, m.capabilities);
}

struct RegisterRankResponse {
    bool ok = false;
    std::string message;
    uint64_t rank_epoch = 0, control_generation = 0;
    std::vector<ArenaFd> arenas;
    uint32_t control_fd_index = 0;
    uint64_t control_size = 0;
    uint32_t num_slots = 0;
    uint32_t ring_index = 0xFFFFFFFFu;
};
template <class V> void fields(V& v, RegisterRankResponse& m) {
    v(m.ok, m.message, m.rank_epoch, m.control_generation, m.arenas, m.control_fd_index,
      m.control_size, m.num_slots, m.ring_index);
}

struct HeartbeatRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, timestamp_ns = 0;
};
template <class V> void fields(V& v, HeartbeatRequest& m) {
    v(m.rank_id, m.rank_epoch, m.timestamp_ns);
}

// Responses that carry only (ok, message).
struct StatusResponse {
    bool ok = false;
    std::string message;
};
template <class V> void fields(V& v, StatusResponse& m) { v(m.ok, m.message); }
using HeartbeatResponse = StatusResponse;
using MarkD2HSubmittedResponse = StatusResponse;
using MarkH2DSubmittedResponse = StatusResponse;
using MarkH2DCompleteResponse = StatusResponse;
using ReleaseLeaseResponse = StatusResponse;
using ShutdownResponse = StatusResponse;
using ReleaseCanonicalRestoreResponse = StatusResponse;

struct RequestOffloadRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, tensor_id = 0, version = 0, nbytes = 0;
    uint32_t gpu_id = 0, numa_node = 0, alignment = 0, priority = 0;
    uint64_t flags = 0;
    std::string debug_name;
};
template <class V> void fields(V& v, RequestOffloadRequest& m) {
    v(m.rank_id, m.rank_epoch, m.tensor_id, m.version, m.nbytes, m.gpu_id, m.numa_node,
      m.alignment, m.priority, m.flags, m.debug_name);
}

struct RequestOffloadResponse {
    bool ok = false;
    std::string message;
    uint64_t lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t arena_id = 0, arena_offset = 0, capacity = 0;
    uint32_t state = 0;
    bool blocked = false;
};
template <class V> void fields(V& v, RequestOffloadResponse& m) {
    v(m.ok, m.message, m.lease_id, m.slot_id, m.arena_id, m.arena_offset, m.capacity, m.state,
      m.blocked);
}

// MarkD2HSubmitted / MarkD2HComplete / MarkH2DSubmitted share one body layout.
struct TransferMark {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, lease_id = 0, tensor_id = 0, version = 0;
    uint32_t slot_id = 0;
    uint64_t seq = 0, timestamp_ns = 0;
};
template <class V> void fields(V& v, TransferMark& m) {
    v(m.rank_id, m.rank_epoch, m.lease_id, m.tensor_id, m.version, m.slot_id, m.seq,
      m.timestamp_ns);
}
using MarkD2HSubmittedRequest = TransferMark;
using MarkD2HCompleteRequest = TransferMark;
using MarkH2DSubmittedRequest = TransferMark;

struct MarkD2HCompleteResponse {
    bool ok = false;
    std::string message;
    bool latest_version = false, drain_enqueued = false;
};
template <class V> void fields(V& v, MarkD2HCompleteResponse& m) {
    v(m.ok, m.message, m.latest_version, m.drain_enqueued);
}

struct RequestPrefetchRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, tensor_id = 0, version = 0, nbytes = 0;
    uint32_t gpu_id = 0, numa_node = 0, priority = 0;
    uint64_t flags = 0;
};
template <class V> void fields(V& v, RequestPrefetchRequest& m) {
    v(m.rank_id, m.rank_epoch, m.tensor_id, m.version, m.nbytes, m.gpu_id, m.numa_node,
      m.priority, m.flags);
}

struct RequestPrefetchResponse {
    bool ok = false;
    std::string message;
    uint64_t lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t arena_id = 0, arena_offset = 0, nbytes = 0;
    uint32_t state = 0;
    bool ready = false;
    uint64_t version = 0;
};
template <class V> void fields(V& v, RequestPrefetchResponse& m) {
    v(m.ok, m.message, m.lease_id, m.slot_id, m.arena_id, m.arena_offset, m.nbytes, m.state,
      m.ready, m.version);
}

struct MarkH2DCompleteRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, lease_id = 0, tensor_id = 0, version = 0;
    uint32_t slot_id = 0;
    bool keep_pinned = false;
    uint64_t seq = 0, timestamp_ns = 0;
};
template <class V> void fields(V& v, MarkH2DCompleteRequest& m) {
    v(m.rank_id, m.rank_epoch, m.lease_id, m.tensor_id, m.version, m.slot_id, m.keep_pinned,
      m.seq, m.timestamp_ns);
}

struct ReleaseLeaseRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, lease_id = 0;
    uint32_t slot_id = 0;
    std::string reason;
};
template <class V> void fields(V& v, ReleaseLeaseRequest& m) {
    v(m.rank_id, m.rank_epoch, m.lease_id, m.slot_id, m.reason);
}

struct LocationQueryRequest {
    uint64_t tensor_id = 0, version = 0;
};
template <class V> void fields(V& v, LocationQueryRequest& m) { v(m.tensor_id, m.version); }

struct LocationQueryResponse {
    bool ok = false;
    std::string message;
    uint32_t location_kind = 0, slot_id = 0;
    uint64_t nbytes = 0, version = 0;
};
template <class V> void fields(V& v, LocationQueryResponse& m) {
    v(m.ok, m.message, m.location_kind, m.slot_id, m.nbytes, m.version);
}

struct BatchCompletion {
    uint32_t event_type = 0;
    uint64_t lease_id = 0, tensor_id = 0, version = 0;
    uint32_t slot_id = 0;
    uint64_t seq = 0, timestamp_ns = 0;
    bool keep_pinned = false;
};
template <class V> void fields(V& v, BatchCompletion& m) {
    v(m.event_type, m.lease_id, m.tensor_id, m.version, m.slot_id, m.seq, m.timestamp_ns,
      m.keep_pinned);
}

struct BatchCompleteRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    std::vector<BatchCompletion> completions;
};
template <class V> void fields(V& v, BatchCompleteRequest& m) {
    v(m.rank_id, m.rank_epoch, m.completions);
}

struct BatchCompleteResponse {
    bool ok = false;
    std::string message;
    uint32_t accepted = 0, rejected = 0;
};
template <class V> void fields(V& v, BatchCompleteResponse& m) {
    v(m.ok, m.message, m.accepted, m.rejected);
}

struct GetStatsRequest {
    uint32_t rank_id = 0xFFFFFFFFu;
};
template <class V> void fields(V& v, GetStatsRequest& m) { v(m.rank_id); }

// One (name, value) pair; the wire interleaves key and value per entry.
struct StatEntry {
    std::string key;
    uint64_t value = 0;
};
template <class V> void fields(V& v, StatEntry& m) { v(m.key, m.value); }

struct GetStatsResponse {
    bool ok = false;
    std::string message;
    std::vector<StatEntry> stats;
};
template <class V> void fields(V& v, GetStatsResponse& m) { v(m.ok, m.message, m.stats); }

struct ShutdownRequest {
    uint64_t token = 0;
};
template <class V> void fields(V& v, ShutdownRequest& m) { v(m.token); }

// --------------------------------------------------------------------------
// v2 canonical model-state messages
// --------------------------------------------------------------------------
struct JobKeyWire {
    uint64_t tenant_id = 0, job_id = 0, launch_epoch = 0;
    std::string job_name;
};
template <class V> void fields(V& v, JobKeyWire& m) {
    v(m.tenant_id, m.job_id, m.launch_epoch, m.job_name);
}

struct RegisterJobRequest {
    uint64_t tenant_id = 0;
    std::string job_name;
    uint64_t scheduler_job_id = 0;
    std::vector<std::string> label_keys, label_values;
};
template <class V> void fields(V& v, RegisterJobRequest& m) {
    v(m.tenant_id, m.job_name, m.scheduler_job_id, m.label_keys, m.label_values);
}

struct RegisterJobResponse {
    bool ok = false;
    std::string message;
    JobKeyWire job;
    uint64_t control_generation = 0;
};
template <class V> void fields(V& v, RegisterJobResponse& m) {
    v(m.ok, m.message, m.job, m.control_generation);
}

// Identity of one logical model-state shard. dp_rank is deliberately absent:
// replicas across data parallelism share one identity and deduplicate.
struct CanonicalTensorKeyWire {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0, param_id = 0, param_fqn_hash = 0;
    std::string param_fqn_debug;
    uint32_t dtype = 0, layout = 0;
    uint64_t nbytes = 0, shape_hash = 0, stride_hash = 0;
    uint32_t pp_rank = 0, tp_rank = 0, ep_rank = 0, etp_rank = 0;
    int32_t expert_id = -1;
    uint64_t shard_offset = 0, shard_nbytes = 0;
};
template <class V> void fields(V& v, CanonicalTensorKeyWire& m) {
    v(m.job, m.model_role, m.model_version, m.param_id, m.param_fqn_hash, m.param_fqn_debug,
      m.dtype, m.layout, m.nbytes, m.shape_hash, m.stride_hash, m.pp_rank, m.tp_rank, m.ep_rank,
      m.etp_rank, m.expert_id, m.shard_offset, m.shard_nbytes);
}

struct RequestCanonicalEvictRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    CanonicalTensorKeyWire key;
    uint64_t local_tensor_id = 0, local_version = 0;
    bool destructive = true, attach_if_exists = true, create_if_missing = true;
    uint32_t dedup_mode = 0;
    bool allow_duplicate_candidate = false;
    uint32_t alignment = 0, priority = 0, gpu_id = 0, numa_node = 0;
};
template <class V> void fields(V& v, RequestCanonicalEvictRequest& m) {
    v(m.rank_id, m.rank_epoch, m.key, m.local_tensor_id, m.local_version, m.destructive,
      m.attach_if_exists, m.create_if_missing, m.dedup_mode, m.allow_duplicate_candidate,
      m.alignment, m.priority, m.gpu_id, m.numa_node);
}

struct RequestCanonicalEvictResponse {
    bool ok = false;
    std::string message;
    uint32_t action = 0;
    uint64_t object_id = 0, lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t arena_id = 0, arena_offset = 0, capacity = 0, synthetic_tid = 0;
};
template <class V> void fields(V& v, RequestCanonicalEvictResponse& m) {
    v(m.ok, m.message, m.action, m.object_id, m.lease_id, m.slot_id, m.arena_id,
      m.arena_offset, m.capacity, m.synthetic_tid);
}

struct CommitCanonicalObjectRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, object_id = 0, lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t content_hash_lo = 0, content_hash_hi = 0;
};
template <class V> void fields(V& v, CommitCanonicalObjectRequest& m) {
    v(m.rank_id, m.rank_epoch, m.object_id, m.lease_id, m.slot_id, m.content_hash_lo,
      m.content_hash_hi);
}

struct CommitCanonicalObjectResponse {
    bool ok = false;
    std::string message;
    uint64_t object_id = 0;
    bool won = true;
};
template <class V> void fields(V& v, CommitCanonicalObjectResponse& m) {
    v(m.ok, m.message, m.object_id, m.won);
}

struct SealModelVersionRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0;
    bool fail_if_missing = true;
    std::vector<uint64_t> expected_param_ids;
    bool promote = false;
};
template <class V> void fields(V& v, SealModelVersionRequest& m) {
    v(m.job, m.model_role, m.model_version, m.fail_if_missing, m.expected_param_ids, m.promote);
}

struct SealModelVersionResponse {
    bool ok = false;
    std::string message;
    uint32_t state = 0;
    uint64_t tensor_count = 0, total_nbytes = 0, manifest_hash_lo = 0, manifest_hash_hi = 0;
};
template <class V> void fields(V& v, SealModelVersionResponse& m) {
    v(m.ok, m.message, m.state, m.tensor_count, m.total_nbytes, m.manifest_hash_lo,
      m.manifest_hash_hi);
}

struct GetLatestSealedVersionRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
};
template <class V> void fields(V& v, GetLatestSealedVersionRequest& m) {
    v(m.job, m.model_role);
}

struct GetLatestSealedVersionResponse {
    bool ok = false;
    std::string message;
    bool found = false;
    uint64_t model_version = 0;
};
template <class V> void fields(V& v, GetLatestSealedVersionResponse& m) {
    v(m.ok, m.message, m.found, m.model_version);
}

struct ManifestFilterWire {
    bool pp_present = false;
    uint32_t pp_rank = 0;
    bool tp_present = false;
    uint32_t tp_rank = 0;
    bool ep_present = false;
    uint32_t ep_rank = 0;
    bool etp_present = false;
    uint32_t etp_rank = 0;
    bool expert_present = false;
    int32_t expert_id = 0;
};
template <class V> void fields(V& v, ManifestFilterWire& m) {
    v(m.pp_present, m.pp_rank, m.tp_present, m.tp_rank, m.ep_present, m.ep_rank,
      m.etp_present, m.etp_rank, m.expert_present, m.expert_id);
}

struct GetManifestRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0;
    ManifestFilterWire filter;
};
template <class V> void fields(V& v, GetManifestRequest& m) {
    v(m.job, m.model_role, m.model_version, m.filter);
}

struct TensorManifestEntryWire {
    CanonicalTensorKeyWire key;
    uint64_t object_id = 0, nbytes = 0, content_hash_lo = 0, content_hash_hi = 0;
    std::string location_hint;
};
template <class V> void fields(V& v, TensorManifestEntryWire& m) {
    v(m.key, m.object_id, m.nbytes, m.content_hash_lo, m.content_hash_hi, m.location_hint);
}

struct GetManifestResponse {
    bool ok = false;
    std::string message;
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0;
    uint32_t state = 0;
    std::vector<TensorManifestEntryWire> tensors;
};
template <class V> void fields(V& v, GetManifestResponse& m) {
    v(m.ok, m.message, m.job, m.model_role, m.model_version, m.state, m.tensors);
}

struct PullTensorRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0, object_id = 0;
    uint32_t transport = 0;
    std::string target_descriptor;
};
template <class V> void fields(V& v, PullTensorRequest& m) {
    v(m.job, m.model_role, m.model_version, m.object_id, m.transport, m.target_descriptor);
}

struct PullTensorResponse {
    bool ok = false;
    std::string message;
    uint64_t object_id = 0, nbytes = 0;
    uint32_t transport = 0;
    uint64_t content_hash_lo = 0, content_hash_hi = 0;
    std::string transport_metadata;
};
template <class V> void fields(V& v, PullTensorResponse& m) {
    v(m.ok, m.message, m.object_id, m.nbytes, m.transport, m.content_hash_lo, m.content_hash_hi,
      m.transport_metadata);
}

struct RequestCanonicalRestoreRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, object_id = 0;
    uint32_t gpu_id = 0, numa_node = 0;
};
template <class V> void fields(V& v, RequestCanonicalRestoreRequest& m) {
    v(m.rank_id, m.rank_epoch, m.object_id, m.gpu_id, m.numa_node);
}

struct RequestCanonicalRestoreResponse {
    bool ok = false;
    std::string message;
    bool retriable = false;
    uint64_t object_id = 0, nbytes = 0, arena_id = 0, arena_offset = 0;
};
template <class V> void fields(V& v, RequestCanonicalRestoreResponse& m) {
    v(m.ok, m.message, m.retriable, m.object_id, m.nbytes, m.arena_id, m.arena_offset);
}

struct ReleaseCanonicalRestoreRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, object_id = 0;
};
template <class V> void fields(V& v, ReleaseCanonicalRestoreRequest& m) {
    v(m.rank_id, m.rank_epoch, m.object_id);
}

struct DropCanonicalVersionRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0;
};
template <class V> void fields(V& v, DropCanonicalVersionRequest& m) {
    v(m.job, m.model_role, m.model_version);
}

struct DropCanonicalVersionResponse {
    bool ok = false;
    std::string message;
    uint64_t dropped_count = 0, skipped_inflight = 0, bytes_freed = 0;
};
template <class V> void fields(V& v, DropCanonicalVersionResponse& m) {
    v(m.ok, m.message, m.dropped_count, m.skipped_inflight, m.bytes_freed);
}

struct ReleaseCanonicalRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0, object_id = 0;
};
template <class V> void fields(V& v, ReleaseCanonicalRequest& m) {
    v(m.rank_id, m.rank_epoch, m.job, m.model_role, m.model_version, m.object_id);
}

struct ReleaseCanonicalResponse {
    bool ok = false;
    std::string message;
    uint64_t released_count = 0, freed_count = 0, bytes_freed = 0;
};
template <class V> void fields(V& v, ReleaseCanonicalResponse& m) {
    v(m.ok, m.message, m.released_count, m.freed_count, m.bytes_freed);
}

// --------------------------------------------------------------------------
// Extensions (opcodes >= 40)
// --------------------------------------------------------------------------
struct BatchRequestOffloadRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    std::vector<RequestOffloadRequest> items;
};
template <class V> void fields(V& v, BatchRequestOffloadRequest& m) {
    v(m.rank_id, m.rank_epoch, m.items);
}

struct BatchRequestOffloadResponse {
    bool ok = false;
    std::string message;
    std::vector<RequestOffloadResponse> grants;
};
template <class V> void fields(V& v, BatchRequestOffloadResponse& m) {
    v(m.ok, m.message, m.grants);
}

struct BatchRequestPrefetchRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    std::vector<RequestPrefetchRequest> items;
};
template <class V> void fields(V& v, BatchRequestPrefetchRequest& m) {
    v(m.rank_id, m.rank_epoch, m.items);
}

struct BatchRequestPrefetchResponse {
    bool ok = false;
    std::string message;
    std::vector<RequestPrefetchResponse> results;
};
template <class V> void fields(V& v, BatchRequestPrefetchResponse& m) {
    v(m.ok, m.message, m.results);
}

// A GPU buffer a rank shares with peers on the same node. `kind` 1 = CUDA IPC
// memory handle carried in `handle` (64 bytes); kind 2 = POSIX fd of a CUDA VMM
// allocation carried out of band via SCM_RIGHTS.
struct PeerBufferDesc {
    std::string key;
    uint32_t owner_rank = 0, device = 0, kind = 0;
    uint64_t nbytes = 0, offset = 0;
    std::string handle;
};
template <class V> void fields(V& v, PeerBufferDesc& m) {
    v(m.key, m.owner_rank, m.device, m.kind, m.nbytes, m.offset, m.handle);
}

struct PublishPeerBufferRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    PeerBufferDesc desc;
};
template <class V> void fields(V& v, PublishPeerBufferRequest& m) {
    v(m.rank_id, m.rank_epoch, m.desc);
}

struct LookupPeerBufferRequest {
    std::string key;
    uint32_t wait_ms = 0;
};
template <class V> void fields(V& v, LookupPeerBufferRequest& m) { v(m.key, m.wait_ms); }

struct LookupPeerBufferResponse {
    bool ok = false;
    std::string message;
    bool found = false;
    PeerBufferDesc desc;
};
template <class V> void fields(V& v, LookupPeerBufferResponse& m) {
    v(m.ok, m.message, m.found, m.desc);
}

// Carry-forward: for every object of `from_version` whose param_id is listed
// (all objects when the list is empty), create the same key at `to_version`
// sharing the old object's storage and content hash. No bytes move; the
// storage is freed when the last object that shares it is released.
// `shard`: only objects of this partition (pp, tp, ep, etp, expert) are
// carried; without it every partition of each listed parameter is.
struct CarryForwardRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t from_version = 0, to_version = 0;
    std::vector<uint64_t> param_ids;
    bool shard = false;
    uint32_t pp_rank = 0, tp_rank = 0, ep_rank = 0, etp_rank = 0;
    int32_t expert_id = -1;
};
template <class V> void fields(V& v, CarryForwardRequest& m) {
    v(m.rank_id, m.rank_epoch, m.job, m.model_role, m.from_version, m.to_version, m.param_ids, m.shard, m.pp_rank,
      m.tp_rank, m.ep_rank, m.etp_rank, m.expert_id);
}

struct CarryForwardResponse {
    bool ok = false;
    std::string message;
    uint32_t carried_count = 0, existing_count = 0, missing_count = 0;
    uint64_t bytes_shared = 0;
};
template <class V> void fields(V& v, CarryForwardResponse& m) {
    v(m.ok, m.message, m.carried_count, m.existing_count, m.missing_count, m.bytes_shared);
}

struct JobStatsEntry {
    JobKeyWire job;
    uint64_t pinned_bytes = 0, pageable_bytes = 0, nvme_bytes = 0, inflight_d2h_bytes = 0,
             inflight_export_bytes = 0, canonical_object_count = 0, dedup_bytes_saved = 0;
};
template <class V> void fields(V& v, JobStatsEntry& m) {
    v(m.job, m.pinned_bytes, m.pageable_bytes, m.nvme_bytes, m.inflight_d2h_bytes,
      m.inflight_export_bytes, m.canonical_object_count, m.dedup_bytes_saved);
}

struct GetJobStatsRequest {
    uint64_t tenant_id = 0;
    bool all_tenants = true;
};
template <class V> void fields(V& v, GetJobStatsRequest& m) { v(m.tenant_id, m.all_tenants); }

struct GetJobStatsResponse {
    bool ok = false;
    std::string message;
    std::vector<JobStatsEntry> jobs;
};
template <class V> void fields(V& v, GetJobStatsResponse& m) { v(m.ok, m.message, m.jobs); }

struct OptionEntry {
    std::string key, value;
};
template <class V> void fields(V& v, OptionEntry& m) { v(m.key, m.value); }

struct GetAgentOptionsRequest {
    uint32_t rank_id = 0;
    uint32_t gpu_id = 0;
};
template <class V> void fields(V& v, GetAgentOptionsRequest& m) { v(m.rank_id, m.gpu_id); }

struct GetAgentOptionsResponse {
    bool ok = false;
    std::string message;
    std::vector<OptionEntry> options;
};
template <class V> void fields(V& v, GetAgentOptionsResponse& m) { v(m.ok, m.message, m.options); }

struct ExportManifestRequest {
    JobKeyWire job;
    uint32_t model_role = 0;
    uint64_t model_version = 0;
    std::string path;
};
template <class V> void fields(V& v, ExportManifestRequest& m) {
    v(m.job, m.model_role, m.model_version, m.path);
}

struct DiscardTensorRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, tensor_id = 0, version = 0;
};
template <class V> void fields(V& v, DiscardTensorRequest& m) {
    v(m.rank_id, m.rank_epoch, m.tensor_id, m.version);
}

struct TensorVersion {
    uint64_t tensor_id = 0, version = 0;
};
template <class V> void fields(V& v, TensorVersion& m) { v(m.tensor_id, m.version); }

struct BatchDiscardTensorRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0;
    std::vector<TensorVersion> items;
};
template <class V> void fields(V& v, BatchDiscardTensorRequest& m) { v(m.rank_id, m.rank_epoch, m.items); }

struct BatchDiscardTensorResponse {
    bool ok = false;
    std::string message;
    std::vector<StatusResponse> results;
};
template <class V> void fields(V& v, BatchDiscardTensorResponse& m) { v(m.ok, m.message, m.results); }

// The rank that holds a reservation records how the bytes it copies into the
// run are coded (canonical evicts: their request has no flags field). Only
// before the copy is marked complete.
struct SetRunFormatRequest {
    uint32_t rank_id = 0;
    uint64_t rank_epoch = 0, lease_id = 0;
    uint32_t slot_id = 0;
    uint64_t format = 0;  // OFLD_FLAG_FORMAT_* bits (0 = raw)
};
template <class V> void fields(V& v, SetRunFormatRequest& m) {
    v(m.rank_id, m.rank_epoch, m.lease_id, m.slot_id, m.format);
}

struct ExportManifestResponse {
    bool ok = false;
    std::string message;
    uint64_t bytes_written = 0, tensor_count = 0;
};
template <class V> void fields(V& v, ExportManifestResponse& m) {
    v(m.ok, m.message, m.bytes_written, m.tensor_count);
}

}  // namespace ofld
