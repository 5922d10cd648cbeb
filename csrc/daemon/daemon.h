// offloadd: the node-level, CUDA-free offload daemon.
//
// Owns the NUMA-local pinned data arenas (memfd), the shared control region
// (slot table + completion rings), the slot allocator, leases and rank
// sessions, the tensor location table, the cold tiers (pageable DRAM and
// striped NVMe) with their drain/readback workers, and the canonical
// model-state store (jobs, deduplicated objects, sealed manifests, rollout
// export). Behaviour follows StateSpectre's daemon (reference:
// src/daemon/daemon.h:41-408, daemon.cpp, canonical.cpp, canonical_rollout.cpp);
// the data structures are this runtime's own:
//   * per-window free-slot bitmaps (word-at-a-time run search) instead of a
//     linear state scan,
//   * an LRU index of drainable runs so pressure relief is O(log n),
//   * an index of prefetch leases by (tensor, version) for idempotent re-polls,
//   * export streams straight from the pinned slot / pageable buffer / NVMe
//     extents in bounded chunks instead of staging a full heap copy.
//
// Locking: one mutex (mu_) guards every table. Workers copy metadata out under
// the lock, release it for memcpy/NVMe/network IO, and re-lock to commit.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "config.h"
#include "ofld/abi/offload_canonical_abi.hpp"
#include "ofld/codec.h"
#include "ofld/shm.h"

namespace ofld {

using namespace offload_v2;

// Synthetic tensor ids. Rank-assigned ids are (rank << 40 | counter) and never
// set bit 63; the daemon marks canonical objects with bit 63 and throwaway
// verification candidates with bits 63 and 62.
constexpr uint64_t kCanonicalTidBit = 1ull << 63;
constexpr uint64_t kCandidateTidBit = 1ull << 62;
inline uint64_t canonical_tid(uint64_t oid) { return kCanonicalTidBit | oid; }
inline bool is_canonical_tid(uint64_t t) { return (t & kCanonicalTidBit) != 0; }
inline bool is_candidate_tid(uint64_t t) { return (t & (kCanonicalTidBit | kCandidateTidBit)) == (kCanonicalTidBit | kCandidateTidBit); }

// Extension values (outside the interoperable enum ranges).
constexpr uint32_t kDedupDeviceHashVerified = 4;     // DedupMode extension
constexpr uint32_t kActionVerifyHashOnly = 6;        // AttachCreateAction extension
// Mode 5: the replica compared its bytes with the owner's GPU copy over NVLink
// (K3) before asking; an existing object is attached and answered with 7.
constexpr uint32_t kDedupP2PVerified = 5;            // DedupMode extension
constexpr uint32_t kActionVerifiedByP2P = 7;         // AttachCreateAction extension

struct JobUID {
    uint64_t tenant_id = 0, job_id = 0, launch_epoch = 0;
    bool operator==(const JobUID& o) const {
        return tenant_id == o.tenant_id && job_id == o.job_id && launch_epoch == o.launch_epoch;
    }
    bool operator<(const JobUID& o) const {
        if (tenant_id != o.tenant_id) return tenant_id < o.tenant_id;
        if (job_id != o.job_id) return job_id < o.job_id;
        return launch_epoch < o.launch_epoch;
    }
};

enum class JobState : uint32_t { kRegistered = 0, kRunning = 1, kDraining = 2, kTerminating = 3, kTerminated = 4 };

struct Job {
    JobUID uid;
    std::string name;
    JobState state = JobState::kRunning;
    uint64_t created_ns = 0;
    uint64_t pinned_bytes = 0, pageable_bytes = 0, nvme_bytes = 0;
    uint64_t inflight_d2h_bytes = 0, inflight_export_bytes = 0;
    uint64_t object_count = 0, dedup_bytes_saved = 0;
    uint32_t exports_in_flight = 0;
    uint64_t max_pinned = 0, max_pageable = 0, max_nvme = 0, max_inflight_d2h = 0, max_inflight_export = 0;
    std::vector<std::pair<std::string, std::string>> labels;
};

struct CanonicalObject {
    uint64_t object_id = 0;
    CanonicalTensorKeyWire key;
    std::string key_str;
    uint64_t nbytes = 0;
    CanonicalObjectState state = OBJ_MISSING;
    std::set<uint32_t> holders;  // ranks holding a reference (creator + attachers)
    uint32_t export_refs = 0;
    uint32_t restore_refs = 0;
    uint32_t producer_rank = 0;
    uint64_t hash_lo = 0, hash_hi = 0;
    uint64_t synthetic_tid = 0;
    uint64_t lease_id = 0;
    uint32_t base_slot = 0xFFFFFFFFu, slot_count = 0;
    CanonicalObjectState state_before_export = OBJ_SEALED;
    bool d2h_counted = false;  // counted in the job's inflight_d2h_bytes until its copy settles
    uint64_t created_ns = 0, sealed_ns = 0, last_access_ns = 0;
};

struct VersionKey {
    JobUID job;
    uint32_t role = 0;
    uint64_t version = 0;
    bool operator<(const VersionKey& o) const {
        if (!(job == o.job)) return job < o.job;
        if (role != o.role) return role < o.role;
        return version < o.version;
    }
};

struct Manifest {
    VersionKey vk;
    ManifestState state = MANIFEST_OPEN;
    std::vector<uint64_t> object_ids;  // sorted
    uint64_t total_nbytes = 0, created_ns = 0, sealed_ns = 0, hash_lo = 0, hash_hi = 0;
};

class Daemon {
 public:
    explicit Daemon(const DaemonConfig& cfg);
    ~Daemon();
    Daemon(const Daemon&) = delete;
    Daemon& operator=(const Daemon&) = delete;

    // Serve until stop() or a Shutdown RPC.
    void run();
    // Async-signal-safe stop request.
    void stop();
    bool running() const { return running_.load(); }
    // Block until the listener is up (for in-process harnesses).
    bool wait_ready(int timeout_ms) const;

    const DaemonConfig& config() const { return cfg_; }
    uint32_t num_slots() const { return layout_.num_slots; }
    // Test hook: inject an IO failure into the next `n` cold writes/reads.
    void inject_io_failures(int writes, int reads) {
        fail_writes_.store(writes);
        fail_reads_.store(reads);
    }
    // Test hook: report this many bytes of available host memory instead of
    // /proc/meminfo's MemAvailable (0 = the real figure).
    void fake_host_memory(uint64_t available) { fake_mem_available_.store(available); }
    // Test hook: stop (and resume) consuming the ranks' completion rings, so
    // a test can fill a ring and watch the agents fall back to RPCs.
    void pause_rings(bool paused) { rings_paused_.store(paused); }

 private:
    // ---------------- memory ----------------
    struct Arena {
        uint32_t numa_node = 0;
        uint64_t size = 0;
        int fd = -1;
        char* base = nullptr;
        uint32_t reg_gran = 0, alloc_gran = 0;
    };
    static constexpr uint32_t kOverflowGpu = 0xFFFFFFFFu;
    struct Window {
        uint32_t numa_node = 0, gpu = 0;
        bool overflow = false;
        uint32_t first_slot = 0, nslots = 0;
        std::vector<uint64_t> free_bits;  // bit set = slot free
    };
    struct Session {
        uint32_t rank_id = 0;
        uint64_t epoch = 0, pid = 0;
        uint32_t gpu = 0, numa = 0;
        uint64_t last_hb_ns = 0;
        bool alive = true;
        uint32_t ring = 0xFFFFFFFFu;
    };
    struct Lease {
        uint64_t id = 0;
        uint32_t base = 0, count = 0;
        uint64_t tensor_id = 0, version = 0;
        uint32_t owner_rank = 0;
        uint64_t owner_pid = 0, epoch = 0, nbytes = 0;
        bool prefetch = false;
        uint64_t lru_ts = 0;  // key of this lease's entry in lru_ (0 = none)
    };
    struct Location {
        uint64_t version = 0;
        ofld_location_kind_t kind = OFLD_LOC_NONE;
        uint32_t slot = 0;
        uint64_t cold_ref = 0, nbytes = 0;
        uint64_t fmt = 0;  // OFLD_FLAG_FORMAT_* of the stored bytes
    };
    struct Extent {
        std::string path;
        uint64_t offset = 0, length = 0;
    };
    struct ColdEntry {
        ofld_location_kind_t kind = OFLD_LOC_NONE;
        uint64_t nbytes = 0;
        char* pageable = nullptr;
        std::vector<Extent> extents;
        uint32_t readers = 0;     // unlocked readers in flight (readback/export)
        bool doomed = false;      // free once the last reader is done
        bool persisted = false;   // extents are a durable version file: unlink, do not punch
        uint64_t pageable_size = 0;  // mapping size of `pageable` (pool size class)
    };
    // A read hold on a canonical object's bytes (export, persistence): the
    // source is pinned against drains and frees until end_read.
    struct ReadSrc {
        const char* pinned = nullptr;
        ColdEntry cold;
        uint64_t cold_ref = 0, nbytes = 0;
        ofld_location_kind_t kind = OFLD_LOC_NONE;
        uint64_t fmt = 0;  // OFLD_FLAG_FORMAT_* of the stored bytes (exports decode them)
    };
    struct PeerBuffer {
        PeerBufferDesc desc;
        int fd = -1;
    };

    // ---------------- setup (daemon.cpp) ----------------
    void build_arenas();
    void build_control();
    void build_windows();
    void teardown();

    // ---------------- slots (slots.cpp) ----------------
    void set_state(uint32_t slot, ofld_slot_state_t st);
    void set_run_state(uint32_t base, uint32_t count, ofld_slot_state_t st);
    uint32_t state_of(uint32_t slot) const;
    void publish_slot(uint32_t slot);
    void set_cold_ref(uint32_t base, uint32_t count, uint64_t ref);
    char* slot_ptr(uint32_t slot);
    uint32_t slots_for(uint64_t nbytes) const;
    double pinned_pressure() const;
    bool alloc_in_window(Window& w, uint32_t count, uint32_t* base);
    bool allocate(uint32_t gpu, uint32_t numa, uint64_t nbytes, uint64_t flags, uint32_t* base,
                  uint32_t* count, std::unique_lock<std::mutex>& lk);
    void free_run(uint32_t base, uint32_t count);
    Window* window_of_slot(uint32_t slot);
    void stamp_run(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint64_t lease,
                   uint32_t rank, uint64_t pid, uint64_t epoch, uint64_t nbytes, uint64_t flags,
                   ofld_slot_state_t st);
    uint64_t new_lease(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint32_t rank,
                       uint64_t epoch, uint64_t nbytes, bool prefetch);
    void note_drainable(uint64_t lease_id);
    bool epoch_ok(uint32_t rank, uint64_t epoch);
    Lease* lease(uint64_t id);
    void erase_lease(uint64_t id);
    bool set_location(uint64_t tid, uint64_t ver, ofld_location_kind_t kind, uint32_t slot,
                      uint64_t cold_ref, uint64_t nbytes);

    RequestOffloadResponse do_request_offload(const RequestOffloadRequest& r, std::unique_lock<std::mutex>& lk);
    bool apply_d2h_complete(uint32_t rank, uint64_t epoch, uint64_t lease_id, uint64_t tid,
                            uint64_t ver, uint32_t slot, uint64_t seq, bool* latest, bool* drained);
    bool apply_h2d_complete(uint32_t rank, uint64_t epoch, uint64_t lease_id, uint64_t tid,
                            uint64_t ver, uint32_t slot, bool keep_pinned, uint64_t seq);
    RequestPrefetchResponse do_request_prefetch(const RequestPrefetchRequest& r, std::unique_lock<std::mutex>& lk);

    // ---------------- RPC handlers ----------------
    RegisterRankResponse on_register(const RegisterRankRequest& r, std::vector<int>* fds);
    StatusResponse on_heartbeat(const HeartbeatRequest& r);
    RequestOffloadResponse on_request_offload(const RequestOffloadRequest& r);
    StatusResponse on_d2h_submitted(const TransferMark& r);
    MarkD2HCompleteResponse on_d2h_complete(const TransferMark& r);
    RequestPrefetchResponse on_request_prefetch(const RequestPrefetchRequest& r);
    StatusResponse on_h2d_submitted(const TransferMark& r);
    StatusResponse on_h2d_complete(const MarkH2DCompleteRequest& r);
    StatusResponse on_release_lease(const ReleaseLeaseRequest& r);
    LocationQueryResponse on_query_location(const LocationQueryRequest& r);
    BatchCompleteResponse on_batch_complete(const BatchCompleteRequest& r);
    GetStatsResponse on_get_stats(const GetStatsRequest& r);
    StatusResponse on_shutdown(const ShutdownRequest& r);
    BatchRequestOffloadResponse on_batch_request_offload(const BatchRequestOffloadRequest& r);
    BatchRequestPrefetchResponse on_batch_request_prefetch(const BatchRequestPrefetchRequest& r);
    StatusResponse on_publish_peer_buffer(const PublishPeerBufferRequest& r, std::vector<int>* fds_in);
    LookupPeerBufferResponse on_lookup_peer_buffer(const LookupPeerBufferRequest& r, std::vector<int>* fds_out);
    GetJobStatsResponse on_get_job_stats(const GetJobStatsRequest& r);
    GetAgentOptionsResponse on_get_agent_options(const GetAgentOptionsRequest& r);
    StatusResponse on_discard_tensor(const DiscardTensorRequest& r);
    BatchDiscardTensorResponse on_batch_discard(const BatchDiscardTensorRequest& r);
    StatusResponse on_set_run_format(const SetRunFormatRequest& r);
    StatusResponse do_discard(uint32_t rank, uint64_t tid, uint64_t ver);  // mu_ held, epoch checked

    // canonical.cpp
    RegisterJobResponse on_register_job(const RegisterJobRequest& r);
    void init_job_quotas(Job& j) const;
    void settle_d2h(CanonicalObject& o);  // mu_ held: the creating copy is no longer in flight
    RequestCanonicalEvictResponse on_canonical_evict(const RequestCanonicalEvictRequest& r);
    CommitCanonicalObjectResponse on_commit_canonical(const CommitCanonicalObjectRequest& r);
    ReleaseCanonicalResponse on_release_canonical(const ReleaseCanonicalRequest& r);
    static std::string key_string(const CanonicalTensorKeyWire& k, bool cross_job);
    Job* find_job(const JobKeyWire& j);
    CanonicalObject* find_object(uint64_t oid);
    bool release_object(CanonicalObject& o);
    bool maybe_free_object(CanonicalObject& o);
    void purge_rank_holds(uint32_t rank);
    bool quota_allows_pinned(const Job& j, uint64_t nbytes) const;

    // rollout.cpp
    SealModelVersionResponse on_seal(const SealModelVersionRequest& r);
    CarryForwardResponse on_carry_forward(const CarryForwardRequest& r);
    GetLatestSealedVersionResponse on_get_latest(const GetLatestSealedVersionRequest& r);
    GetManifestResponse on_get_manifest(const GetManifestRequest& r);
    PullTensorResponse on_pull_tensor(const PullTensorRequest& r);
    RequestCanonicalRestoreResponse on_canonical_restore(const RequestCanonicalRestoreRequest& r);
    StatusResponse on_release_canonical_restore(const ReleaseCanonicalRestoreRequest& r);
    DropCanonicalVersionResponse on_drop_version(const DropCanonicalVersionRequest& r);
    ExportManifestResponse on_export_manifest(const ExportManifestRequest& r);
    void enforce_retention(const JobUID& job, uint32_t role);
    std::vector<uint64_t> objects_of_version(const JobUID& job, uint32_t role, uint64_t ver);

    // ---------------- sessions / connections (daemon.cpp) ----------------
    void recover_session(Session& s, const char* why);
    void accept_loop();
    void serve(int fd);
    void dispatch(int fd, Op op, const std::vector<uint8_t>& body, std::vector<int>& fds_in);
    void reap_connections(bool all);

    // ---------------- tiers (tiers.cpp) ----------------
    struct DrainJob {
        uint32_t base, count;
    };
    struct ReadbackJob {
        uint32_t base, count;
        uint64_t cold_ref, nbytes;
    };
    void drain_loop();
    void readback_loop();
    void heartbeat_loop();
    void ring_loop();

    // ---------------- pageable tier memory (tiers.cpp) ----------------
    // Anonymous mappings in 2 MiB size classes; freed ones are kept up to
    // drain_policy.pageable_pool_mb for reuse. Thread-safe.
    class PageablePool {
     public:
        char* get(uint64_t nbytes, uint64_t* size_out);
        void put(char* p, uint64_t size, uint64_t cap);
        ~PageablePool();
        uint64_t pooled() const { return pooled_.load(); }
     private:
        std::mutex mu_;
        std::multimap<uint64_t, char*> free_;
        std::atomic<uint64_t> pooled_{0};
    };
    PageablePool pageable_pool_;
    // Persistent memcpy threads shared by every drain and readback worker. A
    // copy of at least two pieces (1 MiB each) is split: the calling worker
    // copies one piece and pool threads take the rest, so a few concurrent
    // 4 MiB KV-block copies keep drain_policy.copy_threads + workers cores
    // busy without a thread start per copy.
    class CopyPool {
     public:
        void start(uint32_t threads);
        void stop();
        void copy(char* dst, const char* src, uint64_t n);
        // fn(0) .. fn(tasks - 1) over the pool threads and the caller; returns
        // when all have run (coded-object decoding on export uses it too).
        void run(uint32_t tasks, const std::function<void(uint32_t)>& fn);
        uint32_t threads() {
            std::lock_guard<std::mutex> g(mu_);
            return on_ ? uint32_t(ts_.size()) : 0;
        }
        ~CopyPool() { stop(); }
     private:
        struct Piece {
            const std::function<void(uint32_t)>* fn;
            uint32_t index;
            std::atomic<uint32_t>* left;
        };
        void run_piece(const Piece& p);
        std::mutex mu_;
        std::condition_variable cv_, done_cv_;
        std::deque<Piece> q_;
        std::vector<std::thread> ts_;
        bool on_ = false;
    };
    mutable CopyPool copy_pool_;
    void copy_bytes(char* dst, const char* src, uint64_t n) const;  // split over the copy pool

    // ---------------- read holds and durable versions (persist.cpp) ----------------
    bool begin_read(CanonicalObject& o, ReadSrc* src, std::string* why);  // mu_ held
    void end_read(uint64_t oid, const ReadSrc& src);                      // mu_ held
    bool copy_out(const ReadSrc& src, char* dst, uint64_t off, uint64_t n);  // no lock; stored bytes
    // Raw bytes [off, off + n) of a coded object from its stored bytes at the
    // same offsets, decoded in 1 MiB tasks over the copy pool (no lock).
    bool decode_out(const ReadSrc& src, const char* stored, uint64_t off, uint64_t n, char* out);
    // Sealed versions are written under manifest.persist_dir by a worker and
    // reloaded when a daemon starts on the same directory.
    static constexpr uint32_t kPersistHolder = 0xFFFFFFFEu;  // holder id that keeps persisted objects
    void enqueue_persist(const VersionKey& vk);               // mu_ held
    void persist_loop();
    int persist_version(const VersionKey& vk);                // 1 done, 0 retry later, -1 failed
    void recover_persisted();
    std::string persist_job_dir(const JobUID& uid) const;
    void unlink_persisted_manifest(const VersionKey& vk);    // mu_ held
    void forget_persisted_storage(uint64_t tid);             // mu_ held
    std::atomic<bool> rings_paused_{false};
    std::mutex persist_mu_;
    std::condition_variable persist_cv_;
    std::deque<VersionKey> persist_queue_;
    std::unordered_map<uint64_t, std::string> persisted_files_;  // storage tid -> file (mu_)
    // Applies every completion already published in the rings. mu_ held.
    void drain_rings();
    // Ring i of the control region, addressed from the daemon's own layout
    // (the copy of the geometry in the shared header is writable by ranks).
    RingHeader* ring(uint32_t i) const {
        return i < ring_max_ ? reinterpret_cast<RingHeader*>(static_cast<char*>(control_) + layout_.ring_offset +
                                                             uint64_t(i) * ring_stride_)
                             : nullptr;
    }
    // The live session the daemon assigned ring i to (never the owner and
    // epoch copies in the ring header, which its rank can write), or null.
    const Session* ring_session(uint32_t i) const;
    void apply_ring_entry(uint32_t rank, uint64_t epoch, const ofld_completion_entry_t& e);
    void enqueue_drain(const Lease& L);
    bool force_drain_one(std::unique_lock<std::mutex>& lk);
    void pressure_drain();
    void drain_settled(uint32_t base);  // a queued drain left the count (done, skipped or freed); mu_ held
    bool write_cold(const char* src, uint64_t nbytes, ColdEntry* out, bool allow_pageable, bool allow_nvme = true);
    // Cold tiers a drain of `tid` may use under its job's pageable / NVMe
    // quotas (both true for non-canonical tensors). mu_ held.
    void cold_quota(uint64_t tid, uint64_t nbytes, bool* allow_pageable, bool* allow_nvme);
    bool read_cold(const ColdEntry& c, char* dst, uint64_t off, uint64_t nbytes);
    void free_cold(uint64_t cold_ref);
    uint64_t commit_cold(ColdEntry&& c);
    // Keep a cold entry alive across an unlocked read; returns a descriptor
    // copy (not owning the pageable buffer) or false when absent.
    uint64_t reusable_cold(uint64_t tid, uint64_t ver);
    void finish_drain(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint64_t lid, uint32_t owner,
                      uint64_t nbytes, uint64_t ref);
    bool pin_cold(uint64_t cold_ref, ColdEntry* desc);
    void unpin_cold(uint64_t cold_ref);
    void discard_storage(ColdEntry& c);

    // nvme.cpp
    bool nvme_write(const char* src, uint64_t nbytes, std::vector<Extent>* out);
    bool nvme_read(const std::vector<Extent>& ext, char* dst, uint64_t off, uint64_t nbytes);
    void nvme_release(const std::vector<Extent>& ext);
    std::string stripe_path(uint32_t stripe) const;

    // ---------------- state ----------------
    DaemonConfig cfg_;
    uint64_t daemon_epoch_ = 0;
    std::vector<Arena> arenas_;
    int control_fd_ = -1;
    char* control_ = nullptr;
    ControlLayout layout_{};
    ofld_slot_table_header_t* header_ = nullptr;
    // The slot table. slots_ is the daemon's own copy, the one every decision
    // and every copy address is taken from; pub_slots_ is the table in the
    // shared control region, which ranks map writable and read (state,
    // flags). Each state change publishes the whole entry, its state last.
    std::unique_ptr<ofld_slot_entry_t[]> slot_store_;
    ofld_slot_entry_t* slots_ = nullptr;
    ofld_slot_entry_t* pub_slots_ = nullptr;
    uint32_t ring_max_ = 0, ring_cap_ = 0, ring_stride_ = 0;
    std::vector<Window> windows_;
    std::vector<uint32_t> slot_window_;  // slot -> window index

    mutable std::mutex mu_;
    std::unordered_map<uint32_t, Session> sessions_;
    std::unordered_map<uint64_t, Lease> leases_;
    std::unordered_map<uint64_t, Location> locations_;
    std::unordered_map<uint64_t, ColdEntry> cold_;
    std::set<std::pair<uint64_t, uint64_t>> lru_;            // (touch ns, lease id)
    std::map<std::pair<uint64_t, uint64_t>, uint64_t> prefetch_by_tv_;  // (tid, ver) -> lease
    std::vector<uint32_t> ring_owner_;
    uint64_t next_lease_ = 1, next_epoch_ = 1, next_cold_ = 1;
    uint64_t used_slots_ = 0;

    std::map<JobUID, Job> jobs_;
    std::unordered_map<uint64_t, CanonicalObject> objects_;
    // Canonical storage (keyed by synthetic tensor id) shared by the objects
    // of carried-forward versions: `objects` counts the objects that reference
    // it, `io` the exports / restores reading it across all of them.
    struct StorageRef {
        uint32_t objects = 0;
        uint32_t io = 0;
    };
    std::unordered_map<uint64_t, StorageRef> storage_;
    void storage_io(uint64_t tid, int delta);
    bool storage_busy(uint64_t tid) const;
    std::unordered_map<std::string, uint64_t> object_by_key_;
    std::map<VersionKey, Manifest> manifests_;
    std::map<std::pair<JobUID, uint32_t>, uint64_t> latest_sealed_;
    uint64_t next_object_ = 1, next_launch_epoch_ = 1;

    std::map<std::string, PeerBuffer> peer_buffers_;
    std::condition_variable peer_cv_;

    std::deque<DrainJob> drain_q_;
    std::deque<ReadbackJob> readback_q_;
    std::mutex q_mu_;
    std::condition_variable drain_cv_, readback_cv_;
    // Queued drains not yet finished (mu_), and the signal a blocked
    // reservation waits on for one of them to free its pinned run.
    uint32_t drains_pending_ = 0;
    uint64_t draining_slots_ = 0;  // slots of runs queued for or in a drain (still counted in used_slots_)
    std::unordered_map<uint32_t, uint32_t> drain_queued_;  // run base -> slots counted in draining_slots_
    std::condition_variable_any drained_cv_;

    std::vector<std::thread> workers_;
    struct Conn {
        int fd;
        std::thread th;
        std::shared_ptr<std::atomic<bool>> done;
    };
    std::mutex conn_mu_;
    std::list<Conn> conns_;

    int listen_fd_ = -1, tcp_fd_ = -1;
    int stop_pipe_[2] = {-1, -1};
    std::atomic<bool> running_{false}, workers_on_{false}, ready_{false};

    std::vector<std::atomic<uint64_t>> stripe_cursor_;
    uint32_t stripes_ = 1;
    std::atomic<int> fail_writes_{0}, fail_reads_{0};
    std::atomic<uint64_t> fake_mem_available_{0};
    // Whether the pageable tier can take `nbytes` more: within
    // drain_policy.pageable_limit_gb when set, else within the host memory
    // the kernel reports available (plus reusable pooled buffers), less a
    // reserve of max(4 GiB, 5 % of the host): anonymous memory is committed
    // only as the copy touches it, so an unchecked drain of tens of GB runs
    // the host out of memory and the kernel kills the daemon.
    bool pageable_room(uint64_t nbytes) const;
    // MemAvailable of /proc/meminfo in bytes (the test hook's figure when set;
    // 0 when unreadable).
    uint64_t host_memory_available() const;
};

}  // namespace ofld
