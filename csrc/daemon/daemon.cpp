// Daemon construction, connection serving, dispatch, rank sessions, heartbeat
// monitoring and the completion-ring poller.
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "daemon.h"

#include <fcntl.h>
#include <poll.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <cerrno>
#include <cstring>
#include <stdexcept>

#include "ofld/log.h"
#include "ofld/metrics.h"
#include "ofld/numa.h"
#include "ofld/transport.h"

namespace ofld {

namespace {
constexpr const char* TAG = "offloadd";

int make_memfd(const char* name) {
    int fd = static_cast<int>(::syscall(SYS_memfd_create, name, 1u /* MFD_CLOEXEC */));
    if (fd < 0) throw std::runtime_error(std::string("memfd_create: ") + std::strerror(errno));
    return fd;
}

char* map_shared(int fd, uint64_t size) {
    void* p = ::mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) throw std::runtime_error(std::string("mmap: ") + std::strerror(errno));
    return static_cast<char*>(p);
}
}  // namespace

Daemon::Daemon(const DaemonConfig& cfg) : cfg_(cfg) {
    validate(cfg_);
    Metrics::get().reset();  // counters describe this daemon instance
    daemon_epoch_ = real_ns();
    stripes_ = cfg_.nvme_stripe ? std::max<uint32_t>(1, cfg_.nvme_stripe_count) : 1;
    stripe_cursor_ = std::vector<std::atomic<uint64_t>>(stripes_);
    for (auto& c : stripe_cursor_) c.store(0);
    try {
        build_arenas();
        build_control();
        build_windows();
        if (!cfg_.v2_persist_dir.empty()) recover_persisted();
    } catch (...) {
        teardown();
        throw;
    }
}

Daemon::~Daemon() {
    stop();
    teardown();
}

void Daemon::build_arenas() {
    // Arenas are shared memory faulted in here: more than the host has would
    // get the daemon killed in the middle of the first touch. Refuse instead,
    // with the numbers (skipped when /proc/meminfo is unreadable).
    if (cfg_.numa_first_touch) {
        uint64_t want = 0;
        for (const NumaArena& ac : cfg_.per_numa) want += round_up(ac.size_bytes, cfg_.allocation_granularity_bytes);
        const uint64_t avail = host_memory_available();
        if (avail && want > avail)
            throw std::runtime_error("arenas need " + std::to_string(want >> 20) + " MiB but the host has " +
                                     std::to_string(avail >> 20) + " MiB available");
    }
    for (size_t i = 0; i < cfg_.per_numa.size(); ++i) {
        const NumaArena& ac = cfg_.per_numa[i];
        Arena a;
        a.numa_node = ac.numa_node;
        a.size = round_up(ac.size_bytes, cfg_.allocation_granularity_bytes);
        a.reg_gran = uint32_t(std::min<uint64_t>(cfg_.registration_chunk_bytes, 0xFFFFFFFFull));
        a.alloc_gran = uint32_t(std::min<uint64_t>(cfg_.allocation_granularity_bytes, 0xFFFFFFFFull));
        std::string name = "ofld_arena_" + std::to_string(i);
        a.fd = make_memfd(name.c_str());
        arenas_.push_back(a);  // registered before any throw so teardown closes it
        Arena& A = arenas_.back();
        if (::ftruncate(A.fd, off_t(A.size)) != 0)
            throw std::runtime_error(std::string("ftruncate(arena): ") + std::strerror(errno));
        A.base = map_shared(A.fd, A.size);
        // Bind the pages to the arena's node and fault them in from a thread
        // running on that node so placement holds even without mbind support.
        int node = int(ac.numa_node);
        char* base = A.base;
        uint64_t sz = A.size;
        bool touch = cfg_.numa_first_touch;
        bool huge = cfg_.arena_huge_pages;
        std::thread t([node, base, sz, touch, huge] {
            pin_thread_to_node(node);
            int rc = bind_range_to_node(base, sz, node, false);
            if (rc != 0) LOG_WARN(TAG, "mbind(node=%d) failed rc=%d (continuing)", node, rc);
            if (huge && ::madvise(base, sz, MADV_HUGEPAGE) != 0)
                LOG_WARN(TAG, "madvise(MADV_HUGEPAGE) failed: %s (continuing with base pages)", std::strerror(errno));
            if (touch) {
                // fault the pages in from several threads on the node (a
                // 100 GB arena is millions of page faults)
                const uint64_t n = std::max<uint64_t>(1, std::min<uint64_t>(8, sz >> 30));
                const uint64_t step = (sz / n + (2u << 20) - 1) & ~uint64_t((2u << 20) - 1);
                std::vector<std::thread> ts;
                for (uint64_t k = 0; k < n; ++k) {
                    const uint64_t off = k * step;
                    if (off >= sz) break;
                    const uint64_t len = std::min(step, sz - off);
                    ts.emplace_back([node, base, off, len] {
                        pin_thread_to_node(node);
                        first_touch(base + off, len);
                    });
                }
                for (auto& th : ts) th.join();
            }
        });
        t.join();
        LOG_INFO(TAG, "arena %zu: node=%u size=%llu MiB", i, A.numa_node,
                 (unsigned long long)(A.size >> 20));
    }
}

void Daemon::build_control() {
    uint64_t total_slots = 0;
    for (const Arena& a : arenas_) total_slots += a.size / cfg_.allocation_granularity_bytes;
    if (total_slots > 0xFFFFFFF0ull) throw std::runtime_error("too many slots");
    uint32_t cap = std::max<uint32_t>(2, cfg_.completion_ring_capacity);
    uint32_t p2 = 1;
    while (p2 < cap) p2 <<= 1;
    ring_cap_ = p2;
    ring_max_ = cfg_.completion_ring_max_ranks;
    ring_stride_ = uint32_t(ring_stride_bytes(ring_cap_));
    uint64_t ring_area = uint64_t(ring_max_) * ring_stride_;
    layout_ = control_layout(uint32_t(arenas_.size()), uint32_t(total_slots), ring_area);

    control_fd_ = make_memfd("ofld_control");
    if (::ftruncate(control_fd_, off_t(layout_.total_bytes)) != 0)
        throw std::runtime_error(std::string("ftruncate(control): ") + std::strerror(errno));
    control_ = map_shared(control_fd_, layout_.total_bytes);
    std::memset(control_, 0, layout_.total_bytes);

    header_ = header_of(control_);
    header_->magic = OFLD_MAGIC;
    header_->abi_version = OFLD_ABI_VERSION;
    header_->num_slots = layout_.num_slots;
    header_->num_arenas = layout_.num_arenas;
    header_->generation = 1;
    header_->daemon_pid = uint64_t(::getpid());
    header_->daemon_epoch = daemon_epoch_;
    header_->heartbeat_ns.store(real_ns(), std::memory_order_release);
    header_->arena_desc_offset = layout_.arena_desc_offset;
    header_->slot_entries_offset = layout_.slot_entries_offset;
    header_->control_ring_offset = layout_.ring_offset;

    ofld_arena_desc_t* d = arena_descs_of(control_);
    for (size_t i = 0; i < arenas_.size(); ++i) {
        d[i].arena_id = i;
        d[i].base_offset = 0;
        d[i].size = arenas_[i].size;
        d[i].numa_node = arenas_[i].numa_node;
        d[i].kind = OFLD_ARENA_DATA_PINNED;
        d[i].registration_granularity = arenas_[i].reg_gran;
        d[i].allocation_granularity = arenas_[i].alloc_gran;
    }
    pub_slots_ = slots_of(control_);
    slot_store_.reset(new ofld_slot_entry_t[std::max<uint32_t>(layout_.num_slots, 1)]());
    slots_ = slot_store_.get();

    RingGeometry* g = ring_geometry(header_);
    g->max_ranks = ring_max_;
    g->stride = ring_stride_;
    g->capacity = ring_cap_;
    for (uint32_t i = 0; i < ring_max_; ++i) {
        RingHeader* r = ring(i);
        if (!r) break;
        r->capacity = ring_cap_;
        r->owner_rank = 0xFFFFFFFFu;
        r->rank_epoch = 0;
        r->head.store(0);
        r->tail.store(0);
    }
    ring_owner_.assign(ring_max_, 0xFFFFFFFFu);
    LOG_INFO(TAG, "control: %u slots, %u arenas, %u rings x %u, %llu bytes", layout_.num_slots,
             layout_.num_arenas, ring_max_, ring_cap_, (unsigned long long)layout_.total_bytes);
}

void Daemon::build_windows() {
    const uint64_t gran = cfg_.allocation_granularity_bytes;
    uint32_t next = 0;
    slot_window_.assign(layout_.num_slots, 0xFFFFFFFFu);
    for (size_t ai = 0; ai < arenas_.size(); ++ai) {
        const NumaArena& ac = cfg_.per_numa[ai];
        uint64_t cursor = 0;
        uint64_t arena_slots = arenas_[ai].size / gran;
        auto carve = [&](uint32_t gpu, bool overflow, uint64_t nslots) {
            nslots = std::min<uint64_t>(nslots, arena_slots - cursor / gran);
            if (nslots == 0) return;
            Window w;
            w.numa_node = ac.numa_node;
            w.gpu = overflow ? kOverflowGpu : gpu;
            w.overflow = overflow;
            w.first_slot = next;
            w.nslots = uint32_t(nslots);
            w.free_bits.assign((nslots + 63) / 64, 0);
            for (uint64_t s = 0; s < nslots; ++s) {
                w.free_bits[s / 64] |= 1ull << (s % 64);
                uint32_t id = next + uint32_t(s);
                ofld_slot_entry_t& e = slots_[id];
                e.slot_id = id;
                e.numa_node = ac.numa_node;
                e.gpu_preferred = w.gpu;
                e.arena_id = ai;
                e.arena_offset = cursor + s * gran;
                e.capacity = gran;
                e.flags = overflow ? 0 : OFLD_FLAG_BORROWABLE;
                e.state.store(OFLD_SLOT_FREE, std::memory_order_release);
                slot_window_[id] = uint32_t(windows_.size());
            }
            next += uint32_t(nslots);
            cursor += nslots * gran;
            windows_.push_back(std::move(w));
        };
        for (const GpuWindow& gw : ac.gpu_windows) carve(gw.gpu, false, gw.size_bytes / gran);
        carve(kOverflowGpu, true, ac.overflow_bytes / gran);
        // Slots not claimed by any window join the overflow pool of this arena.
        uint64_t rest = arena_slots - cursor / gran;
        if (rest) carve(kOverflowGpu, true, rest);
    }
    for (uint32_t i = 0; i < layout_.num_slots; ++i) publish_slot(i);
    LOG_INFO(TAG, "slot plan: %zu windows, %u slots", windows_.size(), next);
}

void Daemon::teardown() {
    if (control_) {
        ::munmap(control_, layout_.total_bytes);
        control_ = nullptr;
    }
    close_fd(control_fd_);
    control_fd_ = -1;
    for (Arena& a : arenas_) {
        if (a.base) ::munmap(a.base, a.size);
        close_fd(a.fd);
        a.base = nullptr;
        a.fd = -1;
    }
    for (auto& kv : cold_)
        if (kv.second.pageable) pageable_pool_.put(kv.second.pageable, kv.second.pageable_size, 0);
    cold_.clear();
    for (auto& kv : peer_buffers_) close_fd(kv.second.fd);
    peer_buffers_.clear();
}

// ============================================================================
// Serving
// ============================================================================
void Daemon::run() {
    if (::pipe2(stop_pipe_, O_CLOEXEC) != 0) throw std::runtime_error("pipe2 failed");
    listen_fd_ = uds_listen(cfg_.socket_path);
    if (cfg_.v2_control_tcp_port) tcp_fd_ = tcp_listen(uint16_t(cfg_.v2_control_tcp_port));
    running_.store(true);
    workers_on_.store(true);
    copy_pool_.start(cfg_.copy_threads);
    for (uint32_t i = 0; i < std::max<uint32_t>(1, cfg_.drain_workers); ++i)
        workers_.emplace_back([this] { drain_loop(); });
    for (uint32_t i = 0; i < std::max<uint32_t>(1, cfg_.readback_workers); ++i)
        workers_.emplace_back([this] { readback_loop(); });
    workers_.emplace_back([this] { heartbeat_loop(); });
    if (ring_max_) workers_.emplace_back([this] { ring_loop(); });
    if (!cfg_.v2_persist_dir.empty()) workers_.emplace_back([this] { persist_loop(); });
    LOG_INFO(TAG, "serving on %s (pid %d, tcp port %u)", cfg_.socket_path.c_str(), int(::getpid()),
             cfg_.v2_control_tcp_port);
    ready_.store(true);

    accept_loop();

    ready_.store(false);
    workers_on_.store(false);
    drain_cv_.notify_all();
    readback_cv_.notify_all();
    peer_cv_.notify_all();
    persist_cv_.notify_all();
    reap_connections(true);
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
    copy_pool_.stop();
    close_fd(listen_fd_);
    close_fd(tcp_fd_);
    listen_fd_ = tcp_fd_ = -1;
    ::unlink(cfg_.socket_path.c_str());
    close_fd(stop_pipe_[0]);
    close_fd(stop_pipe_[1]);
    stop_pipe_[0] = stop_pipe_[1] = -1;
    LOG_INFO(TAG, "stopped");
}

void Daemon::stop() {
    running_.store(false);
    if (stop_pipe_[1] >= 0) {
        char b = 1;
        ssize_t r = ::write(stop_pipe_[1], &b, 1);
        (void)r;
    }
}

bool Daemon::wait_ready(int timeout_ms) const {
    uint64_t end = mono_ns() + uint64_t(timeout_ms) * 1000000ull;
    while (!ready_.load()) {
        if (mono_ns() > end) return false;
        sleep_us(1000);
    }
    return true;
}

void Daemon::accept_loop() {
    while (running_.load()) {
        pollfd p[3] = {{listen_fd_, POLLIN, 0}, {stop_pipe_[0], POLLIN, 0}, {tcp_fd_, POLLIN, 0}};
        int rc = ::poll(p, 3, 1000);
        if (rc < 0) {
            if (errno == EINTR) continue;
            LOG_ERR(TAG, "poll: %s", std::strerror(errno));
            break;
        }
        reap_connections(false);
        if (p[1].revents & POLLIN) break;
        for (int k : {0, 2}) {
            if (!(p[k].revents & POLLIN) || p[k].fd < 0) continue;
            int fd = accept_conn(p[k].fd);
            if (fd < 0) continue;
            auto done = std::make_shared<std::atomic<bool>>(false);
            std::lock_guard<std::mutex> g(conn_mu_);
            conns_.push_back(Conn{fd, std::thread([this, fd, done] {
                                      serve(fd);
                                      done->store(true);
                                  }),
                                  done});
        }
    }
}

void Daemon::reap_connections(bool all) {
    std::list<Conn> finished;
    {
        std::lock_guard<std::mutex> g(conn_mu_);
        for (auto it = conns_.begin(); it != conns_.end();) {
            if (all && !it->done->load()) ::shutdown(it->fd, SHUT_RDWR);
            if (all || it->done->load()) {
                finished.splice(finished.end(), conns_, it++);
            } else {
                ++it;
            }
        }
    }
    for (Conn& c : finished)
        if (c.th.joinable()) c.th.join();
}

void Daemon::serve(int fd) {
    for (;;) {
        Op op = Op::kInvalid;
        std::vector<uint8_t> body;
        std::vector<int> fds;
        bool got = false;
        try {
            got = recv_frame(fd, &op, &body, &fds);
        } catch (const std::exception& e) {
            LOG_DEBUG(TAG, "connection closed: %s", e.what());
            break;
        }
        if (!got) break;
        try {
            dispatch(fd, op, body, fds);
        } catch (const std::exception& e) {
            LOG_WARN(TAG, "dispatch %s failed: %s", op_name(op), e.what());
            for (int f : fds) close_fd(f);
            break;
        }
        for (int f : fds) close_fd(f);  // handlers take ownership by clearing
        if (!running_.load()) break;
    }
    ::close(fd);
}

void Daemon::dispatch(int fd, Op op, const std::vector<uint8_t>& b, std::vector<int>& fds_in) {
    std::vector<uint8_t> out;
    std::vector<int> fds_out;
    const uint8_t* p = b.data();
    size_t n = b.size();
#define ROUTE(OPC, CALL)                                                   \
    case Op::OPC: {                                                        \
        auto req = decode<OpTypes<Op::OPC>::Request>(p, n);                \
        out = encode(CALL);                                                \
        break;                                                             \
    }
    switch (op) {
        ROUTE(kRegisterRank, on_register(req, &fds_out))
        ROUTE(kHeartbeat, on_heartbeat(req))
        ROUTE(kRequestOffload, on_request_offload(req))
        ROUTE(kMarkD2HSubmitted, on_d2h_submitted(req))
        ROUTE(kMarkD2HComplete, on_d2h_complete(req))
        ROUTE(kRequestPrefetch, on_request_prefetch(req))
        ROUTE(kMarkH2DSubmitted, on_h2d_submitted(req))
        ROUTE(kMarkH2DComplete, on_h2d_complete(req))
        ROUTE(kReleaseLease, on_release_lease(req))
        ROUTE(kQueryLocation, on_query_location(req))
        ROUTE(kBatchComplete, on_batch_complete(req))
        ROUTE(kGetStats, on_get_stats(req))
        ROUTE(kShutdown, on_shutdown(req))
        ROUTE(kRegisterJob, on_register_job(req))
        ROUTE(kRequestCanonicalEvict, on_canonical_evict(req))
        ROUTE(kCommitCanonicalObject, on_commit_canonical(req))
        ROUTE(kSealModelVersion, on_seal(req))
        ROUTE(kGetLatestSealedVersion, on_get_latest(req))
        ROUTE(kGetManifest, on_get_manifest(req))
        ROUTE(kPullTensor, on_pull_tensor(req))
        ROUTE(kRequestCanonicalRestore, on_canonical_restore(req))
        ROUTE(kReleaseCanonicalRestore, on_release_canonical_restore(req))
        ROUTE(kDropCanonicalVersion, on_drop_version(req))
        ROUTE(kReleaseCanonical, on_release_canonical(req))
        ROUTE(kBatchRequestOffload, on_batch_request_offload(req))
        ROUTE(kBatchRequestPrefetch, on_batch_request_prefetch(req))
        ROUTE(kPublishPeerBuffer, on_publish_peer_buffer(req, &fds_in))
        ROUTE(kLookupPeerBuffer, on_lookup_peer_buffer(req, &fds_out))
        ROUTE(kGetJobStats, on_get_job_stats(req))
        ROUTE(kExportManifest, on_export_manifest(req))
        ROUTE(kDiscardTensor, on_discard_tensor(req))
        ROUTE(kCarryForward, on_carry_forward(req))
        ROUTE(kGetAgentOptions, on_get_agent_options(req))
        ROUTE(kBatchDiscardTensor, on_batch_discard(req))
        ROUTE(kSetRunFormat, on_set_run_format(req))
        default:
            LOG_WARN(TAG, "unknown opcode %u", unsigned(op));
            throw std::runtime_error("unknown opcode");
    }
#undef ROUTE
    send_frame(fd, make_frame(op, out), fds_out);
    // fds_out of RegisterRank are the daemon's own arena fds (kept); lookup
    // replies carry dup()ed fds that the daemon must close after sending.
    if (op == Op::kLookupPeerBuffer)
        for (int f : fds_out) close_fd(f);
}

// ============================================================================
// Sessions
// ============================================================================
bool Daemon::epoch_ok(uint32_t rank, uint64_t epoch) {
    auto it = sessions_.find(rank);
    return it != sessions_.end() && it->second.alive && it->second.epoch == epoch;
}

// A session ended (re-register, pid reuse, or heartbeat timeout). Completed
// data stays readable; reservations that never completed are reclaimed; the
// rank's ring is drained and released; its canonical holds and published peer
// buffers are dropped. mu_ held.
void Daemon::recover_session(Session& s, const char* why) {
    if (!s.alive) return;
    s.alive = false;
    Metrics::get().inc(M::kRankSessionsInvalidated);
    LOG_WARN(TAG, "rank %u epoch %llu ended (%s)", s.rank_id, (unsigned long long)s.epoch, why);
    if (s.ring < ring_max_) {
        RingHeader* r = ring(s.ring);
        ofld_completion_entry_t e;
        // Completions the rank published before dying are still valid.
        s.alive = true;
        while (ring_pop(r, ring_cap_, &e)) apply_ring_entry(s.rank_id, s.epoch, e);
        s.alive = false;
        r->owner_rank = 0xFFFFFFFFu;
        r->rank_epoch = 0;
        ring_owner_[s.ring] = 0xFFFFFFFFu;
        s.ring = 0xFFFFFFFFu;
    }
    std::vector<uint64_t> gone;
    for (auto& kv : leases_) {
        Lease& L = kv.second;
        if (L.owner_rank != s.rank_id || L.epoch != s.epoch) continue;
        uint32_t st = state_of(L.base);
        bool safe = st == OFLD_SLOT_PINNED_VALID || st == OFLD_SLOT_COLD_VALID ||
                    st == OFLD_SLOT_DRAIN_IN_FLIGHT;
        if (!safe) {
            // A canonical object being created by this rank is abandoned.
            if (is_canonical_tid(L.tensor_id) && !is_candidate_tid(L.tensor_id)) {
                CanonicalObject* o = find_object(L.tensor_id & ~kCanonicalTidBit);
                if (o && o->state == OBJ_CREATING) {
                    settle_d2h(*o);
                    object_by_key_.erase(o->key_str);
                    o->state = OBJ_ERROR;
                }
            }
            set_run_state(L.base, L.count, OFLD_SLOT_ERROR);
            free_run(L.base, L.count);
            Trace::get().event("ERROR", s.rank_id, s.gpu, L.tensor_id, L.version, L.id, L.base, L.nbytes);
            auto lit = locations_.find(L.tensor_id);
            if (lit != locations_.end() && lit->second.kind == OFLD_LOC_PINNED &&
                lit->second.slot == L.base && lit->second.version == L.version)
                lit->second.kind = OFLD_LOC_NONE;
        }
        gone.push_back(L.id);
    }
    for (uint64_t id : gone) erase_lease(id);
    // Objects whose creator died before committing are unreferenced garbage.
    std::vector<uint64_t> dead;
    for (auto& kv : objects_)
        if (kv.second.state == OBJ_ERROR) dead.push_back(kv.first);
    for (uint64_t oid : dead) {
        CanonicalObject& o = objects_[oid];
        o.holders.clear();
        release_object(o);
    }
    purge_rank_holds(s.rank_id);
    for (auto it = peer_buffers_.begin(); it != peer_buffers_.end();) {
        if (it->second.desc.owner_rank == s.rank_id) {
            close_fd(it->second.fd);
            it = peer_buffers_.erase(it);
        } else {
            ++it;
        }
    }
}

RegisterRankResponse Daemon::on_register(const RegisterRankRequest& r, std::vector<int>* fds) {
    std::lock_guard<std::mutex> g(mu_);
    RegisterRankResponse resp;
    auto it = sessions_.find(r.rank_id);
    if (it != sessions_.end()) recover_session(it->second, "re-registered");
    // A process re-registering under a new rank id replaces its old session,
    // unless it declares that it holds several sessions at once.
    if (!(r.capabilities & kCapMultiSession))
        for (auto& kv : sessions_)
            if (kv.first != r.rank_id && kv.second.alive && kv.second.pid == r.pid)
                recover_session(kv.second, "pid re-registered under a new rank id");

    Session s;
    s.rank_id = r.rank_id;
    s.epoch = next_epoch_++;
    s.pid = r.pid;
    s.gpu = r.gpu_id;
    s.numa = r.numa_node;
    s.last_hb_ns = real_ns();
    for (uint32_t i = 0; i < ring_max_; ++i) {
        if (ring_owner_[i] != 0xFFFFFFFFu) continue;
        RingHeader* rh = ring(i);
        if (!rh) break;
        rh->head.store(0, std::memory_order_relaxed);
        rh->tail.store(0, std::memory_order_relaxed);
        rh->owner_rank = r.rank_id;
        std::atomic_thread_fence(std::memory_order_release);
        rh->rank_epoch = s.epoch;
        ring_owner_[i] = r.rank_id;
        s.ring = i;
        break;
    }
    sessions_[r.rank_id] = s;

    resp.ok = true;
    resp.message = "ok";
    resp.rank_epoch = s.epoch;
    resp.control_generation = header_->generation;
    for (size_t i = 0; i < arenas_.size(); ++i) {
        ArenaFd a;
        a.arena_id = i;
        a.numa_node = arenas_[i].numa_node;
        a.kind = OFLD_ARENA_DATA_PINNED;
        a.size = arenas_[i].size;
        a.fd_index = uint32_t(i);
        a.registration_granularity = arenas_[i].reg_gran;
        a.allocation_granularity = arenas_[i].alloc_gran;
        resp.arenas.push_back(a);
        fds->push_back(arenas_[i].fd);
    }
    resp.control_fd_index = uint32_t(arenas_.size());
    fds->push_back(control_fd_);
    resp.control_size = layout_.total_bytes;
    resp.num_slots = layout_.num_slots;
    resp.ring_index = s.ring;
    LOG_INFO(TAG, "rank %u registered (pid %llu gpu %u numa %u) epoch %llu ring %d", r.rank_id,
             (unsigned long long)r.pid, r.gpu_id, r.numa_node, (unsigned long long)s.epoch,
             s.ring == 0xFFFFFFFFu ? -1 : int(s.ring));
    return resp;
}

StatusResponse Daemon::on_heartbeat(const HeartbeatRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    uint64_t now = real_ns();
    sessions_[r.rank_id].last_hb_ns = now;
    header_->heartbeat_ns.store(now, std::memory_order_release);
    return {true, "ok"};
}

void Daemon::heartbeat_loop() {
    const uint64_t timeout_ns = cfg_.heartbeat_timeout_ms * 1000000ull;
    const uint64_t period_ms = std::max<uint64_t>(cfg_.heartbeat_timeout_ms / 4, 20);
    while (workers_on_.load()) {
        for (uint64_t t = 0; t < period_ms && workers_on_.load(); t += 10) sleep_us(10000);
        if (!workers_on_.load()) break;
        uint64_t now = real_ns();
        std::lock_guard<std::mutex> g(mu_);
        header_->heartbeat_ns.store(now, std::memory_order_release);
        for (auto& kv : sessions_) {
            Session& s = kv.second;
            if (s.alive && now > s.last_hb_ns && now - s.last_hb_ns > timeout_ns)
                recover_session(s, "heartbeat timeout");
        }
    }
}

void Daemon::apply_ring_entry(uint32_t rank, uint64_t epoch, const ofld_completion_entry_t& e) {
    Metrics::get().inc(M::kRingCompletionsApplied);
    if (e.event_type == uint32_t(EventType::kD2HComplete)) {
        bool latest = false, drained = false;
        apply_d2h_complete(rank, epoch, e.lease_id, e.tensor_id, e.version, e.slot_id, 0, &latest, &drained);
    } else if (e.event_type == uint32_t(EventType::kH2DComplete)) {
        apply_h2d_complete(rank, epoch, e.lease_id, e.tensor_id, e.version, e.slot_id, false, 0);
    } else {
        Metrics::get().inc(M::kInvalidTransitionRejected);
    }
}

// Handlers whose answer depends on completions (prefetch, location, discard)
// call this first: an agent publishes a completion before it sends the next
// request, so the request sees its own earlier transfers without waiting for
// the poller.
void Daemon::drain_rings() {
    if (rings_paused_.load()) return;
    for (uint32_t i = 0; i < ring_max_; ++i) {
        const Session* s = ring_session(i);
        if (!s) continue;
        const uint32_t rank = s->rank_id;
        const uint64_t epoch = s->epoch;
        RingHeader* r = ring(i);
        ofld_completion_entry_t e;
        while (ring_pop(r, ring_cap_, &e)) apply_ring_entry(rank, epoch, e);
    }
}

const Daemon::Session* Daemon::ring_session(uint32_t i) const {
    if (i >= ring_max_ || ring_owner_[i] == 0xFFFFFFFFu) return nullptr;
    auto it = sessions_.find(ring_owner_[i]);
    if (it == sessions_.end() || !it->second.alive || it->second.ring != i) return nullptr;
    return &it->second;
}

void Daemon::ring_loop() {
    const uint64_t idle_us = cfg_.ring_poll_us ? cfg_.ring_poll_us : 50;
    while (workers_on_.load()) {
        bool any = false;
        if (rings_paused_.load()) {
            sleep_us(idle_us);
            continue;
        }
        {
            std::lock_guard<std::mutex> g(mu_);
            for (uint32_t i = 0; i < ring_max_; ++i) {
                const Session* s = ring_session(i);
                if (!s) continue;
                const uint32_t rank = s->rank_id;
                const uint64_t epoch = s->epoch;
                RingHeader* r = ring(i);
                ofld_completion_entry_t e;
                for (int budget = 256; budget > 0 && ring_pop(r, ring_cap_, &e); --budget) {
                    apply_ring_entry(rank, epoch, e);
                    any = true;
                }
            }
        }
        if (!any) sleep_us(idle_us);
    }
    std::lock_guard<std::mutex> g(mu_);
    for (uint32_t i = 0; i < ring_max_; ++i) {
        const Session* s = ring_session(i);
        if (!s) continue;
        const uint32_t rank = s->rank_id;
        const uint64_t epoch = s->epoch;
        RingHeader* r = ring(i);
        ofld_completion_entry_t e;
        while (ring_pop(r, ring_cap_, &e)) apply_ring_entry(rank, epoch, e);
    }
}

GetStatsResponse Daemon::on_get_stats(const GetStatsRequest&) {
    GetStatsResponse resp;
    resp.ok = true;
    resp.message = "ok";
    std::unique_lock<std::mutex> g(mu_);
    drain_rings();
    g.unlock();
    for (auto& kv : Metrics::get().snapshot()) resp.stats.push_back(StatEntry{kv.first, kv.second});
    g.lock();
    uint64_t live = 0;
    for (auto& kv : sessions_) live += kv.second.alive ? 1 : 0;
    resp.stats.push_back({"live_rank_sessions", live});
    resp.stats.push_back({"total_slots", layout_.num_slots});
    resp.stats.push_back({"used_slots", used_slots_});
    resp.stats.push_back({"slot_bytes", cfg_.allocation_granularity_bytes});
    resp.stats.push_back({"pinned_pressure_ppm", uint64_t(pinned_pressure() * 1e6)});
    resp.stats.push_back({"canonical_objects", objects_.size()});
    resp.stats.push_back({"sealed_manifests", manifests_.size()});
    resp.stats.push_back({"jobs", jobs_.size()});
    resp.stats.push_back({"pageable_pool_bytes", pageable_pool_.pooled()});
    // Per-GPU window (and per-NUMA overflow pool) occupancy: "<scope>.<name>",
    // rendered as labelled series by offload-stat --prometheus.
    const uint64_t gran = cfg_.allocation_granularity_bytes;
    for (const Window& w : windows_) {
        uint64_t free_slots = 0;
        for (uint64_t word : w.free_bits) free_slots += uint64_t(__builtin_popcountll(word));
        const std::string scope =
            w.overflow ? "numa" + std::to_string(w.numa_node) + "_overflow" : "gpu" + std::to_string(w.gpu);
        resp.stats.push_back({scope + ".window_bytes", uint64_t(w.nslots) * gran});
        resp.stats.push_back({scope + ".window_used_bytes", (uint64_t(w.nslots) - free_slots) * gran});
    }
    std::map<uint32_t, uint64_t> per_gpu;
    for (auto& kv : sessions_)
        if (kv.second.alive) per_gpu[kv.second.gpu]++;
    for (auto& kv : per_gpu) resp.stats.push_back({"gpu" + std::to_string(kv.first) + ".live_sessions", kv.second});
    resp.stats.push_back({"daemon_epoch", daemon_epoch_});
    return resp;
}

StatusResponse Daemon::on_shutdown(const ShutdownRequest&) {
    LOG_INFO(TAG, "shutdown requested");
    stop();
    return {true, "shutting down"};
}

StatusResponse Daemon::on_publish_peer_buffer(const PublishPeerBufferRequest& r, std::vector<int>* fds_in) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    if (r.desc.key.empty()) return {false, "empty key"};
    PeerBuffer pb;
    pb.desc = r.desc;
    pb.desc.owner_rank = r.rank_id;
    if (!fds_in->empty()) {
        pb.fd = (*fds_in)[0];
        fds_in->erase(fds_in->begin());  // keep ownership of the first fd
    }
    auto it = peer_buffers_.find(r.desc.key);
    if (it != peer_buffers_.end()) close_fd(it->second.fd);
    peer_buffers_[r.desc.key] = pb;
    Metrics::get().inc(M::kPeerBuffersPublished);
    peer_cv_.notify_all();
    return {true, "ok"};
}

LookupPeerBufferResponse Daemon::on_lookup_peer_buffer(const LookupPeerBufferRequest& r, std::vector<int>* fds_out) {
    std::unique_lock<std::mutex> lk(mu_);
    LookupPeerBufferResponse resp;
    resp.ok = true;
    auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(r.wait_ms);
    for (;;) {
        auto it = peer_buffers_.find(r.key);
        if (it != peer_buffers_.end()) {
            resp.found = true;
            resp.desc = it->second.desc;
            if (it->second.fd >= 0) {
                int d = ::fcntl(it->second.fd, F_DUPFD_CLOEXEC, 0);
                if (d >= 0) fds_out->push_back(d);
            }
            resp.message = "ok";
            return resp;
        }
        if (r.wait_ms == 0 || !workers_on_.load() ||
            peer_cv_.wait_until(lk, deadline) == std::cv_status::timeout) {
            auto again = peer_buffers_.find(r.key);
            if (again == peer_buffers_.end()) {
                resp.found = false;
                resp.message = "not published";
                return resp;
            }
        }
    }
}

// The `kernels:` and `nvlink:` sections of the config, flattened to dotted
// keys; sessions apply them before they start (explicit options win).
GetAgentOptionsResponse Daemon::on_get_agent_options(const GetAgentOptionsRequest&) {
    GetAgentOptionsResponse resp;
    resp.ok = true;
    resp.message = "ok";
    for (const auto& kv : cfg_.agent_options) resp.options.push_back(OptionEntry{kv.first, kv.second});
    return resp;
}

GetJobStatsResponse Daemon::on_get_job_stats(const GetJobStatsRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    drain_rings();
    GetJobStatsResponse resp;
    resp.ok = true;
    resp.message = "ok";
    for (auto& kv : jobs_) {
        const Job& j = kv.second;
        if (!r.all_tenants && j.uid.tenant_id != r.tenant_id) continue;
        JobStatsEntry e;
        e.job = JobKeyWire{j.uid.tenant_id, j.uid.job_id, j.uid.launch_epoch, j.name};
        e.pinned_bytes = j.pinned_bytes;
        e.pageable_bytes = j.pageable_bytes;
        e.nvme_bytes = j.nvme_bytes;
        e.inflight_d2h_bytes = j.inflight_d2h_bytes;
        e.inflight_export_bytes = j.inflight_export_bytes;
        e.canonical_object_count = j.object_count;
        e.dedup_bytes_saved = j.dedup_bytes_saved;
        resp.jobs.push_back(e);
    }
    return resp;
}

}  // namespace ofld
