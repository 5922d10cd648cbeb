// Cold tiers: background drain (pinned -> pageable/NVMe), readback
// (cold -> pinned), forced drains under pinned pressure, and the pressure
// thresholds of drain_policy.
//
// Tier choice for a drain:
//   pageable            -> malloc'd pageable buffer
//   nvme                -> striped NVMe extents (pageable when NVMe is off)
//   pageable_then_nvme  -> pageable while the pageable tier is under
//                          drain_policy.pageable_limit_gb, NVMe beyond it
// (StateSpectre's pageable_then_nvme never reaches NVMe, reference:
// src/daemon/daemon.cpp:1772; this runtime spills once the budget is hit.)
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <thread>
#include <vector>

#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"

namespace ofld {

namespace {
constexpr const char* TAG = "tiers";

void record_bw(uint64_t nbytes, uint64_t t0) {
    uint64_t dt = mono_ns() - t0;
    if (dt) Metrics::get().record_mbps(double(nbytes) / 1048576.0 / (double(dt) / 1e9));
}
}  // namespace

// ---------------------------------------------------------------------------
// Pageable memory
// ---------------------------------------------------------------------------
char* Daemon::PageablePool::get(uint64_t nbytes, uint64_t* size_out) {
    const uint64_t cls = 2ull << 20;
    const uint64_t need = (std::max<uint64_t>(nbytes, 1) + cls - 1) / cls * cls;
    {
        std::lock_guard<std::mutex> g(mu_);
        auto it = free_.lower_bound(need);
        if (it != free_.end() && it->first <= need + need / 8) {  // reuse up to 12.5 % slack
            char* p = it->second;
            *size_out = it->first;
            pooled_ -= it->first;
            free_.erase(it);
            return p;
        }
    }
    void* p = ::mmap(nullptr, need, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p == MAP_FAILED) return nullptr;
    *size_out = need;
    return static_cast<char*>(p);
}

void Daemon::PageablePool::put(char* p, uint64_t size, uint64_t cap) {
    if (!p) return;
    {
        std::lock_guard<std::mutex> g(mu_);
        if (pooled_.load() + size <= cap) {
            free_.emplace(size, p);
            pooled_ += size;
            return;
        }
    }
    ::munmap(p, size);
}

Daemon::PageablePool::~PageablePool() {
    for (auto& kv : free_) ::munmap(kv.second, kv.first);
}

void Daemon::CopyPool::start(uint32_t threads) {
    std::lock_guard<std::mutex> g(mu_);
    if (on_) return;
    on_ = true;
    for (uint32_t i = 0; i < threads; ++i)
        ts_.emplace_back([this] {
            for (;;) {
                Piece p;
                {
                    std::unique_lock<std::mutex> l(mu_);
                    cv_.wait(l, [&] { return !q_.empty() || !on_; });
                    if (q_.empty()) return;
                    p = q_.front();
                    q_.pop_front();
                }
                run_piece(p);
            }
        });
}

void Daemon::CopyPool::stop() {
    {
        std::lock_guard<std::mutex> g(mu_);
        on_ = false;
    }
    cv_.notify_all();
    for (auto& t : ts_) t.join();
    ts_.clear();
}

void Daemon::CopyPool::run_piece(const Piece& p) {
    (*p.fn)(p.index);
    if (p.left->fetch_sub(1, std::memory_order_acq_rel) == 1) {
        std::lock_guard<std::mutex> g(mu_);  // the waiter checks `left` under mu_
        done_cv_.notify_all();
    }
}

void Daemon::CopyPool::run(uint32_t tasks, const std::function<void(uint32_t)>& fn) {
    if (tasks == 0) return;
    if (tasks == 1 || threads() == 0) {
        for (uint32_t i = 0; i < tasks; ++i) fn(i);
        return;
    }
    std::atomic<uint32_t> left{tasks};
    {
        std::lock_guard<std::mutex> g(mu_);
        for (uint32_t i = 1; i < tasks; ++i) q_.push_back(Piece{&fn, i, &left});
    }
    cv_.notify_all();
    run_piece(Piece{&fn, 0, &left});
    // Help with queued pieces (this call's or another's) until ours are done.
    for (;;) {
        Piece p;
        {
            std::unique_lock<std::mutex> l(mu_);
            if (left.load(std::memory_order_acquire) == 0) return;
            if (q_.empty()) {
                done_cv_.wait(l, [&] { return left.load(std::memory_order_acquire) == 0 || !q_.empty(); });
                continue;
            }
            p = q_.front();
            q_.pop_front();
        }
        run_piece(p);
    }
}

void Daemon::CopyPool::copy(char* dst, const char* src, uint64_t n) {
    constexpr uint64_t kPiece = 1ull << 20;
    const uint64_t parts = std::min<uint64_t>(threads() + 1, n / kPiece);
    if (parts <= 1) {
        std::memcpy(dst, src, n);
        return;
    }
    const uint64_t step = (n / parts + 4095) & ~uint64_t(4095);
    const uint32_t tasks = uint32_t((n + step - 1) / step);
    run(tasks, [&](uint32_t i) {
        const uint64_t off = uint64_t(i) * step;
        std::memcpy(dst + off, src + off, std::min(step, n - off));
    });
}

void Daemon::copy_bytes(char* dst, const char* src, uint64_t n) const { copy_pool_.copy(dst, src, n); }

void Daemon::cold_quota(uint64_t tid, uint64_t nbytes, bool* allow_pageable, bool* allow_nvme) {
    *allow_pageable = *allow_nvme = true;
    if (!is_canonical_tid(tid) || is_candidate_tid(tid)) return;
    CanonicalObject* o = find_object(tid & ~kCanonicalTidBit);
    Job* j = o ? find_job(o->key.job) : nullptr;
    if (!j) return;
    *allow_pageable = !j->max_pageable || j->pageable_bytes + nbytes <= j->max_pageable;
    *allow_nvme = !j->max_nvme || j->nvme_bytes + nbytes <= j->max_nvme;
}

namespace {
// A /proc/meminfo field in bytes (0 when unreadable).
uint64_t meminfo_bytes(const char* field) {
    FILE* f = std::fopen("/proc/meminfo", "r");
    if (!f) return 0;
    char line[256];
    uint64_t v = 0;
    const size_t n = std::strlen(field);
    while (std::fgets(line, sizeof(line), f)) {
        if (std::strncmp(line, field, n) == 0 && line[n] == ':') {
            v = std::strtoull(line + n + 1, nullptr, 10) * 1024;  // kB
            break;
        }
    }
    std::fclose(f);
    return v;
}
}  // namespace

uint64_t Daemon::host_memory_available() const {
    const uint64_t fake = fake_mem_available_.load();
    return fake ? fake : meminfo_bytes("MemAvailable");
}

bool Daemon::pageable_room(uint64_t nbytes) const {
    const uint64_t resident = Metrics::get().value(M::kPageableResidentBytes);
    if (cfg_.pageable_limit_bytes) return resident + nbytes <= cfg_.pageable_limit_bytes;
    const uint64_t avail = host_memory_available();
    if (!avail) return true;  // no /proc/meminfo: nothing to go by
    static const uint64_t total = meminfo_bytes("MemTotal");
    const uint64_t reserve = std::max<uint64_t>(4ull << 30, total / 20);
    return nbytes + reserve <= avail + pageable_pool_.pooled();
}

bool Daemon::write_cold(const char* src, uint64_t nbytes, ColdEntry* out, bool allow_pageable, bool allow_nvme) {
    out->nbytes = nbytes;
    if (fail_writes_.load() > 0 && fail_writes_.fetch_sub(1) > 0) {
        LOG_WARN(TAG, "injected cold write failure");
        return false;
    }
    bool pageable = false;
    switch (cfg_.drain_target) {
        case DrainTarget::kPageableOnly: pageable = true; break;
        case DrainTarget::kNvmeOnly: pageable = !cfg_.nvme_enabled; break;
        case DrainTarget::kPageableThenNvme: pageable = true; break;
    }
    if (pageable && allow_pageable && !pageable_room(nbytes)) {
        // over the pageable budget or out of host memory: NVMe when it may
        // take the bytes, else the drain fails and the run stays pinned
        pageable = false;
        Metrics::get().inc(M::kPageableRoomRejected);
    }
    pageable = pageable && allow_pageable;
    uint64_t t0 = mono_ns();
    if (pageable) {
        uint64_t size = 0;
        char* buf = pageable_pool_.get(nbytes, &size);
        if (buf) {
            copy_bytes(buf, src, nbytes);
            out->kind = OFLD_LOC_PAGEABLE;
            out->pageable = buf;
            out->pageable_size = size;
            Metrics::get().add(M::kPinnedToPageableBytes, nbytes);
            Metrics::get().add(M::kPageableResidentBytes, nbytes);
            record_bw(nbytes, t0);
            return true;
        }
        LOG_WARN(TAG, "pageable allocation of %llu bytes failed", (unsigned long long)nbytes);
        if (!cfg_.nvme_enabled) return false;
    }
    if (!cfg_.nvme_enabled || !allow_nvme) return false;
    if (!nvme_write(src, nbytes, &out->extents)) return false;
    out->kind = OFLD_LOC_NVME;
    Metrics::get().add(M::kNvmeWriteBytes, nbytes);
    Metrics::get().add(M::kNvmeResidentBytes, nbytes);
    record_bw(nbytes, t0);
    return true;
}

bool Daemon::read_cold(const ColdEntry& c, char* dst, uint64_t off, uint64_t nbytes) {
    if (fail_reads_.load() > 0 && fail_reads_.fetch_sub(1) > 0) {
        LOG_WARN(TAG, "injected cold read failure");
        return false;
    }
    if (off + nbytes > c.nbytes) return false;
    uint64_t t0 = mono_ns();
    if (c.kind == OFLD_LOC_PAGEABLE) {
        if (!c.pageable) return false;
        copy_bytes(dst, c.pageable + off, nbytes);
        Metrics::get().add(M::kPageableToPinnedBytes, nbytes);
    } else if (c.kind == OFLD_LOC_NVME) {
        if (!nvme_read(c.extents, dst, off, nbytes)) return false;
        Metrics::get().add(M::kNvmeReadBytes, nbytes);
    } else {
        return false;
    }
    record_bw(nbytes, t0);
    return true;
}

void Daemon::discard_storage(ColdEntry& c) {
    if (c.kind == OFLD_LOC_PAGEABLE && c.pageable) {
        pageable_pool_.put(c.pageable, c.pageable_size, cfg_.pageable_pool_bytes);
        c.pageable = nullptr;
        Metrics::get().sub(M::kPageableResidentBytes, c.nbytes);
    } else if (c.kind == OFLD_LOC_NVME && c.persisted) {
        for (const Extent& e : c.extents) ::unlink(e.path.c_str());  // a durable version file
        c.extents.clear();
    } else if (c.kind == OFLD_LOC_NVME) {
        nvme_release(c.extents);
        c.extents.clear();
        Metrics::get().sub(M::kNvmeResidentBytes, c.nbytes);
    }
    Metrics::get().add(M::kColdBytesReclaimed, c.nbytes);
}

// Free a cold entry's storage (pageable buffer or NVMe extents), or defer the
// free until in-flight unlocked readers finish. mu_ held.
void Daemon::free_cold(uint64_t cold_ref) {
    auto it = cold_.find(cold_ref);
    if (it == cold_.end()) return;
    if (it->second.readers > 0) {
        it->second.doomed = true;
        return;
    }
    discard_storage(it->second);
    cold_.erase(it);
}

bool Daemon::pin_cold(uint64_t cold_ref, ColdEntry* desc) {
    auto it = cold_.find(cold_ref);
    if (it == cold_.end() || it->second.doomed) return false;
    it->second.readers++;
    *desc = it->second;
    return true;
}

void Daemon::unpin_cold(uint64_t cold_ref) {
    auto it = cold_.find(cold_ref);
    if (it == cold_.end()) return;
    if (it->second.readers) it->second.readers--;
    if (it->second.readers == 0 && it->second.doomed) {
        discard_storage(it->second);
        cold_.erase(it);
    }
}

uint64_t Daemon::commit_cold(ColdEntry&& c) {
    uint64_t ref = next_cold_++;
    cold_.emplace(ref, std::move(c));
    return ref;
}

void Daemon::enqueue_drain(const Lease& L) {
    set_run_state(L.base, L.count, OFLD_SLOT_DRAIN_IN_FLIGHT);
    ++drains_pending_;
    drain_settled(L.base);  // a stale entry for this base (run freed and reused) leaves the count first
    draining_slots_ += L.count;
    drain_queued_[L.base] = L.count;
    {
        std::lock_guard<std::mutex> q(q_mu_);
        drain_q_.push_back(DrainJob{L.base, L.count});
    }
    drain_cv_.notify_one();
    Metrics::get().inc(M::kDrainsEnqueued);
    Metrics::get().add(M::kDrainingBytes, L.nbytes);
}

// The slots of a queued drain stop counting as "about to be freed" once the
// drain is done or skipped, or as soon as the run is freed by another path
// (discard, recovery) while the job still waits in the queue: used_slots_
// drops at that moment, so keeping them in draining_slots_ would subtract
// them twice and make pressure drains stop short. mu_ held.
void Daemon::drain_settled(uint32_t base) {
    auto it = drain_queued_.find(base);
    if (it == drain_queued_.end()) return;
    draining_slots_ -= std::min<uint64_t>(draining_slots_, it->second);
    drain_queued_.erase(it);
}

// Under the normal/priority/aggressive thresholds, queue background drains of
// the least recently touched pinned runs until pressure falls back under the
// normal threshold. Runs already queued for a drain count as gone: this runs
// on every D2H completion, and a batch completes many runs before the first
// drain frees its slots, so counting them again would drain the whole batch.
// mu_ held.
void Daemon::pressure_drain() {
    double p = pinned_pressure();
    if (p < cfg_.normal_threshold || layout_.num_slots == 0) return;
    M bucket = p >= cfg_.aggressive_threshold ? M::kPressureDrainsAggressive
               : p >= cfg_.priority_threshold ? M::kPressureDrainsPriority
                                              : M::kPressureDrainsNormal;
    uint64_t target = uint64_t(cfg_.normal_threshold * double(layout_.num_slots));
    uint64_t projected = used_slots_ > draining_slots_ ? used_slots_ - draining_slots_ : 0;
    if (projected <= target) return;
    for (auto it = lru_.begin(); it != lru_.end() && projected > target;) {
        uint64_t lid = it->second;
        ++it;
        Lease* L = lease(lid);
        if (!L || L->prefetch || state_of(L->base) != OFLD_SLOT_PINNED_VALID) continue;
        if (is_canonical_tid(L->tensor_id)) {
            CanonicalObject* o = find_object(L->tensor_id & ~kCanonicalTidBit);
            if (!o || o->state == OBJ_CREATING || o->restore_refs || o->export_refs) continue;
        }
        lru_.erase({L->lru_ts, lid});
        L->lru_ts = 0;
        enqueue_drain(*L);
        Metrics::get().inc(bucket);
        projected = projected > L->count ? projected - L->count : 0;
    }
}

// Source of a drain: returns an existing cold copy of the same (tensor,
// version) when one is still valid, so a re-drain of a warmed run only frees
// the pinned copy. mu_ held.
uint64_t Daemon::reusable_cold(uint64_t tid, uint64_t ver) {
    auto lit = locations_.find(tid);
    if (lit == locations_.end() || lit->second.version != ver || !lit->second.cold_ref) return 0;
    auto cit = cold_.find(lit->second.cold_ref);
    return cit != cold_.end() && !cit->second.doomed ? lit->second.cold_ref : 0;
}

// Commit a finished drain of run [base, base+count) (mu_ held). `ref` is the
// cold copy (0 when the write failed). A canonical object with an export or
// local restore streaming from the pinned run keeps the run resident and just
// gains the cold copy (multi-tier).
void Daemon::finish_drain(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint64_t lid,
                          uint32_t owner, uint64_t nbytes, uint64_t ref) {
    if (state_of(base) != OFLD_SLOT_DRAIN_IN_FLIGHT || slots_[base].lease_id != lid) {
        if (ref && ref != reusable_cold(tid, ver)) free_cold(ref);  // raced with recovery
        return;
    }
    if (!lease(lid)) {
        // The owner released the object while its bytes were being drained
        // (release leaves a draining run alone): drop both copies here.
        if (ref && ref != reusable_cold(tid, ver)) free_cold(ref);
        free_run(base, count);
        return;
    }
    if (!ref) {
        set_run_state(base, count, OFLD_SLOT_PINNED_VALID);
        note_drainable(lid);
        Metrics::get().inc(M::kIoFailure);
        return;
    }
    ofld_location_kind_t kind = cold_[ref].kind;
    set_cold_ref(base, count, ref);
    CanonicalObject* o = nullptr;
    if (is_canonical_tid(tid) && !is_candidate_tid(tid)) o = find_object(tid & ~kCanonicalTidBit);
    if (storage_busy(tid) || (o && (o->export_refs || o->restore_refs))) {
        set_run_state(base, count, OFLD_SLOT_PINNED_VALID);
        set_location(tid, ver, OFLD_LOC_PINNED, base, ref, nbytes);
        // `o` is null when the storage outlived the object that created it
        // (carried-forward objects still read it)
        if (o && o->state == OBJ_VALID_PINNED) o->state = OBJ_VALID_MULTI_TIER;
        note_drainable(lid);
        return;
    }
    set_state(base, OFLD_SLOT_COLD_VALID);
    set_location(tid, ver, kind, base, ref, nbytes);
    Trace::get().event("COLD_VALID", owner, 0, tid, ver, lid, base, nbytes);
    if (o) {
        if (o->state == OBJ_VALID_PINNED || o->state == OBJ_VALID_MULTI_TIER)
            o->state = kind == OFLD_LOC_NVME ? OBJ_VALID_NVME : OBJ_VALID_PAGEABLE;
        o->base_slot = 0xFFFFFFFFu;
        if (Job* j = find_job(o->key.job)) {
            j->pinned_bytes -= std::min(j->pinned_bytes, nbytes);
            (kind == OFLD_LOC_NVME ? j->nvme_bytes : j->pageable_bytes) += nbytes;
        }
    }
    free_run(base, count);
    erase_lease(lid);
    Metrics::get().inc(M::kDrainsCompleted);
}

// Synchronously drain the least recently touched pinned run to make room.
// Drops the lock for the copy. Returns true when a run was freed.
bool Daemon::force_drain_one(std::unique_lock<std::mutex>& lk) {
    Lease victim;
    bool found = false;
    for (auto it = lru_.begin(); it != lru_.end();) {
        uint64_t lid = it->second;
        Lease* L = lease(lid);
        if (!L || L->prefetch || state_of(L->base) != OFLD_SLOT_PINNED_VALID) {
            it = lru_.erase(it);
            if (L) L->lru_ts = 0;
            continue;
        }
        if (is_canonical_tid(L->tensor_id)) {
            CanonicalObject* o = find_object(L->tensor_id & ~kCanonicalTidBit);
            bool cp = true, cn = true;
            cold_quota(L->tensor_id, L->nbytes, &cp, &cn);
            if (is_candidate_tid(L->tensor_id) ||
                (o && (o->restore_refs || o->export_refs || o->state == OBJ_CREATING)) ||
                (!cp && !(cn && cfg_.nvme_enabled))) {
                ++it;
                continue;
            }
        }
        it = lru_.erase(it);
        L->lru_ts = 0;
        victim = *L;
        found = true;
        break;
    }
    if (!found) return false;
    set_run_state(victim.base, victim.count, OFLD_SLOT_DRAIN_IN_FLIGHT);
    Trace::get().event("DRAIN_STARTED", victim.owner_rank, 0, victim.tensor_id, victim.version, victim.id,
                       victim.base, victim.nbytes);
    uint64_t ref = reusable_cold(victim.tensor_id, victim.version);
    if (!ref) {
        Metrics::get().add(M::kDrainingBytes, victim.nbytes);
        char* src = slot_ptr(victim.base);
        bool allow_p = true, allow_n = true;
        cold_quota(victim.tensor_id, victim.nbytes, &allow_p, &allow_n);
        lk.unlock();
        ColdEntry cold;
        bool ok = write_cold(src, victim.nbytes, &cold, allow_p, allow_n);
        lk.lock();
        Metrics::get().sub(M::kDrainingBytes, victim.nbytes);
        ref = ok ? commit_cold(std::move(cold)) : 0;
    }
    bool freed = ref != 0 && state_of(victim.base) == OFLD_SLOT_DRAIN_IN_FLIGHT;
    finish_drain(victim.base, victim.count, victim.tensor_id, victim.version, victim.id, victim.owner_rank,
                 victim.nbytes, ref);
    return freed || state_of(victim.base) == OFLD_SLOT_FREE;
}

void Daemon::drain_loop() {
    for (;;) {
        DrainJob job;
        {
            std::unique_lock<std::mutex> q(q_mu_);
            drain_cv_.wait(q, [&] { return !drain_q_.empty() || !workers_on_.load(); });
            if (drain_q_.empty()) return;
            job = drain_q_.front();
            drain_q_.pop_front();
        }
        uint64_t nbytes, tid, ver, lid, ref;
        uint32_t owner;
        char* src;
        bool allow_p = true, allow_n = true;
        {
            std::lock_guard<std::mutex> g(mu_);
            if (state_of(job.base) != OFLD_SLOT_DRAIN_IN_FLIGHT) {
                Metrics::get().sub(M::kDrainingBytes, slots_[job.base].nbytes);
                if (drains_pending_) --drains_pending_;
                drain_settled(job.base);
                drained_cv_.notify_all();
                continue;
            }
            const ofld_slot_entry_t& e = slots_[job.base];
            nbytes = e.nbytes;
            tid = e.tensor_id;
            ver = e.version;
            lid = e.lease_id;
            owner = uint32_t(e.owner_rank);
            src = slot_ptr(job.base);
            ref = reusable_cold(tid, ver);
            cold_quota(tid, nbytes, &allow_p, &allow_n);
            if (!ref && !allow_p && !(allow_n && cfg_.nvme_enabled)) {
                // the job is at its cold-tier quotas: the run stays pinned
                set_run_state(job.base, job.count, OFLD_SLOT_PINNED_VALID);
                Metrics::get().inc(M::kQuotaRejections);
                Metrics::get().sub(M::kDrainingBytes, nbytes);
                if (drains_pending_) --drains_pending_;
                drain_settled(job.base);
                drained_cv_.notify_all();
                continue;
            }
        }
        Trace::get().event("DRAIN_STARTED", owner, 0, tid, ver, lid, job.base, nbytes);
        ColdEntry cold;
        bool ok = ref != 0 || write_cold(src, nbytes, &cold, allow_p, allow_n);
        std::lock_guard<std::mutex> g(mu_);
        Metrics::get().sub(M::kDrainingBytes, nbytes);
        if (!ref && ok) ref = commit_cold(std::move(cold));
        finish_drain(job.base, job.count, tid, ver, lid, owner, nbytes, ref);
        if (drains_pending_) --drains_pending_;
        drain_settled(job.base);
        drained_cv_.notify_all();
    }
}

void Daemon::readback_loop() {
    for (;;) {
        ReadbackJob job;
        {
            std::unique_lock<std::mutex> q(q_mu_);
            readback_cv_.wait(q, [&] { return !readback_q_.empty() || !workers_on_.load(); });
            if (readback_q_.empty()) return;
            job = readback_q_.front();
            readback_q_.pop_front();
        }
        ColdEntry cold;
        char* dst;
        // A failed readback gives the run back; the location still points at
        // the cold copy, so the rank's next prefetch poll retries.
        auto fail_job = [&] {
            uint64_t lid = slots_[job.base].lease_id;
            free_run(job.base, job.count);
            erase_lease(lid);
            Metrics::get().inc(M::kIoFailure);
        };
        {
            std::lock_guard<std::mutex> g(mu_);
            if (state_of(job.base) != OFLD_SLOT_READBACK_IN_FLIGHT) continue;
            if (!pin_cold(job.cold_ref, &cold)) {
                fail_job();
                continue;
            }
            dst = slot_ptr(job.base);
        }
        bool ok = read_cold(cold, dst, 0, job.nbytes);
        std::lock_guard<std::mutex> g(mu_);
        unpin_cold(job.cold_ref);
        if (state_of(job.base) != OFLD_SLOT_READBACK_IN_FLIGHT) continue;
        if (!ok) {
            fail_job();
            continue;
        }
        uint64_t tid = slots_[job.base].tensor_id, ver = slots_[job.base].version;
        set_run_state(job.base, job.count, OFLD_SLOT_PINNED_VALID);
        set_location(tid, ver, OFLD_LOC_PINNED, job.base, job.cold_ref, job.nbytes);
        Metrics::get().inc(M::kReadbacksCompleted);
        Trace::get().event("PINNED_READY", uint32_t(slots_[job.base].owner_rank), 0, tid, ver,
                           slots_[job.base].lease_id, job.base, job.nbytes);
    }
}

}  // namespace ofld
