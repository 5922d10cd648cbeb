// Slot allocator, leases, the location table and the v1 transfer RPCs.
//
// Slot state machine and RPC semantics follow StateSpectre
// (reference: src/daemon/daemon.cpp:298-461 allocator, :856-1437 handlers):
// RequestOffload reserves a contiguous run (own GPU window, then same-NUMA
// overflow, then borrowable peer windows, then remote NUMA only when allowed),
// forcing synchronous drains of the least recently touched pinned runs when
// full; completions are rejected on a stale epoch, wrong owner, wrong
// (tensor, version) or an invalid state transition, and each rejection is
// counted.
#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstring>

#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"

namespace ofld {

namespace {
constexpr const char* TAG = "slots";

// First run of `count` set bits in a bitmap of `nbits` bits, or -1.
int64_t find_free_run(const std::vector<uint64_t>& bm, uint32_t nbits, uint32_t count) {
    uint64_t run = 0, start = 0;
    for (uint32_t w = 0; w < bm.size(); ++w) {
        uint64_t x = bm[w];
        if (x == ~0ull) {
            if (run == 0) start = uint64_t(w) * 64;
            run += 64;
            if (run >= count) return int64_t(start);
            continue;
        }
        if (x == 0) {
            run = 0;
            continue;
        }
        for (uint32_t b = 0; b < 64; ++b) {
            if ((x >> b) & 1ull) {
                if (run == 0) start = uint64_t(w) * 64 + b;
                if (++run >= count) return start + count <= nbits ? int64_t(start) : -1;
            } else {
                run = 0;
            }
        }
    }
    return -1;
}

// Best fit: the smallest free run that holds `count` bits (ties: the higher
// one), placed at the top of that run.
int64_t find_free_run_best(const std::vector<uint64_t>& bm, uint32_t nbits, uint32_t count) {
    int64_t best = -1;
    uint64_t best_len = ~0ull;
    uint64_t run = 0, start = 0;
    auto close = [&](uint64_t end) {  // run occupies [start, end)
        if (run >= count && run <= best_len) {
            best_len = run;
            best = int64_t(end - count);
        }
        run = 0;
    };
    for (uint32_t w = 0; w < bm.size(); ++w) {
        const uint64_t x = bm[w];
        const uint64_t base = uint64_t(w) * 64;
        if (x == ~0ull && base + 64 <= nbits) {
            if (run == 0) start = base;
            run += 64;
            continue;
        }
        for (uint32_t b = 0; b < 64; ++b) {
            const uint64_t i = base + b;
            if (i >= nbits) break;
            if ((x >> b) & 1ull) {
                if (run == 0) start = i;
                ++run;
            } else if (run) {
                close(i);
            }
        }
    }
    if (run) close(start + run);
    return best;
}
}  // namespace

void Daemon::set_state(uint32_t s, ofld_slot_state_t st) {
    slots_[s].last_touch_ns = real_ns();
    slots_[s].state.store(uint32_t(st), std::memory_order_relaxed);
    publish_slot(s);
}
void Daemon::publish_slot(uint32_t s) {
    constexpr size_t kBody = offsetof(ofld_slot_entry_t, slot_id);  // everything after the atomic state
    std::memcpy(reinterpret_cast<char*>(&pub_slots_[s]) + kBody, reinterpret_cast<const char*>(&slots_[s]) + kBody,
                sizeof(ofld_slot_entry_t) - kBody);
    pub_slots_[s].state.store(slots_[s].state.load(std::memory_order_relaxed), std::memory_order_release);
}
void Daemon::set_cold_ref(uint32_t base, uint32_t count, uint64_t ref) {
    for (uint32_t k = 0; k < count; ++k) {
        slots_[base + k].cold_ref = ref;
        publish_slot(base + k);
    }
}
void Daemon::set_run_state(uint32_t base, uint32_t count, ofld_slot_state_t st) {
    for (uint32_t k = 0; k < count; ++k) set_state(base + k, st);
}
uint32_t Daemon::state_of(uint32_t s) const { return slots_[s].state.load(std::memory_order_relaxed); }
char* Daemon::slot_ptr(uint32_t s) { return arenas_[slots_[s].arena_id].base + slots_[s].arena_offset; }
uint32_t Daemon::slots_for(uint64_t nbytes) const {
    uint64_t n = (nbytes + cfg_.allocation_granularity_bytes - 1) / cfg_.allocation_granularity_bytes;
    return uint32_t(std::max<uint64_t>(n, 1));
}
double Daemon::pinned_pressure() const {
    return layout_.num_slots ? double(used_slots_) / double(layout_.num_slots) : 0.0;
}
Daemon::Window* Daemon::window_of_slot(uint32_t s) {
    return s < slot_window_.size() && slot_window_[s] != 0xFFFFFFFFu ? &windows_[slot_window_[s]] : nullptr;
}

// Size-segregated placement: runs of kLargeRun slots or more go best-fit
// (smallest hole that holds them, placed at its top; model tensors repeat in
// size, so a freed hole is usually refilled exactly), smaller ones first-fit
// from the bottom, so freeing many small objects (norms, biases, KV blocks)
// does not splinter the space that multi-GB tensors need as one run.
bool Daemon::alloc_in_window(Window& w, uint32_t count, uint32_t* base) {
    constexpr uint32_t kLargeRun = 8;
    if (count > w.nslots) return false;
    int64_t rel = count >= kLargeRun ? find_free_run_best(w.free_bits, w.nslots, count)
                                     : find_free_run(w.free_bits, w.nslots, count);
    if (rel < 0) return false;
    for (uint32_t k = 0; k < count; ++k) {
        uint64_t i = uint64_t(rel) + k;
        w.free_bits[i / 64] &= ~(1ull << (i % 64));
    }
    *base = w.first_slot + uint32_t(rel);
    used_slots_ += count;
    Metrics::get().add(M::kUsedPinnedBytes, uint64_t(count) * cfg_.allocation_granularity_bytes);
    return true;
}

void Daemon::free_run(uint32_t base, uint32_t count) {
    drain_settled(base);
    for (uint32_t k = 0; k < count; ++k) {
        uint32_t id = base + k;
        ofld_slot_entry_t& e = slots_[id];
        e.nbytes = e.tensor_id = e.version = e.lease_id = 0;
        e.owner_rank = e.owner_pid = e.rank_epoch = e.cold_ref = 0;
        e.submit_seq = e.complete_seq = e.checksum = 0;
        set_state(id, OFLD_SLOT_FREE);
        if (Window* w = window_of_slot(id)) {
            uint32_t rel = id - w->first_slot;
            uint64_t bit = 1ull << (rel % 64);
            if (!(w->free_bits[rel / 64] & bit)) {
                w->free_bits[rel / 64] |= bit;
                if (used_slots_) --used_slots_;
                Metrics::get().sub(M::kUsedPinnedBytes, cfg_.allocation_granularity_bytes);
            }
        }
    }
}

// Allocation preference chain; forces drains when nothing fits. mu_ held via lk.
bool Daemon::allocate(uint32_t gpu, uint32_t numa, uint64_t nbytes, uint64_t flags, uint32_t* base,
                      uint32_t* count, std::unique_lock<std::mutex>& lk) {
    *count = slots_for(nbytes);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(30);
    for (int attempt = 0; attempt <= 64; ++attempt) {
        auto pick = [&](auto pred) {
            for (Window& w : windows_)
                if (pred(w) && alloc_in_window(w, *count, base)) return true;
            return false;
        };
        if (pick([&](const Window& w) { return !w.overflow && w.numa_node == numa && w.gpu == gpu; }))
            return true;
        if (pick([&](const Window& w) { return w.overflow && w.numa_node == numa; })) return true;
        if (pick([&](const Window& w) { return !w.overflow && w.numa_node == numa; })) return true;
        if ((flags & OFLD_FLAG_ALLOW_REMOTE_NUMA) && pick([&](const Window& w) { return w.numa_node != numa; })) {
            Metrics::get().inc(M::kRemoteNumaAllocs);
            return true;
        }
        if (force_drain_one(lk)) continue;
        // Nothing left to drain synchronously: wait (bounded) for queued
        // background drains to give their pinned runs back, then retry.
        if (drains_pending_ == 0 || std::chrono::steady_clock::now() > deadline) break;
        const uint32_t before = drains_pending_;
        while (drains_pending_ == before && drains_pending_ > 0 && running_.load())
            if (drained_cv_.wait_until(lk, deadline) == std::cv_status::timeout) break;
        if (drains_pending_ == before) break;  // no progress within the bound
        --attempt;                            // a finished drain is not a forced-drain attempt
    }
    return false;
}

void Daemon::stamp_run(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint64_t lease_id,
                       uint32_t rank, uint64_t pid, uint64_t epoch, uint64_t nbytes, uint64_t flags,
                       ofld_slot_state_t st) {
    for (uint32_t k = 0; k < count; ++k) {
        ofld_slot_entry_t& e = slots_[base + k];
        e.tensor_id = tid;
        e.version = ver;
        e.lease_id = lease_id;
        e.owner_rank = rank;
        e.owner_pid = pid;
        e.rank_epoch = epoch;
        e.nbytes = k == 0 ? nbytes : e.capacity;
        e.flags = flags;
        set_state(base + k, st);
    }
}

uint64_t Daemon::new_lease(uint32_t base, uint32_t count, uint64_t tid, uint64_t ver, uint32_t rank,
                           uint64_t epoch, uint64_t nbytes, bool prefetch) {
    Lease L;
    L.id = next_lease_++;
    L.base = base;
    L.count = count;
    L.tensor_id = tid;
    L.version = ver;
    L.owner_rank = rank;
    auto it = sessions_.find(rank);
    L.owner_pid = it != sessions_.end() ? it->second.pid : 0;
    L.epoch = epoch;
    L.nbytes = nbytes;
    L.prefetch = prefetch;
    leases_[L.id] = L;
    if (prefetch) prefetch_by_tv_[{tid, ver}] = L.id;
    return L.id;
}

void Daemon::note_drainable(uint64_t lease_id) {
    auto it = leases_.find(lease_id);
    if (it == leases_.end() || it->second.prefetch) return;
    Lease& L = it->second;
    if (L.lru_ts) lru_.erase({L.lru_ts, lease_id});
    L.lru_ts = std::max<uint64_t>(1, slots_[L.base].last_touch_ns);
    lru_.insert({L.lru_ts, lease_id});
}

Daemon::Lease* Daemon::lease(uint64_t id) {
    auto it = leases_.find(id);
    return it == leases_.end() ? nullptr : &it->second;
}

void Daemon::erase_lease(uint64_t id) {
    auto it = leases_.find(id);
    if (it == leases_.end()) return;
    if (it->second.prefetch) {
        auto p = prefetch_by_tv_.find({it->second.tensor_id, it->second.version});
        if (p != prefetch_by_tv_.end() && p->second == id) prefetch_by_tv_.erase(p);
    }
    if (it->second.lru_ts) lru_.erase({it->second.lru_ts, id});
    leases_.erase(it);
}

bool Daemon::set_location(uint64_t tid, uint64_t ver, ofld_location_kind_t kind, uint32_t slot,
                          uint64_t cold_ref, uint64_t nbytes) {
    auto it = locations_.find(tid);
    if (it != locations_.end() && ver < it->second.version) {
        Metrics::get().inc(M::kStaleVersionRejected);
        return false;
    }
    // The byte format follows the data: read it off a pinned run, keep it
    // while the same version moves between tiers.
    const uint64_t prev_fmt = it != locations_.end() && it->second.version == ver ? it->second.fmt : 0;
    Location& L = locations_[tid];
    L.fmt = kind == OFLD_LOC_PINNED && slot < layout_.num_slots ? (slots_[slot].flags & OFLD_FLAG_FORMAT_MASK)
                                                                 : prev_fmt;
    L.version = ver;
    L.kind = kind;
    L.slot = slot;
    L.cold_ref = cold_ref;
    L.nbytes = nbytes;
    return true;
}

// ============================================================================
// RequestOffload
// ============================================================================
RequestOffloadResponse Daemon::do_request_offload(const RequestOffloadRequest& r,
                                                  std::unique_lock<std::mutex>& lk) {
    RequestOffloadResponse resp;
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        Trace::get().event("ERROR", r.rank_id, r.gpu_id, r.tensor_id, r.version, 0, 0, r.nbytes);
        resp.message = "epoch invalid";
        return resp;
    }
    if (r.nbytes == 0) {
        resp.message = "nbytes must be > 0";
        return resp;
    }
    Metrics::get().inc(M::kOffloadRequests);
    Trace::get().event("REQUEST_OFFLOAD", r.rank_id, r.gpu_id, r.tensor_id, r.version, 0, 0, r.nbytes);
    uint32_t base = 0, count = 0;
    if (!allocate(r.gpu_id, r.numa_node, r.nbytes, r.flags, &base, &count, lk)) {
        Metrics::get().inc(M::kBlockedReservations);
        Trace::get().event("ERROR", r.rank_id, r.gpu_id, r.tensor_id, r.version, 0, 0, r.nbytes);
        resp.blocked = true;
        resp.message = "no pinned capacity (blocked / backpressure)";
        return resp;
    }
    // The session may have been invalidated while a forced drain had the lock
    // released; re-check before committing the reservation.
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        free_run(base, count);
        resp.message = "epoch invalid";
        return resp;
    }
    for (uint32_t k = 0; k < count; ++k) {
        if (state_of(base + k) != OFLD_SLOT_FREE) {
            Metrics::get().inc(M::kSlotOverlapPrevented);
            resp.message = "slot overlap prevented";
            return resp;
        }
    }
    const bool submit = (r.flags & OFLD_FLAG_SUBMIT_ON_GRANT) != 0;
    uint64_t lid = new_lease(base, count, r.tensor_id, r.version, r.rank_id, r.rank_epoch, r.nbytes, false);
    stamp_run(base, count, r.tensor_id, r.version, lid, r.rank_id, leases_[lid].owner_pid, r.rank_epoch,
              r.nbytes, r.flags, submit ? OFLD_SLOT_D2H_IN_FLIGHT : OFLD_SLOT_RESERVED_D2H);
    if (submit) Metrics::get().add(M::kInflightD2HBytes, r.nbytes);
    Metrics::get().inc(M::kLeasesGranted);
    resp.ok = true;
    resp.message = "ok";
    resp.lease_id = lid;
    resp.slot_id = base;
    resp.arena_id = slots_[base].arena_id;
    resp.arena_offset = slots_[base].arena_offset;
    resp.capacity = uint64_t(count) * cfg_.allocation_granularity_bytes;
    resp.state = submit ? OFLD_SLOT_D2H_IN_FLIGHT : OFLD_SLOT_RESERVED_D2H;
    Trace::get().event("LEASE_GRANTED", r.rank_id, r.gpu_id, r.tensor_id, r.version, lid, base, r.nbytes);
    if (submit) Trace::get().event("D2H_SUBMITTED", r.rank_id, r.gpu_id, r.tensor_id, r.version, lid, base, r.nbytes);
    return resp;
}

RequestOffloadResponse Daemon::on_request_offload(const RequestOffloadRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    return do_request_offload(r, lk);
}

BatchRequestOffloadResponse Daemon::on_batch_request_offload(const BatchRequestOffloadRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    BatchRequestOffloadResponse resp;
    resp.ok = true;
    resp.message = "ok";
    resp.grants.reserve(r.items.size());
    for (RequestOffloadRequest it : r.items) {
        it.rank_id = r.rank_id;
        it.rank_epoch = r.rank_epoch;
        resp.grants.push_back(do_request_offload(it, lk));
        Metrics::get().inc(M::kBatchOffloadItems);
    }
    return resp;
}

StatusResponse Daemon::on_d2h_submitted(const TransferMark& r) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    Lease* L = lease(r.lease_id);
    if (!L || L->owner_rank != r.rank_id || L->base != r.slot_id) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return {false, "lease/owner/slot mismatch"};
    }
    if (state_of(L->base) != OFLD_SLOT_RESERVED_D2H) {
        Metrics::get().inc(M::kInvalidTransitionRejected);
        return {false, "not in RESERVED_D2H"};
    }
    for (uint32_t k = 0; k < L->count; ++k) slots_[L->base + k].submit_seq = r.seq;
    set_run_state(L->base, L->count, OFLD_SLOT_D2H_IN_FLIGHT);
    Metrics::get().add(M::kInflightD2HBytes, L->nbytes);
    Trace::get().event("D2H_SUBMITTED", r.rank_id, sessions_[r.rank_id].gpu, r.tensor_id, r.version, r.lease_id, r.slot_id, L->nbytes);
    return {true, "ok"};
}

// The coding of a run's bytes, recorded by the rank that copies into it
// (canonical evicts decide it after their reservation). The slot entries carry
// it like the format bits of a v1 reservation, so drains, readbacks,
// restores and exports see it.
StatusResponse Daemon::on_set_run_format(const SetRunFormatRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    if ((r.format & ~OFLD_FLAG_FORMAT_MASK) || r.format == OFLD_FLAG_FORMAT_MASK) return {false, "bad format bits"};
    Lease* L = lease(r.lease_id);
    if (!L || L->owner_rank != r.rank_id || L->base != r.slot_id) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return {false, "lease/owner/slot mismatch"};
    }
    const uint32_t st = state_of(L->base);
    if (st != OFLD_SLOT_RESERVED_D2H && st != OFLD_SLOT_D2H_IN_FLIGHT) {
        Metrics::get().inc(M::kInvalidTransitionRejected);
        return {false, "run not being written"};
    }
    for (uint32_t k = 0; k < L->count; ++k) {
        slots_[L->base + k].flags = (slots_[L->base + k].flags & ~OFLD_FLAG_FORMAT_MASK) | r.format;
        publish_slot(L->base + k);
    }
    return {true, "ok"};
}

bool Daemon::apply_d2h_complete(uint32_t rank, uint64_t epoch, uint64_t lease_id, uint64_t tid,
                                uint64_t ver, uint32_t slot, uint64_t seq, bool* latest, bool* drained) {
    *latest = *drained = false;
    if (!epoch_ok(rank, epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return false;
    }
    Lease* L = lease(lease_id);
    if (!L || L->owner_rank != rank || L->base != slot) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return false;
    }
    if (L->tensor_id != tid || L->version != ver || state_of(L->base) != OFLD_SLOT_D2H_IN_FLIGHT) {
        Metrics::get().inc(M::kInvalidTransitionRejected);
        return false;
    }
    for (uint32_t k = 0; k < L->count; ++k) slots_[L->base + k].complete_seq = seq;
    set_run_state(L->base, L->count, OFLD_SLOT_PINNED_VALID);
    Metrics::get().sub(M::kInflightD2HBytes, L->nbytes);
    Metrics::get().add(M::kD2HBytes, L->nbytes);
    *latest = set_location(tid, ver, OFLD_LOC_PINNED, L->base, 0, L->nbytes);
    uint32_t gpu = sessions_.count(rank) ? sessions_[rank].gpu : 0;
    Trace::get().event("D2H_COMPLETE", rank, gpu, tid, ver, lease_id, L->base, L->nbytes);

    // Canonical bytes stay pinned until their commit lands; candidates are
    // always discarded on commit so they never drain.
    bool hold = false;
    if (is_candidate_tid(tid)) {
        hold = true;
    } else if (is_canonical_tid(tid)) {
        CanonicalObject* o = find_object(tid & ~kCanonicalTidBit);
        hold = o && o->state == OBJ_CREATING;
    }
    if (!hold && cfg_.drain_on_d2h_complete) {
        enqueue_drain(*L);
        *drained = true;
        Trace::get().event("DRAIN_ENQUEUED", rank, gpu, tid, ver, lease_id, L->base, L->nbytes);
    } else {
        note_drainable(lease_id);
        if (!hold) pressure_drain();
    }
    return true;
}

MarkD2HCompleteResponse Daemon::on_d2h_complete(const TransferMark& r) {
    std::lock_guard<std::mutex> g(mu_);
    MarkD2HCompleteResponse resp;
    resp.ok = apply_d2h_complete(r.rank_id, r.rank_epoch, r.lease_id, r.tensor_id, r.version, r.slot_id,
                                 r.seq, &resp.latest_version, &resp.drain_enqueued);
    resp.message = resp.ok ? "ok" : "rejected";
    if (!resp.ok) Trace::get().event("ERROR", r.rank_id, 0, r.tensor_id, r.version, r.lease_id, r.slot_id, 0);
    return resp;
}

// ============================================================================
// Prefetch / H2D
// ============================================================================
RequestPrefetchResponse Daemon::do_request_prefetch(const RequestPrefetchRequest& r,
                                                    std::unique_lock<std::mutex>& lk) {
    RequestPrefetchResponse resp;
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    Metrics::get().inc(M::kPrefetchRequests);
    auto it = locations_.find(r.tensor_id);
    if (it == locations_.end()) {
        resp.message = "unknown tensor";
        return resp;
    }
    Location loc = it->second;
    uint64_t want = r.version ? r.version : loc.version;
    if (want != loc.version) {
        resp.message = "requested version not latest/available";
        return resp;
    }
    if (loc.kind == OFLD_LOC_NONE || loc.kind == OFLD_LOC_DELETED || loc.kind == OFLD_LOC_ERROR) {
        resp.message = "tensor not resident";
        return resp;
    }
    const uint32_t gpu = r.gpu_id;
    Trace::get().event("PREFETCH_REQUESTED", r.rank_id, gpu, r.tensor_id, want, 0, loc.slot, loc.nbytes);
    const bool submit = (r.flags & OFLD_FLAG_SUBMIT_ON_READY) != 0;
    auto fill = [&](uint64_t lid, uint32_t base, uint32_t st) {
        resp.ok = true;
        resp.lease_id = lid;
        resp.slot_id = base;
        resp.arena_id = slots_[base].arena_id;
        resp.arena_offset = slots_[base].arena_offset;
        resp.nbytes = loc.nbytes;
        resp.version = want;
        resp.state = st;
    };
    auto mark_ready = [&](Lease& L) {
        if (submit) {
            set_run_state(L.base, L.count, OFLD_SLOT_H2D_IN_FLIGHT);
            Metrics::get().add(M::kInflightH2DBytes, L.nbytes);
            Trace::get().event("H2D_SUBMITTED", r.rank_id, gpu, r.tensor_id, want, L.id, L.base, L.nbytes);
        }
        resp.ready = true;
        resp.state = submit ? OFLD_SLOT_H2D_IN_FLIGHT : OFLD_SLOT_PINNED_VALID;
        resp.message = "ok";  // StateSpectre's text for a pinned-ready prefetch
        Trace::get().event("PINNED_READY", r.rank_id, gpu, r.tensor_id, want, L.id, L.base, L.nbytes);
    };

    // Re-poll while a readback is in flight: hand back the same lease.
    auto pit = prefetch_by_tv_.find({r.tensor_id, want});
    if (pit != prefetch_by_tv_.end()) {
        Lease* EL = lease(pit->second);
        if (EL) {
            uint32_t st = state_of(EL->base);
            if (st == OFLD_SLOT_READBACK_IN_FLIGHT || st == OFLD_SLOT_PINNED_VALID) {
                fill(EL->id, EL->base, st);
                if (st == OFLD_SLOT_PINNED_VALID) {
                    mark_ready(*EL);
                    resp.message = "ready";  // StateSpectre's text for a landed readback
                } else {
                    resp.message = "readback in flight";
                }
                return resp;
            }
        }
    }

    if (loc.kind == OFLD_LOC_PINNED && state_of(loc.slot) == OFLD_SLOT_PINNED_VALID) {
        uint64_t lid = new_lease(loc.slot, slots_for(loc.nbytes), r.tensor_id, want, r.rank_id,
                                 r.rank_epoch, loc.nbytes, true);
        fill(lid, loc.slot, OFLD_SLOT_PINNED_VALID);
        mark_ready(leases_[lid]);
        return resp;
    }
    if (loc.kind == OFLD_LOC_PINNED) {
        // Drain or another transfer in flight on the run: not ready yet, the
        // caller polls again (a finished drain turns this into a readback).
        resp.ok = true;
        resp.ready = false;
        resp.state = state_of(loc.slot);
        resp.version = want;
        resp.nbytes = loc.nbytes;
        resp.message = "pinned copy transitioning";
        return resp;
    }
    // Cold: allocate a pinned run and read it back in the background.
    uint32_t base = 0, count = 0;
    if (!allocate(r.gpu_id, r.numa_node, loc.nbytes, r.flags | OFLD_FLAG_ALLOW_REMOTE_NUMA, &base, &count, lk)) {
        Metrics::get().inc(M::kBlockedReservations);
        uint32_t largest = 0;
        for (const Window& w : windows_) largest = std::max(largest, w.nslots);
        if (slots_for(loc.nbytes) > largest) {
            resp.message = "no pinned window can hold this tensor for readback";
            return resp;
        }
        // Every pinned run is busy (transfers in flight, prefetch leases not
        // yet released, nothing left to drain): they free up as other
        // restores finish, so this is backpressure, not a failure. The caller
        // polls again, as it does while a readback is in flight.
        resp.ok = true;
        resp.ready = false;
        resp.state = OFLD_SLOT_FREE;
        resp.version = want;
        resp.nbytes = loc.nbytes;
        resp.message = "waiting for pinned capacity for readback";
        return resp;
    }
    // The lock may have been released by a forced drain; re-validate.
    auto it2 = locations_.find(r.tensor_id);
    if (!epoch_ok(r.rank_id, r.rank_epoch) || it2 == locations_.end() || it2->second.version != want ||
        it2->second.cold_ref != loc.cold_ref) {
        free_run(base, count);
        resp.message = "location changed during allocation; retry";
        return resp;
    }
    uint64_t lid = new_lease(base, count, r.tensor_id, want, r.rank_id, r.rank_epoch, loc.nbytes, true);
    stamp_run(base, count, r.tensor_id, want, lid, r.rank_id, leases_[lid].owner_pid, r.rank_epoch,
              loc.nbytes, (r.flags & ~OFLD_FLAG_FORMAT_MASK) | loc.fmt, OFLD_SLOT_READBACK_IN_FLIGHT);
    set_cold_ref(base, count, loc.cold_ref);
    {
        std::lock_guard<std::mutex> q(q_mu_);
        readback_q_.push_back(ReadbackJob{base, count, loc.cold_ref, loc.nbytes});
    }
    readback_cv_.notify_one();
    Metrics::get().inc(M::kReadbacksStarted);
    Trace::get().event("READBACK_STARTED", r.rank_id, gpu, r.tensor_id, want, lid, base, loc.nbytes);
    fill(lid, base, OFLD_SLOT_READBACK_IN_FLIGHT);
    resp.message = "readback started";
    return resp;
}

RequestPrefetchResponse Daemon::on_request_prefetch(const RequestPrefetchRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    drain_rings();
    return do_request_prefetch(r, lk);
}

BatchRequestPrefetchResponse Daemon::on_batch_request_prefetch(const BatchRequestPrefetchRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    drain_rings();
    BatchRequestPrefetchResponse resp;
    resp.ok = true;
    resp.message = "ok";
    for (RequestPrefetchRequest it : r.items) {
        it.rank_id = r.rank_id;
        it.rank_epoch = r.rank_epoch;
        resp.results.push_back(do_request_prefetch(it, lk));
        Metrics::get().inc(M::kBatchPrefetchItems);
    }
    return resp;
}

StatusResponse Daemon::on_h2d_submitted(const TransferMark& r) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    Lease* L = lease(r.lease_id);
    if (!L || L->owner_rank != r.rank_id || L->base != r.slot_id) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return {false, "lease/owner/slot mismatch"};
    }
    if (state_of(L->base) != OFLD_SLOT_PINNED_VALID) {
        Metrics::get().inc(M::kInvalidTransitionRejected);
        return {false, "slot not PINNED_VALID"};
    }
    for (uint32_t k = 0; k < L->count; ++k) slots_[L->base + k].submit_seq = r.seq;
    set_run_state(L->base, L->count, OFLD_SLOT_H2D_IN_FLIGHT);
    Metrics::get().add(M::kInflightH2DBytes, L->nbytes);
    Trace::get().event("H2D_SUBMITTED", r.rank_id, 0, r.tensor_id, r.version, r.lease_id, r.slot_id, L->nbytes);
    return {true, "ok"};
}

bool Daemon::apply_h2d_complete(uint32_t rank, uint64_t epoch, uint64_t lease_id, uint64_t tid,
                                uint64_t ver, uint32_t slot, bool keep_pinned, uint64_t seq) {
    if (!epoch_ok(rank, epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return false;
    }
    Lease* L = lease(lease_id);
    if (!L || L->owner_rank != rank || L->base != slot) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return false;
    }
    if (state_of(L->base) != OFLD_SLOT_H2D_IN_FLIGHT) {
        Metrics::get().inc(M::kInvalidTransitionRejected);
        return false;
    }
    const uint32_t base = L->base, count = L->count;
    const uint64_t nbytes = L->nbytes;
    for (uint32_t k = 0; k < count; ++k) slots_[base + k].complete_seq = seq;
    Metrics::get().sub(M::kInflightH2DBytes, nbytes);
    Metrics::get().add(M::kH2DBytes, nbytes);
    Trace::get().event("H2D_COMPLETE", rank, 0, tid, ver, lease_id, base, nbytes);

    uint64_t cold_ref = slots_[base].cold_ref;
    auto lit = locations_.find(tid);
    if (lit != locations_.end() && lit->second.cold_ref) cold_ref = lit->second.cold_ref;
    auto cit = cold_ref ? cold_.find(cold_ref) : cold_.end();
    if (!keep_pinned && cit != cold_.end()) {
        // The cold copy remains the durable one; give the pinned run back.
        if (lit != locations_.end() && lit->second.slot == base && lit->second.version == ver) {
            lit->second.kind = cit->second.kind;
            lit->second.slot = 0;
        }
        free_run(base, count);
        erase_lease(lease_id);
    } else {
        set_run_state(base, count, OFLD_SLOT_PINNED_VALID);
        set_location(tid, ver, OFLD_LOC_PINNED, base, cold_ref, nbytes);
        // The run is drainable again through the lease that stamped it (the
        // original offload lease); the one-shot prefetch binding goes away.
        note_drainable(slots_[base].lease_id);
        if (L->prefetch) erase_lease(lease_id);
    }
    return true;
}

StatusResponse Daemon::on_h2d_complete(const MarkH2DCompleteRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    bool ok = apply_h2d_complete(r.rank_id, r.rank_epoch, r.lease_id, r.tensor_id, r.version, r.slot_id,
                                 r.keep_pinned, r.seq);
    if (!ok) Trace::get().event("ERROR", r.rank_id, 0, r.tensor_id, r.version, r.lease_id, r.slot_id, 0);
    return {ok, ok ? "ok" : "rejected"};
}

StatusResponse Daemon::on_release_lease(const ReleaseLeaseRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    drain_rings();
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    Lease* L = lease(r.lease_id);
    if (!L) return {true, "already released"};
    if (L->owner_rank != r.rank_id) {
        Metrics::get().inc(M::kLeaseOwnerMismatchRejected);
        return {false, "not lease owner"};
    }
    const uint32_t base = L->base, count = L->count;
    const uint64_t tid = L->tensor_id, ver = L->version;
    const bool prefetch = L->prefetch;
    uint32_t st = state_of(base);
    Trace::get().event("LEASE_RELEASED", r.rank_id, 0, tid, ver, r.lease_id, base, 0);
    if (st == OFLD_SLOT_DRAIN_IN_FLIGHT || st == OFLD_SLOT_COLD_VALID) {
        // The drain worker owns the run now; only the binding goes away.
        erase_lease(r.lease_id);
        return {true, "ok (slot managed by drain)"};
    }
    auto lit = locations_.find(tid);
    // Releasing a prefetch lease over the resident pinned copy only drops the
    // binding when another (offload) lease still owns the run.
    const uint64_t owner_lease = slots_[base].lease_id;
    const bool shared = owner_lease != r.lease_id && leases_.count(owner_lease) != 0;
    if (prefetch && shared) {
        if (st == OFLD_SLOT_H2D_IN_FLIGHT) set_run_state(base, count, OFLD_SLOT_PINNED_VALID);
        erase_lease(r.lease_id);
        return {true, "ok"};
    }
    if (lit != locations_.end() && lit->second.kind == OFLD_LOC_PINNED && lit->second.slot == base &&
        lit->second.version == ver) {
        if (lit->second.cold_ref && cold_.count(lit->second.cold_ref)) {
            lit->second.kind = cold_[lit->second.cold_ref].kind;
            lit->second.slot = 0;
        } else {
            lit->second.kind = OFLD_LOC_NONE;
        }
    }
    free_run(base, count);
    // Any other lease over the same run (offload + prefetch pair) dies too.
    std::vector<uint64_t> dead{r.lease_id};
    if (owner_lease != r.lease_id) dead.push_back(owner_lease);
    auto pf = prefetch_by_tv_.find({tid, ver});
    if (pf != prefetch_by_tv_.end() && pf->second != r.lease_id) {
        Lease* P = lease(pf->second);
        if (P && P->base == base) dead.push_back(pf->second);
    }
    for (uint64_t id : dead) erase_lease(id);
    return {true, "ok"};
}

// Drop every copy of a rank-owned tensor: its pinned run (unless a transfer
// is in flight on it), its cold copy and its location entry. StateSpectre's
// discard released only the lease, so a drained tensor's pageable/NVMe copy
// was never freed (reference: src/agent/agent.cpp:1100-1131).
StatusResponse Daemon::on_discard_tensor(const DiscardTensorRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    drain_rings();
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    return do_discard(r.rank_id, r.tensor_id, r.version);
}

BatchDiscardTensorResponse Daemon::on_batch_discard(const BatchDiscardTensorRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    drain_rings();
    BatchDiscardTensorResponse resp;
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    resp.ok = true;
    resp.message = "ok";
    for (const TensorVersion& it : r.items) resp.results.push_back(do_discard(r.rank_id, it.tensor_id, it.version));
    return resp;
}

StatusResponse Daemon::do_discard(uint32_t rank, uint64_t tid, uint64_t ver) {
    const DiscardTensorRequest r{rank, 0, tid, ver};
    if (is_canonical_tid(r.tensor_id)) return {false, "canonical objects are released, not discarded"};
    auto it = locations_.find(r.tensor_id);
    if (it == locations_.end()) return {true, "unknown tensor (already discarded)"};
    if (r.version && it->second.version != r.version) return {true, "version superseded"};
    Location loc = it->second;
    if (loc.kind == OFLD_LOC_PINNED) {
        uint32_t st = state_of(loc.slot);
        if (st == OFLD_SLOT_H2D_IN_FLIGHT || st == OFLD_SLOT_DRAIN_IN_FLIGHT || st == OFLD_SLOT_READBACK_IN_FLIGHT)
            return {false, "transfer in flight; retry"};
        if (st == OFLD_SLOT_PINNED_VALID && slots_[loc.slot].tensor_id == r.tensor_id) {
            uint64_t owner = slots_[loc.slot].lease_id;
            free_run(loc.slot, slots_for(loc.nbytes));
            erase_lease(owner);
        }
    }
    auto pf = prefetch_by_tv_.find({r.tensor_id, loc.version});
    if (pf != prefetch_by_tv_.end()) erase_lease(pf->second);
    if (loc.cold_ref) free_cold(loc.cold_ref);
    locations_.erase(it);
    Trace::get().event("LEASE_RELEASED", r.rank_id, 0, r.tensor_id, loc.version, 0, loc.slot, loc.nbytes);
    return {true, "ok"};
}

LocationQueryResponse Daemon::on_query_location(const LocationQueryRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    drain_rings();
    LocationQueryResponse resp;
    auto it = locations_.find(r.tensor_id);
    if (it == locations_.end()) {
        resp.message = "unknown tensor";
        return resp;
    }
    if (r.version && r.version != it->second.version) {
        resp.message = "version not latest";
        return resp;
    }
    resp.ok = true;
    resp.message = "ok";
    resp.location_kind = it->second.kind;
    resp.slot_id = it->second.slot;
    resp.nbytes = it->second.nbytes;
    resp.version = it->second.version;
    return resp;
}

BatchCompleteResponse Daemon::on_batch_complete(const BatchCompleteRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    BatchCompleteResponse resp;
    for (const BatchCompletion& c : r.completions) {
        bool ok = false;
        if (c.event_type == uint32_t(EventType::kD2HComplete)) {
            bool latest, drained;
            ok = apply_d2h_complete(r.rank_id, r.rank_epoch, c.lease_id, c.tensor_id, c.version, c.slot_id,
                                    c.seq, &latest, &drained);
        } else if (c.event_type == uint32_t(EventType::kH2DComplete)) {
            ok = apply_h2d_complete(r.rank_id, r.rank_epoch, c.lease_id, c.tensor_id, c.version, c.slot_id,
                                    c.keep_pinned, c.seq);
        } else {
            Metrics::get().inc(M::kInvalidTransitionRejected);
        }
        (ok ? resp.accepted : resp.rejected)++;
    }
    resp.ok = true;
    resp.message = "ok";
    return resp;
}

}  // namespace ofld
