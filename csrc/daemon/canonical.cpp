// Canonical model-state store: job namespaces, attach-or-create
// deduplication, commit/verify, and per-rank holds.
//
// Semantics follow StateSpectre's canonical store (reference:
// src/daemon/canonical.cpp:126-637): a canonical object's bytes ride the v1
// slot/lease/drain machinery under a synthetic tensor id; the first rank to
// evict a key creates the object (NEED_D2H_CREATE), later replicas attach
// without any copy (semantic_trusted) or verify by content hash
// (hash_verified), concurrent creators either wait or get a throwaway
// candidate slot, and an object is reclaimed once no rank holds it and no
// export/restore is in flight.
//
// Additions of this runtime: dedup mode 4 ("device_hash_verified") answers an
// existing object with action 6 (verify-hash-only): the replica hashes its own
// GPU copy and commits the hash with lease 0, so no pinned slot is reserved and
// no byte crosses PCIe for verification. Mode 5 ("p2p_verified") is for a
// replica that already compared its bytes with the owner's GPU copy over
// NVLink (K3, statespectre_b200.parallel.dp_dedup): an existing object is
// attached at once and answered with action 7.
#include <cstring>

#include "daemon.h"
#include "ofld/chunk_hash.h"
#include "ofld/log.h"
#include "ofld/metrics.h"

namespace ofld {

namespace {
constexpr const char* TAG = "canonical";

bool readable(CanonicalObjectState s) {
    return s == OBJ_VALID_PINNED || s == OBJ_VALID_PAGEABLE || s == OBJ_VALID_NVME || s == OBJ_VALID_MULTI_TIER ||
           s == OBJ_SEALED || s == OBJ_EXPORT_IN_FLIGHT;
}
}  // namespace

// Identity string of a key: every partition axis, never dp_rank or the
// display name. With cross-job dedup the job identity is left out so jobs
// that publish the same bytes share one object.
std::string Daemon::key_string(const CanonicalTensorKeyWire& k, bool cross_job) {
    std::string s;
    s.reserve(192);
    auto u = [&](uint64_t v) {
        s += std::to_string(v);
        s += ':';
    };
    if (!cross_job) {
        u(k.job.tenant_id);
        u(k.job.job_id);
        u(k.job.launch_epoch);
    } else {
        u(k.job.tenant_id);
    }
    u(k.model_role);
    u(k.model_version);
    u(k.param_id);
    u(k.param_fqn_hash);
    u(k.dtype);
    u(k.layout);
    u(k.nbytes);
    u(k.shape_hash);
    u(k.stride_hash);
    u(k.pp_rank);
    u(k.tp_rank);
    u(k.ep_rank);
    u(k.etp_rank);
    s += std::to_string(int64_t(k.expert_id));
    s += ':';
    u(k.shard_offset);
    u(k.shard_nbytes);
    return s;
}

Job* Daemon::find_job(const JobKeyWire& j) {
    auto it = jobs_.find(JobUID{j.tenant_id, j.job_id, j.launch_epoch});
    return it == jobs_.end() ? nullptr : &it->second;
}

CanonicalObject* Daemon::find_object(uint64_t oid) {
    auto it = objects_.find(oid);
    return it == objects_.end() ? nullptr : &it->second;
}

bool Daemon::quota_allows_pinned(const Job& j, uint64_t nbytes) const {
    return j.max_pinned == 0 || j.pinned_bytes + nbytes <= j.max_pinned;
}

// quotas.default, then the job name's quotas.per_job_overrides entry.
void Daemon::init_job_quotas(Job& j) const {
    j.max_pinned = cfg_.v2_quota_max_pinned_bytes;
    j.max_pageable = cfg_.v2_quota_max_pageable_bytes;
    j.max_nvme = cfg_.v2_quota_max_nvme_bytes;
    j.max_inflight_d2h = cfg_.v2_quota_max_inflight_d2h_bytes;
    j.max_inflight_export = cfg_.v2_quota_max_inflight_export_bytes;
    auto ov = cfg_.v2_job_quota_overrides.find(j.name);
    if (ov == cfg_.v2_job_quota_overrides.end()) return;
    for (const auto& q : ov->second) {
        if (q.first == "max_pinned_bytes") j.max_pinned = q.second;
        else if (q.first == "max_pageable_bytes") j.max_pageable = q.second;
        else if (q.first == "max_nvme_bytes") j.max_nvme = q.second;
        else if (q.first == "max_inflight_d2h_bytes") j.max_inflight_d2h = q.second;
        else if (q.first == "max_inflight_export_bytes") j.max_inflight_export = q.second;
    }
}

RegisterJobResponse Daemon::on_register_job(const RegisterJobRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    RegisterJobResponse resp;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    uint64_t job_id = r.scheduler_job_id;
    if (job_id == 0) {
        // Stable id from (tenant, name): the low half of the two-stream FNV
        // hash of "<tenant>/<name>", the derivation StateSpectre uses.
        std::string s = std::to_string(r.tenant_id) + "/" + r.job_name;
        uint64_t lo, hi;
        fnv2_hash(s.data(), s.size(), &lo, &hi);
        job_id = lo ? lo : 1;
    }
    // Every rank of one live job joins the same namespace (same epoch).
    for (auto& kv : jobs_) {
        const Job& j = kv.second;
        if (j.uid.tenant_id == r.tenant_id && j.uid.job_id == job_id && j.state != JobState::kTerminated) {
            resp.ok = true;
            resp.message = "ok (joined existing job)";
            resp.job = JobKeyWire{j.uid.tenant_id, j.uid.job_id, j.uid.launch_epoch, j.name};
            resp.control_generation = header_->generation;
            return resp;
        }
    }
    Job j;
    j.uid = JobUID{r.tenant_id, job_id, cfg_.v2_include_launch_epoch ? next_launch_epoch_++ : 1};
    j.name = r.job_name;
    j.created_ns = real_ns();
    init_job_quotas(j);
    for (size_t i = 0; i < r.label_keys.size() && i < r.label_values.size(); ++i)
        j.labels.emplace_back(r.label_keys[i], r.label_values[i]);
    jobs_[j.uid] = j;
    Metrics::get().inc(M::kJobsRegistered);
    resp.ok = true;
    resp.message = "ok";
    resp.job = JobKeyWire{j.uid.tenant_id, j.uid.job_id, j.uid.launch_epoch, j.name};
    resp.control_generation = header_->generation;
    LOG_INFO(TAG, "job '%s' tenant=%llu id=%llu epoch=%llu", j.name.c_str(), (unsigned long long)j.uid.tenant_id,
             (unsigned long long)j.uid.job_id, (unsigned long long)j.uid.launch_epoch);
    return resp;
}

RequestCanonicalEvictResponse Daemon::on_canonical_evict(const RequestCanonicalEvictRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    RequestCanonicalEvictResponse resp;
    resp.action = ATTACH_ACTION_ERROR;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    Job* job = find_job(r.key.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    auto mit = manifests_.find(VersionKey{job->uid, r.key.model_role, r.key.model_version});
    if (mit != manifests_.end() && mit->second.state == MANIFEST_SEALED) {
        Metrics::get().inc(M::kCanonicalStaleVersionReject);
        resp.action = ATTACH_ACTION_REJECTED_STALE_VERSION;
        resp.message = "model_version already sealed";
        return resp;
    }
    if (r.key.nbytes == 0) {
        resp.message = "nbytes must be > 0";
        return resp;
    }
    const std::string ks = key_string(r.key, cfg_.v2_cross_job_dedup);
    auto kit = object_by_key_.find(ks);
    CanonicalObject* existing = kit == object_by_key_.end() ? nullptr : find_object(kit->second);
    if (existing && existing->nbytes != r.key.nbytes) {
        resp.message = "nbytes mismatch vs existing object";
        return resp;
    }
    const uint32_t mode = r.dedup_mode;
    const JobUID juid = job->uid;

    // Reserve a pinned run under a synthetic tid (the lock may drop while a
    // forced drain runs, so the job is re-found afterwards).
    auto reserve = [&](uint64_t syn_tid, uint64_t* lease_out, uint32_t* base_out) -> bool {
        Job* j = &jobs_[juid];
        if (!quota_allows_pinned(*j, r.key.nbytes)) {
            Metrics::get().inc(M::kQuotaRejections);
            return false;
        }
        uint32_t base = 0, count = 0;
        if (!allocate(r.gpu_id, r.numa_node, r.key.nbytes, OFLD_FLAG_DESTRUCTIVE, &base, &count, lk)) {
            Metrics::get().inc(M::kBlockedReservations);
            return false;
        }
        if (!epoch_ok(r.rank_id, r.rank_epoch)) {
            free_run(base, count);
            return false;
        }
        uint64_t lid = new_lease(base, count, syn_tid, 1, r.rank_id, r.rank_epoch, r.key.nbytes, false);
        stamp_run(base, count, syn_tid, 1, lid, r.rank_id, leases_[lid].owner_pid, r.rank_epoch, r.key.nbytes,
                  OFLD_FLAG_DESTRUCTIVE, OFLD_SLOT_RESERVED_D2H);
        jobs_[juid].pinned_bytes += r.key.nbytes;
        *lease_out = lid;
        *base_out = base;
        return true;
    };
    auto fill_slot = [&](uint32_t base, uint64_t syn) {
        resp.slot_id = base;
        resp.arena_id = slots_[base].arena_id;
        resp.arena_offset = slots_[base].arena_offset;
        resp.capacity = uint64_t(slots_for(r.key.nbytes)) * cfg_.allocation_granularity_bytes;
        resp.synthetic_tid = syn;
    };
    auto attach = [&](CanonicalObject& o) {
        o.holders.insert(r.rank_id);
        o.last_access_ns = real_ns();
        jobs_[juid].dedup_bytes_saved += r.key.nbytes;
        Metrics::get().inc(M::kCanonicalAttachExisting);
        Metrics::get().add(M::kCanonicalDedupBytesSaved, r.key.nbytes);
    };

    if (existing && readable(existing->state)) {
        if (!r.attach_if_exists) {
            resp.message = "exists but attach disabled";
            return resp;
        }
        if (mode == kDedupP2PVerified) {
            attach(*existing);
            Metrics::get().add(M::kCanonicalD2HBytesAvoided, r.key.nbytes);
            Metrics::get().inc(M::kCanonicalP2PVerified);
            resp.ok = true;
            resp.action = kActionVerifiedByP2P;
            resp.object_id = existing->object_id;
            resp.message = "attached after peer byte compare";
            return resp;
        }
        if (mode == kDedupDeviceHashVerified) {
            resp.ok = true;
            resp.action = kActionVerifyHashOnly;
            resp.object_id = existing->object_id;
            resp.message = "verify by device hash";
            Metrics::get().add(M::kCanonicalD2HBytesAvoided, r.key.nbytes);
            return resp;
        }
        if (mode != DEDUP_HASH_VERIFIED && mode != DEDUP_SAMPLED_HASH) {
            attach(*existing);
            Metrics::get().add(M::kCanonicalD2HBytesAvoided, r.key.nbytes);
            resp.ok = true;
            resp.action = ATTACH_ACTION_ATTACHED_EXISTING;
            resp.object_id = existing->object_id;
            resp.message = "attached existing";
            return resp;
        }
        uint64_t oid = existing->object_id;
        uint64_t cand = kCanonicalTidBit | kCandidateTidBit | next_object_++;
        uint64_t lid;
        uint32_t base;
        if (!reserve(cand, &lid, &base)) {
            resp.action = ATTACH_ACTION_QUOTA_EXCEEDED;
            resp.message = "no capacity for verify candidate";
            return resp;
        }
        resp.ok = true;
        resp.action = ATTACH_ACTION_DUPLICATE_CANDIDATE;
        resp.object_id = oid;
        resp.lease_id = lid;
        fill_slot(base, cand);
        resp.message = "verify candidate (hash)";
        Metrics::get().inc(M::kCanonicalDuplicateCandidate);
        return resp;
    }

    if (existing && existing->state == OBJ_CREATING) {
        bool pressure_hi = pinned_pressure() >= cfg_.v2_duplicate_candidate_gpu_pressure_threshold;
        bool want_dup = r.allow_duplicate_candidate || (cfg_.v2_creating_policy == 1 && pressure_hi);
        if (!want_dup) {
            resp.ok = true;
            resp.action = ATTACH_ACTION_WAIT_FOR_CREATOR;
            resp.object_id = existing->object_id;
            resp.message = "wait for creator";
            Metrics::get().inc(M::kCanonicalAttachWait);
            return resp;
        }
        uint64_t oid = existing->object_id;
        uint64_t cand = kCanonicalTidBit | kCandidateTidBit | next_object_++;
        uint64_t lid;
        uint32_t base;
        if (!reserve(cand, &lid, &base)) {
            resp.action = ATTACH_ACTION_QUOTA_EXCEEDED;
            resp.message = "no capacity for duplicate candidate";
            return resp;
        }
        resp.ok = true;
        resp.action = ATTACH_ACTION_DUPLICATE_CANDIDATE;
        resp.object_id = oid;
        resp.lease_id = lid;
        fill_slot(base, cand);
        resp.message = "duplicate candidate";
        Metrics::get().inc(M::kCanonicalDuplicateCandidate);
        return resp;
    }

    if (!r.create_if_missing) {
        resp.message = "missing and create disabled";
        return resp;
    }
    {
        const Job& j = jobs_[juid];
        if (j.max_inflight_d2h && j.inflight_d2h_bytes + r.key.nbytes > j.max_inflight_d2h) {
            Metrics::get().inc(M::kQuotaRejections);
            resp.action = ATTACH_ACTION_QUOTA_EXCEEDED;
            resp.message = "inflight D2H quota exceeded";
            return resp;
        }
    }
    uint64_t oid = next_object_++;
    uint64_t syn = canonical_tid(oid);
    uint64_t lid;
    uint32_t base;
    if (!reserve(syn, &lid, &base)) {
        resp.action = ATTACH_ACTION_QUOTA_EXCEEDED;
        resp.message = "no pinned capacity / quota";
        return resp;
    }
    // Another rank may have created the key while the lock was dropped.
    auto again = object_by_key_.find(ks);
    if (again != object_by_key_.end()) {
        Lease* L = lease(lid);
        if (L) {
            free_run(L->base, L->count);
            erase_lease(lid);
        }
        jobs_[juid].pinned_bytes -= std::min(jobs_[juid].pinned_bytes, r.key.nbytes);
        resp.ok = true;
        resp.action = ATTACH_ACTION_WAIT_FOR_CREATOR;
        resp.object_id = again->second;
        resp.message = "wait for creator";
        Metrics::get().inc(M::kCanonicalAttachWait);
        return resp;
    }
    CanonicalObject o;
    o.object_id = oid;
    o.key = r.key;
    o.key_str = ks;
    o.nbytes = r.key.nbytes;
    o.state = OBJ_CREATING;
    o.holders.insert(r.rank_id);
    o.producer_rank = r.rank_id;
    o.synthetic_tid = syn;
    o.lease_id = lid;
    o.base_slot = base;
    o.slot_count = slots_for(r.key.nbytes);
    o.created_ns = o.last_access_ns = real_ns();
    o.d2h_counted = true;
    objects_[oid] = o;
    storage_[syn].objects = 1;
    object_by_key_[ks] = oid;
    jobs_[juid].object_count++;
    jobs_[juid].inflight_d2h_bytes += o.nbytes;
    resp.ok = true;
    resp.action = ATTACH_ACTION_NEED_D2H_CREATE;
    resp.object_id = oid;
    resp.lease_id = lid;
    fill_slot(base, syn);
    resp.message = "need d2h create";
    Metrics::get().inc(M::kCanonicalObjectsCreated);
    return resp;
}

CommitCanonicalObjectResponse Daemon::on_commit_canonical(const CommitCanonicalObjectRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    CommitCanonicalObjectResponse resp;
    resp.object_id = r.object_id;
    resp.won = false;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    CanonicalObject* o = find_object(r.object_id);
    if (!o) {
        resp.message = "unknown object";
        return resp;
    }
    // Creator: validated through the location table (a drain may already
    // have recycled the creating lease; the bytes are safe wherever it points).
    if (o->state == OBJ_CREATING && o->lease_id == r.lease_id && r.lease_id != 0) {
        auto lit = locations_.find(o->synthetic_tid);
        if (lit == locations_.end() || lit->second.kind == OFLD_LOC_NONE || lit->second.kind == OFLD_LOC_DELETED) {
            Metrics::get().inc(M::kInvalidTransitionRejected);
            resp.message = "object bytes not yet valid";
            return resp;
        }
        o->hash_lo = r.content_hash_lo;
        o->hash_hi = r.content_hash_hi;
        settle_d2h(*o);
        o->state = lit->second.kind == OFLD_LOC_PAGEABLE ? OBJ_VALID_PAGEABLE
                   : lit->second.kind == OFLD_LOC_NVME   ? OBJ_VALID_NVME
                                                         : OBJ_VALID_PINNED;
        o->last_access_ns = real_ns();
        // The run becomes drainable now that the object is committed.
        if (Lease* L = lease(o->lease_id)) {
            if (state_of(L->base) == OFLD_SLOT_PINNED_VALID) {
                if (cfg_.drain_on_d2h_complete)
                    enqueue_drain(*L);
                else {
                    note_drainable(L->id);
                    pressure_drain();
                }
            }
        }
        resp.ok = true;
        resp.won = true;
        resp.message = "committed";
        return resp;
    }
    // Candidate / verify commit: compare, discard the candidate, attach.
    const bool valid = readable(o->state);
    bool hash_ok = true;
    if (valid && (o->hash_lo | o->hash_hi) && (r.content_hash_lo | r.content_hash_hi))
        hash_ok = o->hash_lo == r.content_hash_lo && o->hash_hi == r.content_hash_hi;
    if (valid && r.lease_id == 0 && !(r.content_hash_lo | r.content_hash_hi)) hash_ok = false;  // verify needs a hash
    Job* job = find_job(o->key.job);
    if (r.lease_id != 0) {
        Lease* L = lease(r.lease_id);
        if (L && L->owner_rank == r.rank_id && is_candidate_tid(L->tensor_id)) {
            uint32_t st = state_of(L->base);
            if (st == OFLD_SLOT_PINNED_VALID || st == OFLD_SLOT_RESERVED_D2H || st == OFLD_SLOT_D2H_IN_FLIGHT)
                free_run(L->base, L->count);
            locations_.erase(L->tensor_id);
            erase_lease(r.lease_id);
            if (job) job->pinned_bytes -= std::min(job->pinned_bytes, o->nbytes);
        }
    }
    if (!valid) {
        resp.message = "canonical object not valid for attach";
        return resp;
    }
    if (!hash_ok) {
        Metrics::get().inc(M::kCanonicalHashMismatch);
        Metrics::get().inc(M::kChecksumMismatch);
        resp.message = "content hash mismatch (corrupt replica)";
        return resp;
    }
    o->holders.insert(r.rank_id);
    o->last_access_ns = real_ns();
    if (job) job->dedup_bytes_saved += o->nbytes;
    Metrics::get().inc(M::kCanonicalAttachExisting);
    Metrics::get().add(M::kCanonicalDedupBytesSaved, o->nbytes);
    resp.ok = true;
    resp.message = "attached after verify";
    return resp;
}

// Free an object's backing and table entry unless a transfer is in flight.
// Ignores holders (callers decide). mu_ held.
void Daemon::storage_io(uint64_t tid, int delta) {
    auto it = storage_.find(tid);
    if (it == storage_.end()) return;
    if (delta > 0) it->second.io += uint32_t(delta);
    else it->second.io -= std::min(it->second.io, uint32_t(-delta));
}

bool Daemon::storage_busy(uint64_t tid) const {
    auto it = storage_.find(tid);
    return it != storage_.end() && it->second.io > 0;
}

void Daemon::settle_d2h(CanonicalObject& o) {
    if (!o.d2h_counted) return;
    o.d2h_counted = false;
    if (Job* j = find_job(o.key.job)) j->inflight_d2h_bytes -= std::min(j->inflight_d2h_bytes, o.nbytes);
}

bool Daemon::release_object(CanonicalObject& o) {
    if (o.export_refs || o.restore_refs) return false;
    settle_d2h(o);
    const uint64_t oid = o.object_id, nbytes = o.nbytes;
    // Storage shared with carried-forward objects stays until its last user goes.
    auto sit = storage_.find(o.synthetic_tid);
    if (sit != storage_.end() && sit->second.objects > 1) {
        sit->second.objects--;
        auto kit = object_by_key_.find(o.key_str);
        if (kit != object_by_key_.end() && kit->second == oid) object_by_key_.erase(kit);
        if (Job* j = find_job(o.key.job))
            if (j->object_count) j->object_count--;
        Metrics::get().inc(M::kCanonicalObjectsDropped);
        objects_.erase(oid);
        return true;
    }
    if (sit != storage_.end()) storage_.erase(sit);
    forget_persisted_storage(o.synthetic_tid);  // the last object of a durable storage
    auto lit = locations_.find(o.synthetic_tid);
    // pinned bytes were counted at reservation and leave the count at a drain
    const bool counted_pinned = lit != locations_.end() ? lit->second.kind == OFLD_LOC_PINNED
                                                         : (o.state == OBJ_CREATING || o.state == OBJ_ERROR);
    if (lit != locations_.end()) {
        if (Job* j = find_job(o.key.job)) {  // the job's tier accounting follows the bytes out
            auto cit = lit->second.cold_ref ? cold_.find(lit->second.cold_ref) : cold_.end();
            if (cit != cold_.end() && !cit->second.persisted)
                (cit->second.kind == OFLD_LOC_NVME ? j->nvme_bytes : j->pageable_bytes) -=
                    std::min(cit->second.kind == OFLD_LOC_NVME ? j->nvme_bytes : j->pageable_bytes, nbytes);
        }
        if (lit->second.kind == OFLD_LOC_PINNED) {
            uint32_t s = lit->second.slot;
            uint32_t st = state_of(s);
            if (st == OFLD_SLOT_PINNED_VALID || st == OFLD_SLOT_RESERVED_D2H || st == OFLD_SLOT_ERROR) {
                uint64_t lid = slots_[s].lease_id;
                free_run(s, slots_for(nbytes));
                erase_lease(lid);
            }
        }
        if (lit->second.cold_ref) free_cold(lit->second.cold_ref);
        locations_.erase(lit);
    } else if (o.state == OBJ_CREATING || o.state == OBJ_ERROR) {
        if (Lease* L = lease(o.lease_id)) {
            free_run(L->base, L->count);
            erase_lease(o.lease_id);
        }
    }
    erase_lease(o.lease_id);
    auto kit = object_by_key_.find(o.key_str);
    if (kit != object_by_key_.end() && kit->second == oid) object_by_key_.erase(kit);
    if (Job* j = find_job(o.key.job)) {
        if (counted_pinned) j->pinned_bytes -= std::min(j->pinned_bytes, nbytes);
        if (j->object_count) j->object_count--;
    }
    Metrics::get().inc(M::kCanonicalObjectsDropped);
    objects_.erase(oid);
    return true;
}

bool Daemon::maybe_free_object(CanonicalObject& o) {
    if (!o.holders.empty() || o.export_refs || o.restore_refs) return false;
    return release_object(o);
}

void Daemon::purge_rank_holds(uint32_t rank) {
    std::vector<uint64_t> touched;
    for (auto& kv : objects_)
        if (kv.second.holders.erase(rank)) touched.push_back(kv.first);
    for (uint64_t oid : touched)
        if (CanonicalObject* o = find_object(oid)) maybe_free_object(*o);
}

CarryForwardResponse Daemon::on_carry_forward(const CarryForwardRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    CarryForwardResponse resp;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    if (r.to_version == r.from_version) {
        resp.message = "from_version == to_version";
        return resp;
    }
    auto mit = manifests_.find(VersionKey{job->uid, r.model_role, r.to_version});
    if (mit != manifests_.end() && mit->second.state == MANIFEST_SEALED) {
        resp.message = "target version already sealed";
        return resp;
    }
    // param_id -> objects at from_version, one per partition (TP/PP/EP
    // shards of one parameter share its param_id)
    std::unordered_map<uint64_t, std::vector<uint64_t>> by_param;
    for (uint64_t oid : objects_of_version(job->uid, r.model_role, r.from_version)) {
        const CanonicalObject& o = objects_[oid];
        if (!readable(o.state)) continue;
        if (r.shard && (o.key.pp_rank != r.pp_rank || o.key.tp_rank != r.tp_rank || o.key.ep_rank != r.ep_rank ||
                        o.key.etp_rank != r.etp_rank || o.key.expert_id != r.expert_id))
            continue;
        by_param[o.key.param_id].push_back(oid);
    }
    std::vector<uint64_t> want = r.param_ids;
    if (want.empty())
        for (auto& kv : by_param) want.push_back(kv.first);
    std::vector<uint64_t> sources;
    for (uint64_t pid : want) {
        auto bit = by_param.find(pid);
        if (bit == by_param.end()) {
            resp.missing_count++;
            continue;
        }
        sources.insert(sources.end(), bit->second.begin(), bit->second.end());
    }
    for (uint64_t src_oid : sources) {
        const CanonicalObject src = objects_[src_oid];
        CanonicalTensorKeyWire key = src.key;
        key.model_version = r.to_version;
        const std::string ks = key_string(key, cfg_.v2_cross_job_dedup);
        if (object_by_key_.count(ks)) {
            resp.existing_count++;
            continue;
        }
        CanonicalObject o;
        o.object_id = next_object_++;
        o.key = key;
        o.key_str = ks;
        o.nbytes = src.nbytes;
        // The new object is a committed member of its version; where its bytes
        // live is read from the shared storage's location entry.
        o.state = src.state == OBJ_SEALED || src.state == OBJ_EXPORT_IN_FLIGHT ? OBJ_VALID_MULTI_TIER : src.state;
        o.holders.insert(r.rank_id);
        o.producer_rank = src.producer_rank;
        o.hash_lo = src.hash_lo;
        o.hash_hi = src.hash_hi;
        o.synthetic_tid = src.synthetic_tid;
        o.slot_count = src.slot_count;
        o.created_ns = o.last_access_ns = real_ns();
        storage_[src.synthetic_tid].objects++;
        object_by_key_[ks] = o.object_id;
        objects_[o.object_id] = o;
        job->object_count++;
        job->dedup_bytes_saved += src.nbytes;
        resp.carried_count++;
        resp.bytes_shared += src.nbytes;
    }
    Metrics::get().add(M::kCanonicalDedupBytesSaved, resp.bytes_shared);
    resp.ok = true;
    resp.message = "ok";
    return resp;
}

ReleaseCanonicalResponse Daemon::on_release_canonical(const ReleaseCanonicalRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    ReleaseCanonicalResponse resp;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        resp.message = "epoch invalid";
        return resp;
    }
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    std::vector<uint64_t> ids = r.object_id ? std::vector<uint64_t>{r.object_id}
                                            : objects_of_version(job->uid, r.model_role, r.model_version);
    for (uint64_t oid : ids) {
        CanonicalObject* o = find_object(oid);
        if (!o || !o->holders.erase(r.rank_id)) continue;
        resp.released_count++;
        uint64_t nb = o->nbytes;
        if (maybe_free_object(*o)) {
            resp.freed_count++;
            resp.bytes_freed += nb;
        }
    }
    resp.ok = true;
    resp.message = "ok";
    return resp;
}

}  // namespace ofld
