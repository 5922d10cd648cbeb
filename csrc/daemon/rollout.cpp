// Sealed manifests, rollout pull/export, local canonical restore and version GC.
//
// Sealing, promotion, manifest filters, the pull invariants (sealed version,
// sealed member object, export hold while bytes move) and retention follow
// StateSpectre (reference: src/daemon/canonical_rollout.cpp:41-649). The
// manifest hash mixes (object_id, hash_lo, hash_hi, nbytes) of the members in
// object-id order with the same two-stream function, so a manifest sealed here
// is identical to one sealed there from the same objects.
//
// Export differs by design: bytes stream to the transport in export.chunk_mb
// pieces straight from the pinned slot, the pageable buffer or the NVMe
// extents. Nothing is staged in a full-size heap copy, and a cold read never
// touches an unrelated slot (StateSpectre's staging path wrote cold bytes into
// slot 0, reference: canonical_rollout.cpp:266).
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <memory>

#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"
#include "ofld/transport.h"

namespace ofld {

namespace {
constexpr const char* TAG = "rollout";
constexpr uint32_t kExportMagic = 0x4F464558u;  // "OFEX"

bool readable(CanonicalObjectState s) {
    return s == OBJ_VALID_PINNED || s == OBJ_VALID_PAGEABLE || s == OBJ_VALID_NVME || s == OBJ_VALID_MULTI_TIER ||
           s == OBJ_SEALED || s == OBJ_EXPORT_IN_FLIGHT;
}

const char* loc_hint(ofld_location_kind_t k) {
    switch (k) {
        case OFLD_LOC_PINNED: return "pinned";
        case OFLD_LOC_PAGEABLE: return "pageable";
        case OFLD_LOC_NVME: return "nvme";
        case OFLD_LOC_GPU: return "gpu";
        default: return "none";
    }
}

// 40-byte self-describing export header: magic, version, object id, byte
// count, content hash. Receivers (RolloutWeightClient) frame the payload by it.
void export_header(uint8_t out[40], uint64_t oid, uint64_t nbytes, uint64_t hlo, uint64_t hhi) {
    uint32_t magic = kExportMagic, ver = 1;
    std::memcpy(out, &magic, 4);
    std::memcpy(out + 4, &ver, 4);
    std::memcpy(out + 8, &oid, 8);
    std::memcpy(out + 16, &nbytes, 8);
    std::memcpy(out + 24, &hlo, 8);
    std::memcpy(out + 32, &hhi, 8);
}

struct Sink {
    virtual ~Sink() = default;
    virtual bool write(const void* p, size_t n) = 0;
    std::string metadata;
};

struct FdSink : Sink {
    int fd = -1;
    ~FdSink() override { close_fd(fd); }
    bool write(const void* p, size_t n) override { return write_all(fd, p, n); }
};

// Open the transport for one export. Returns null with *err set on failure.
std::unique_ptr<Sink> open_sink(uint32_t transport, const std::string& target, uint32_t* used, std::string* err) {
    auto s = std::make_unique<FdSink>();
    if (transport == TRANSPORT_TCP) {
        std::string host;
        uint16_t port = 0;
        if (!split_host_port(target, &host, &port)) {
            *err = "bad tcp target (want host:port)";
            return nullptr;
        }
        try {
            s->fd = tcp_connect(host, port, 5000);
        } catch (const std::exception& e) {
            *err = std::string("tcp connect failed: ") + e.what();
            return nullptr;
        }
        s->metadata = "tcp:" + target;
    } else if (transport == TRANSPORT_FILE) {
        s->fd = ::open(target.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (s->fd < 0) {
            *err = std::string("open failed: ") + std::strerror(errno);
            return nullptr;
        }
        s->metadata = "file:" + target;
    } else {
        *err = "unknown transport";
        return nullptr;
    }
    *used = transport;
    return s;
}
}  // namespace

std::vector<uint64_t> Daemon::objects_of_version(const JobUID& j, uint32_t role, uint64_t ver) {
    std::vector<uint64_t> ids;
    for (auto& kv : objects_) {
        const CanonicalTensorKeyWire& k = kv.second.key;
        if (k.job.tenant_id == j.tenant_id && k.job.job_id == j.job_id && k.job.launch_epoch == j.launch_epoch &&
            k.model_role == role && k.model_version == ver)
            ids.push_back(kv.first);
    }
    std::sort(ids.begin(), ids.end());
    return ids;
}

SealModelVersionResponse Daemon::on_seal(const SealModelVersionRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    SealModelVersionResponse resp;
    resp.state = MANIFEST_ERROR;
    if (!cfg_.v2_enable_canonical_store || !cfg_.v2_enable_manifests) {
        resp.message = "manifests disabled";
        return resp;
    }
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    VersionKey vk{job->uid, r.model_role, r.model_version};
    auto mit = manifests_.find(vk);
    if (mit != manifests_.end() && mit->second.state == MANIFEST_SEALED) {
        resp.ok = true;
        resp.state = MANIFEST_SEALED;
        resp.tensor_count = mit->second.object_ids.size();
        resp.total_nbytes = mit->second.total_nbytes;
        resp.manifest_hash_lo = mit->second.hash_lo;
        resp.manifest_hash_hi = mit->second.hash_hi;
        resp.message = "already sealed";
        // Promotion of an already sealed version still moves the pointer.
        if (r.promote) latest_sealed_[{job->uid, r.model_role}] = r.model_version;
        return resp;
    }
    Manifest man;
    man.vk = vk;
    man.created_ns = real_ns();
    bool any_invalid = false;
    for (uint64_t oid : objects_of_version(job->uid, r.model_role, r.model_version)) {
        CanonicalObject& o = objects_[oid];
        if (!readable(o.state)) {
            any_invalid = true;
            continue;
        }
        man.object_ids.push_back(oid);
        man.total_nbytes += o.nbytes;
    }
    for (uint64_t pid : r.expected_param_ids) {
        bool found = false;
        for (uint64_t oid : man.object_ids) found |= objects_[oid].key.param_id == pid;
        if (!found) {
            any_invalid = true;
            break;
        }
    }
    if (cfg_.v2_seal_requires_all_objects_valid && r.fail_if_missing && any_invalid) {
        man.state = MANIFEST_ERROR;
        manifests_[vk] = man;
        Metrics::get().inc(M::kManifestSealFailed);
        resp.message = "seal failed: required objects missing/invalid";
        return resp;
    }
    uint64_t lo = 1469598103934665603ull, hi = 1099511628211ull;
    auto mix = [&](uint64_t v) {
        lo = (lo ^ v) * 1099511628211ull;
        hi = (hi ^ (v + 0x9e3779b97f4a7c15ull)) * 1099511628211ull;
    };
    for (uint64_t oid : man.object_ids) {  // ascending object id
        CanonicalObject& o = objects_[oid];
        mix(oid);
        mix(o.hash_lo);
        mix(o.hash_hi);
        mix(o.nbytes);
        o.state = OBJ_SEALED;
        o.sealed_ns = real_ns();
    }
    man.hash_lo = lo;
    man.hash_hi = hi;
    man.state = MANIFEST_SEALED;
    man.sealed_ns = real_ns();
    manifests_[vk] = man;
    Metrics::get().inc(M::kManifestSealed);
    if (r.promote) {
        latest_sealed_[{job->uid, r.model_role}] = r.model_version;
        enforce_retention(job->uid, r.model_role);
    }
    enqueue_persist(vk);
    resp.ok = true;
    resp.state = MANIFEST_SEALED;
    resp.tensor_count = man.object_ids.size();
    resp.total_nbytes = man.total_nbytes;
    resp.manifest_hash_lo = lo;
    resp.manifest_hash_hi = hi;
    resp.message = "sealed";
    LOG_INFO(TAG, "sealed job=%llu role=%u version=%llu tensors=%zu", (unsigned long long)vk.job.job_id,
             r.model_role, (unsigned long long)r.model_version, man.object_ids.size());
    return resp;
}

GetLatestSealedVersionResponse Daemon::on_get_latest(const GetLatestSealedVersionRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    GetLatestSealedVersionResponse resp;
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    resp.ok = true;
    auto it = latest_sealed_.find({job->uid, r.model_role});
    if (it == latest_sealed_.end()) {
        resp.message = "no sealed version promoted";
    } else {
        resp.found = true;
        resp.model_version = it->second;
        resp.message = "ok";
    }
    return resp;
}

GetManifestResponse Daemon::on_get_manifest(const GetManifestRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    GetManifestResponse resp;
    resp.state = MANIFEST_ERROR;
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    resp.job = r.job;
    resp.model_role = r.model_role;
    resp.model_version = r.model_version;
    auto it = manifests_.find(VersionKey{job->uid, r.model_role, r.model_version});
    if (it == manifests_.end() || it->second.state != MANIFEST_SEALED) {
        Metrics::get().inc(M::kRolloutStaleManifestReject);
        resp.message = "no sealed manifest for version";
        return resp;
    }
    resp.state = it->second.state;
    const ManifestFilterWire& f = r.filter;
    for (uint64_t oid : it->second.object_ids) {
        CanonicalObject* o = find_object(oid);
        if (!o) continue;
        const CanonicalTensorKeyWire& k = o->key;
        if ((f.pp_present && k.pp_rank != f.pp_rank) || (f.tp_present && k.tp_rank != f.tp_rank) ||
            (f.ep_present && k.ep_rank != f.ep_rank) || (f.etp_present && k.etp_rank != f.etp_rank) ||
            (f.expert_present && k.expert_id != f.expert_id))
            continue;
        TensorManifestEntryWire e;
        e.key = k;
        e.object_id = oid;
        e.nbytes = o->nbytes;
        e.content_hash_lo = o->hash_lo;
        e.content_hash_hi = o->hash_hi;
        auto lit = locations_.find(o->synthetic_tid);
        e.location_hint = loc_hint(lit == locations_.end() ? OFLD_LOC_NONE : lit->second.kind);
        resp.tensors.push_back(std::move(e));
    }
    resp.ok = true;
    resp.message = "ok";
    Metrics::get().inc(M::kRolloutGetManifest);
    return resp;
}

PullTensorResponse Daemon::on_pull_tensor(const PullTensorRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    PullTensorResponse resp;
    resp.object_id = r.object_id;
    resp.transport = r.transport;
    if (!cfg_.v2_enable_canonical_store || !cfg_.v2_enable_rollout_export) {
        resp.message = "rollout export disabled";
        return resp;
    }
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    const JobUID juid = job->uid;
    auto mit = manifests_.find(VersionKey{juid, r.model_role, r.model_version});
    if (mit == manifests_.end() || mit->second.state != MANIFEST_SEALED) {
        Metrics::get().inc(M::kRolloutStaleManifestReject);
        resp.message = "version not sealed; refusing pull";
        return resp;
    }
    CanonicalObject* o = find_object(r.object_id);
    if (!o) {
        resp.message = "unknown object";
        return resp;
    }
    if (o->state != OBJ_SEALED && o->state != OBJ_EXPORT_IN_FLIGHT) {
        resp.message = "object not sealed";
        return resp;
    }
    const auto& ids = mit->second.object_ids;
    if (!std::binary_search(ids.begin(), ids.end(), r.object_id)) {
        resp.message = "object not in manifest";
        return resp;
    }
    const uint64_t nbytes = o->nbytes;
    if (job->max_inflight_export && job->inflight_export_bytes + nbytes > job->max_inflight_export) {
        Metrics::get().inc(M::kQuotaRejections);
        resp.message = "export inflight quota exceeded";
        return resp;
    }
    if (cfg_.v2_max_concurrent_exports_per_job && job->exports_in_flight >= cfg_.v2_max_concurrent_exports_per_job) {
        Metrics::get().inc(M::kQuotaRejections);
        resp.message = "too many concurrent exports for job";
        return resp;
    }
    // Resolve the source and take the read hold before dropping the lock.
    ReadSrc src;
    std::string why;
    if (!begin_read(*o, &src, &why)) {
        resp.message = why;
        return resp;
    }
    job->inflight_export_bytes += nbytes;
    job->exports_in_flight++;
    Metrics::get().add(M::kExportInflightBytes, nbytes);
    Metrics::get().inc(src.kind == OFLD_LOC_PINNED     ? M::kExportFromPinned
                       : src.kind == OFLD_LOC_PAGEABLE ? M::kExportFromPageable
                                                       : M::kExportFromNvme);
    const uint64_t hlo = o->hash_lo, hhi = o->hash_hi;
    // whole 128 KiB blocks, so a coded object's pieces decode on their own
    const uint64_t chunk = (std::max<uint64_t>(cfg_.v2_export_chunk_bytes, 1 << 20) + (128u << 10) - 1) &
                           ~uint64_t((128u << 10) - 1);
    uint32_t transport = r.transport;
    if (transport == TRANSPORT_LIBFABRIC_SEND || transport == TRANSPORT_RDMA_READ ||
        transport == TRANSPORT_RDMA_WRITE) {
        LOG_WARN(TAG, "libfabric transport not built in; using fallback transport %u", cfg_.v2_fallback_transport);
        transport = cfg_.v2_fallback_transport;
    }
    lk.unlock();

    // ---- stream without the lock ----
    std::string err;
    uint32_t used = transport;
    bool ok = false;
    std::unique_ptr<Sink> sink = open_sink(transport, r.target_descriptor, &used, &err);
    if (sink) {
        uint8_t hdr[40];
        export_header(hdr, r.object_id, nbytes, hlo, hhi);
        ok = sink->write(hdr, sizeof(hdr));
        std::vector<char> bounce, plain;
        for (uint64_t off = 0; ok && off < nbytes; off += chunk) {
            uint64_t n = std::min(chunk, nbytes - off);
            const char* stored = nullptr;  // the stored bytes of [off, off + n)
            if (src.pinned) {
                stored = src.pinned + off;
            } else if (src.kind == OFLD_LOC_PAGEABLE) {
                stored = src.cold.pageable + off;
            } else {
                bounce.resize(n);
                if (!read_cold(src.cold, bounce.data(), off, n)) {
                    ok = false;
                    err = "cold read failed";
                    break;
                }
                stored = bounce.data();
            }
            if (src.fmt) {
                // a coded run (zbf16 / zf32 canonical object): receivers get the raw bytes
                plain.resize(n);
                if (!decode_out(src, stored, off, n, plain.data())) {
                    ok = false;
                    err = "coded object failed to decode";
                    break;
                }
                stored = plain.data();
                Metrics::get().add(M::kExportDecodedBytes, n);
            }
            ok = sink->write(stored, n);
            if (!ok && err.empty()) err = "transport write failed";
        }
        Metrics::get().add(M::kExportStagingBytes, 0);
    }

    lk.lock();
    if (Job* j2 = find_job(r.job)) {
        j2->inflight_export_bytes -= std::min(j2->inflight_export_bytes, nbytes);
        if (j2->exports_in_flight) j2->exports_in_flight--;
    }
    Metrics::get().sub(M::kExportInflightBytes, nbytes);
    end_read(r.object_id, src);
    if (!ok) {
        Metrics::get().inc(M::kExportTransportErrors);
        resp.message = "transport failed: " + err;
        return resp;
    }
    Metrics::get().inc(M::kRolloutPullTensor);
    Metrics::get().add(M::kRolloutPullBytes, nbytes);
    resp.ok = true;
    resp.message = "ok";
    resp.nbytes = nbytes;
    resp.transport = used;
    resp.content_hash_lo = hlo;
    resp.content_hash_hi = hhi;
    resp.transport_metadata = sink ? sink->metadata : "";
    return resp;
}

RequestCanonicalRestoreResponse Daemon::on_canonical_restore(const RequestCanonicalRestoreRequest& r) {
    std::unique_lock<std::mutex> lk(mu_);
    RequestCanonicalRestoreResponse resp;
    resp.object_id = r.object_id;
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
    if (!readable(o->state)) {
        resp.message = "object not readable";
        return resp;
    }
    const uint64_t syn = o->synthetic_tid, nbytes = o->nbytes;
    auto lit = locations_.find(syn);
    if (lit == locations_.end() || lit->second.kind == OFLD_LOC_NONE || lit->second.kind == OFLD_LOC_DELETED) {
        resp.message = "object not resident";
        return resp;
    }
    uint32_t base = 0xFFFFFFFFu;
    if (lit->second.kind == OFLD_LOC_PINNED && state_of(lit->second.slot) == OFLD_SLOT_PINNED_VALID) {
        base = lit->second.slot;
    } else if (lit->second.kind == OFLD_LOC_PAGEABLE || lit->second.kind == OFLD_LOC_NVME) {
        uint64_t cref = lit->second.cold_ref;
        ColdEntry cold;
        if (!cref || !pin_cold(cref, &cold)) {
            resp.retriable = true;
            resp.message = "object cold reference not ready";
            return resp;
        }
        uint32_t count = 0;
        if (!allocate(r.gpu_id, r.numa_node, nbytes, OFLD_FLAG_ALLOW_OVERFLOW | OFLD_FLAG_ALLOW_REMOTE_NUMA, &base,
                      &count, lk)) {
            unpin_cold(cref);
            // busy pinned runs free up as other transfers finish: the caller retries
            resp.retriable = true;
            resp.message = "no pinned capacity to warm object";
            return resp;
        }
        o = find_object(r.object_id);
        if (!o) {
            free_run(base, count);
            unpin_cold(cref);
            resp.message = "object dropped while warming";
            return resp;
        }
        uint64_t lid = new_lease(base, count, syn, 1, r.rank_id, r.rank_epoch, nbytes, false);
        stamp_run(base, count, syn, 1, lid, r.rank_id, leases_[lid].owner_pid, r.rank_epoch, nbytes, 0,
                  OFLD_SLOT_READBACK_IN_FLIGHT);
        o->restore_refs++;  // hold across the unlocked read
        char* dst = slot_ptr(base);
        lk.unlock();
        bool ok = read_cold(cold, dst, 0, nbytes);
        lk.lock();
        unpin_cold(cref);
        o = find_object(r.object_id);
        if (o) o->restore_refs--;
        if (!ok || !o) {
            free_run(base, count);
            erase_lease(lid);
            Metrics::get().inc(M::kIoFailure);
            resp.message = "readback failed";
            return resp;
        }
        set_run_state(base, count, OFLD_SLOT_PINNED_VALID);
        set_cold_ref(base, count, cref);
        Location& loc = locations_[syn];
        loc.kind = OFLD_LOC_PINNED;
        loc.slot = base;
        loc.nbytes = nbytes;
        loc.cold_ref = cref;  // multi-tier: the cold copy is kept
        o->base_slot = base;
        o->slot_count = count;
        o->lease_id = lid;
        if (o->state != OBJ_SEALED && o->state != OBJ_EXPORT_IN_FLIGHT) o->state = OBJ_VALID_MULTI_TIER;
        note_drainable(lid);
    } else {
        resp.retriable = true;
        resp.message = "object transitioning between tiers";
        return resp;
    }
    o->restore_refs++;
    storage_io(o->synthetic_tid, +1);
    o->last_access_ns = real_ns();
    Metrics::get().inc(M::kCanonicalRestoreServed);
    resp.ok = true;
    resp.message = "ok";
    resp.nbytes = nbytes;
    resp.arena_id = slots_[base].arena_id;
    resp.arena_offset = slots_[base].arena_offset;
    return resp;
}

StatusResponse Daemon::on_release_canonical_restore(const ReleaseCanonicalRestoreRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    if (!epoch_ok(r.rank_id, r.rank_epoch)) {
        Metrics::get().inc(M::kEpochMismatchRejected);
        return {false, "epoch invalid"};
    }
    if (CanonicalObject* o = find_object(r.object_id)) {
        if (o->restore_refs) {
            o->restore_refs--;
            storage_io(o->synthetic_tid, -1);
        }
        maybe_free_object(*o);
    }
    return {true, "ok"};
}

DropCanonicalVersionResponse Daemon::on_drop_version(const DropCanonicalVersionRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    DropCanonicalVersionResponse resp;
    if (!cfg_.v2_enable_canonical_store) {
        resp.message = "canonical store disabled";
        return resp;
    }
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    const JobUID uid = job->uid;
    for (uint64_t oid : objects_of_version(uid, r.model_role, r.model_version)) {
        CanonicalObject* o = find_object(oid);
        if (!o) continue;
        uint64_t nb = o->nbytes;
        if (release_object(*o)) {
            resp.dropped_count++;
            resp.bytes_freed += nb;
        } else {
            resp.skipped_inflight++;
        }
    }
    manifests_.erase(VersionKey{uid, r.model_role, r.model_version});
    unlink_persisted_manifest(VersionKey{uid, r.model_role, r.model_version});
    auto lit = latest_sealed_.find({uid, r.model_role});
    if (lit != latest_sealed_.end() && lit->second == r.model_version) latest_sealed_.erase(lit);
    resp.ok = true;
    resp.message = "ok";
    return resp;
}

void Daemon::enforce_retention(const JobUID& uid, uint32_t role) {
    const uint32_t keep = cfg_.v2_retain_sealed_versions;
    if (keep == 0) return;
    std::vector<uint64_t> sealed;
    for (auto& kv : manifests_)
        if (kv.first.job == uid && kv.first.role == role && kv.second.state == MANIFEST_SEALED)
            sealed.push_back(kv.first.version);
    if (sealed.size() <= keep) return;
    std::sort(sealed.begin(), sealed.end(), std::greater<uint64_t>());
    uint64_t latest = 0;
    auto lit = latest_sealed_.find({uid, role});
    if (lit != latest_sealed_.end()) latest = lit->second;
    for (size_t i = keep; i < sealed.size(); ++i) {
        if (sealed[i] == latest) continue;
        bool all = true;
        for (uint64_t oid : objects_of_version(uid, role, sealed[i])) {
            CanonicalObject* o = find_object(oid);
            if (o && !release_object(*o)) all = false;
        }
        if (all) {
            manifests_.erase(VersionKey{uid, role, sealed[i]});
            unlink_persisted_manifest(VersionKey{uid, role, sealed[i]});
        }
    }
}

ExportManifestResponse Daemon::on_export_manifest(const ExportManifestRequest& r) {
    std::lock_guard<std::mutex> g(mu_);
    ExportManifestResponse resp;
    Job* job = find_job(r.job);
    if (!job) {
        resp.message = "job not registered";
        return resp;
    }
    auto it = manifests_.find(VersionKey{job->uid, r.model_role, r.model_version});
    if (it == manifests_.end() || it->second.state != MANIFEST_SEALED) {
        resp.message = "no sealed manifest for version";
        return resp;
    }
    const Manifest& m = it->second;
    ManifestHeaderEntry h;
    std::memset(&h, 0, sizeof(h));
    h.tenant_id = job->uid.tenant_id;
    h.job_id = job->uid.job_id;
    h.launch_epoch = job->uid.launch_epoch;
    h.model_role = r.model_role;
    h.state = m.state;
    h.model_version = r.model_version;
    h.num_tensors = m.object_ids.size();
    h.total_nbytes = m.total_nbytes;
    h.created_ns = m.created_ns;
    h.sealed_ns = m.sealed_ns;
    h.manifest_hash_lo = m.hash_lo;
    h.manifest_hash_hi = m.hash_hi;
    int fd = ::open(r.path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
    if (fd < 0) {
        resp.message = std::string("open failed: ") + std::strerror(errno);
        return resp;
    }
    bool ok = write_all(fd, &h, sizeof(h));
    uint64_t written = sizeof(h);
    for (uint64_t oid : m.object_ids) {
        CanonicalObject* o = find_object(oid);
        if (!o) continue;
        TensorManifestEntryAbi e;
        std::memset(&e, 0, sizeof(e));
        e.object_id = oid;
        const CanonicalTensorKeyWire& k = o->key;
        e.key.tenant_id = k.job.tenant_id;
        e.key.job_id = k.job.job_id;
        e.key.launch_epoch = k.job.launch_epoch;
        e.key.model_role = k.model_role;
        e.key.dtype = k.dtype;
        e.key.model_version = k.model_version;
        e.key.param_id = k.param_id;
        e.key.param_fqn_hash = k.param_fqn_hash;
        e.key.layout = k.layout;
        e.key.nbytes = k.nbytes;
        e.key.shape_hash = k.shape_hash;
        e.key.stride_hash = k.stride_hash;
        e.key.pp_rank = k.pp_rank;
        e.key.tp_rank = k.tp_rank;
        e.key.ep_rank = k.ep_rank;
        e.key.etp_rank = k.etp_rank;
        e.key.expert_id = k.expert_id;
        e.key.shard_offset = k.shard_offset;
        e.key.shard_nbytes = k.shard_nbytes;
        e.content_hash_lo = o->hash_lo;
        e.content_hash_hi = o->hash_hi;
        auto lit = locations_.find(o->synthetic_tid);
        e.location_hint_kind = lit == locations_.end() ? OFLD_LOC_NONE : lit->second.kind;
        ok = ok && write_all(fd, &e, sizeof(e));
        written += sizeof(e);
        resp.tensor_count++;
    }
    ::close(fd);
    resp.ok = ok;
    resp.message = ok ? "ok" : "write failed";
    resp.bytes_written = written;
    return resp;
}

}  // namespace ofld
