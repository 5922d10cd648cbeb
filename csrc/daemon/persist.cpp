// Read holds on canonical objects, and durable sealed versions.
//
// StateSpectre keeps every table on the daemon's heap and its NVMe stripes are
// not self-describing, so a daemon restart loses every sealed version
// (reference: src/daemon/daemon.cpp:277-293, src/daemon/daemon.h:120-128).
// With manifest.persist_dir set, a worker writes each sealed version to disk:
//
//   <dir>/j<tenant>_<job_id>_<launch_epoch>/job.rec   the job key (wire codec)
//   <dir>/j.../s<storage id>.obj                      one file per storage:
//        64-byte header (magic "OFPS", storage id, size, content hash), the
//        bytes from offset 4096, the file padded to 4 KiB
//   <dir>/j.../m<role>_<version>.man                  the version: manifest
//        hashes, promotion, and every object (id, key, size, hash, storage)
//
// Carried-forward objects share their storage, so a version that changed 10 %
// of its tensors writes 10 % of the bytes. Files are written to a temporary
// name, synced and renamed, and a version's manifest is written last: a crash
// leaves at most unreferenced storage files, never a half-written version. A
// daemon started on the same directory reloads every complete version before
// it serves: objects become sealed, file-backed (cold tier) objects that
// export and canonical restore read like any NVMe copy. Dropping a version or
// retention removes its manifest; a storage file goes with the last object
// that uses it. Persisted objects carry a daemon-side holder, so they outlive
// the ranks that created them.
#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <cerrno>
#include <cstdio>
#include <cstring>

#include "daemon.h"
#include "ofld/log.h"
#include "ofld/metrics.h"
#include "ofld/zbf16.h"

namespace ofld {

namespace {

constexpr const char* TAG = "persist";
constexpr uint32_t kStorageMagic = 0x5350464Fu;  // "OFPS"
constexpr uint32_t kFormat = 1;
constexpr uint64_t kDataOffset = 4096;
constexpr uint64_t kPage = 4096;

struct StorageHeader {
    uint32_t magic, format;
    uint64_t storage_id, nbytes, hash_lo, hash_hi;
    uint64_t reserved[3];
};
static_assert(sizeof(StorageHeader) == 64, "storage header is 64 bytes");

struct PersistedObject {
    uint64_t object_id = 0, nbytes = 0, hash_lo = 0, hash_hi = 0, storage_id = 0;
    uint32_t producer_rank = 0;
    CanonicalTensorKeyWire key;
};
template <class V> void fields(V& v, PersistedObject& m) {
    v(m.object_id, m.nbytes, m.hash_lo, m.hash_hi, m.storage_id, m.producer_rank, m.key);
}

struct PersistedVersion {
    uint32_t format = kFormat;
    JobKeyWire job;
    uint32_t role = 0;
    uint64_t version = 0, sealed_ns = 0, total_nbytes = 0, hash_lo = 0, hash_hi = 0;
    bool promoted = false;
    std::vector<PersistedObject> objects;
};
template <class V> void fields(V& v, PersistedVersion& m) {
    v(m.format, m.job, m.role, m.version, m.sealed_ns, m.total_nbytes, m.hash_lo, m.hash_hi, m.promoted, m.objects);
}

bool write_fully(int fd, const void* p, uint64_t n) {
    const char* c = static_cast<const char*>(p);
    while (n) {
        ssize_t w = ::write(fd, c, size_t(std::min<uint64_t>(n, 1ull << 30)));
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) return false;
        c += w;
        n -= uint64_t(w);
    }
    return true;
}

bool read_file(const std::string& path, std::vector<uint8_t>* out) {
    int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return false;
    struct stat st;
    bool ok = ::fstat(fd, &st) == 0;
    if (ok) {
        out->resize(size_t(st.st_size));
        uint64_t got = 0;
        while (ok && got < out->size()) {
            ssize_t r = ::read(fd, out->data() + got, out->size() - got);
            if (r < 0 && errno == EINTR) continue;
            ok = r > 0;
            if (ok) got += uint64_t(r);
        }
    }
    ::close(fd);
    return ok;
}

// Writes `bytes` to `path` through a synced temporary file.
bool write_atomically(const std::string& path, const std::vector<uint8_t>& bytes) {
    const std::string tmp = path + ".tmp";
    int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
    if (fd < 0) return false;
    bool ok = write_fully(fd, bytes.data(), bytes.size()) && ::fsync(fd) == 0;
    ::close(fd);
    if (ok) ok = ::rename(tmp.c_str(), path.c_str()) == 0;
    if (!ok) ::unlink(tmp.c_str());
    return ok;
}

void sync_dir(const std::string& dir) {
    int fd = ::open(dir.c_str(), O_RDONLY | O_DIRECTORY | O_CLOEXEC);
    if (fd >= 0) {
        ::fsync(fd);
        ::close(fd);
    }
}

bool make_dirs(const std::string& dir) {
    std::string cur;
    for (size_t i = 0; i <= dir.size(); ++i) {
        if (i == dir.size() || dir[i] == '/') {
            if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST) return false;
        }
        if (i < dir.size()) cur += dir[i];
    }
    return true;
}

std::string storage_name(uint64_t id) {
    char b[40];
    std::snprintf(b, sizeof(b), "/s%016llx.obj", (unsigned long long)id);
    return b;
}

std::string manifest_name(uint32_t role, uint64_t version) {
    char b[64];
    std::snprintf(b, sizeof(b), "/m%u_%llu.man", role, (unsigned long long)version);
    return b;
}

}  // namespace

// ---------------------------------------------------------------------------
// Read holds
// ---------------------------------------------------------------------------
bool Daemon::begin_read(CanonicalObject& o, ReadSrc* src, std::string* why) {
    auto lit = locations_.find(o.synthetic_tid);
    if (lit == locations_.end()) {
        *why = "object not resident";
        return false;
    }
    *src = ReadSrc{};
    src->kind = lit->second.kind;
    src->nbytes = o.nbytes;
    src->fmt = lit->second.fmt;
    if (src->kind == OFLD_LOC_PINNED) {
        uint32_t st = state_of(lit->second.slot);
        if (st != OFLD_SLOT_PINNED_VALID && st != OFLD_SLOT_DRAIN_IN_FLIGHT) {
            *why = "object transitioning; retry";
            return false;
        }
        src->pinned = slot_ptr(lit->second.slot);
    } else if (src->kind == OFLD_LOC_PAGEABLE || src->kind == OFLD_LOC_NVME) {
        src->cold_ref = lit->second.cold_ref;
        if (!pin_cold(src->cold_ref, &src->cold)) {
            *why = "cold copy unavailable";
            return false;
        }
    } else {
        *why = "object not resident";
        return false;
    }
    if (o.export_refs++ == 0) o.state_before_export = o.state;
    storage_io(o.synthetic_tid, +1);
    o.state = OBJ_EXPORT_IN_FLIGHT;
    return true;
}

void Daemon::end_read(uint64_t oid, const ReadSrc& src) {
    if (src.cold_ref) unpin_cold(src.cold_ref);
    if (CanonicalObject* o = find_object(oid)) {
        if (o->export_refs) {
            o->export_refs--;
            storage_io(o->synthetic_tid, -1);
        }
        if (o->export_refs == 0) o->state = o->state_before_export;
        maybe_free_object(*o);
    }
}

bool Daemon::decode_out(const ReadSrc& src, const char* stored, uint64_t off, uint64_t n, char* out) {
    const zbf16::Coding c = (src.fmt & OFLD_FLAG_FORMAT_ZF32) ? zbf16::Coding::kZf32 : zbf16::Coding::kZbf16;
    constexpr uint64_t kTask = 1ull << 20;  // a multiple of both block sizes
    const uint32_t tasks = uint32_t((n + kTask - 1) / kTask);
    std::atomic<bool> ok{true};
    copy_pool_.run(tasks, [&](uint32_t i) {
        thread_local std::vector<uint32_t> keys;
        const uint64_t o = uint64_t(i) * kTask, len = std::min(kTask, n - o);
        if (!zbf16::decode_range(c, reinterpret_cast<const uint8_t*>(stored) + o, src.nbytes, off + o, len,
                                 reinterpret_cast<uint8_t*>(out) + o, keys))
            ok.store(false);
    });
    return ok.load();
}

bool Daemon::copy_out(const ReadSrc& src, char* dst, uint64_t off, uint64_t n) {
    if (off + n > src.nbytes) return false;
    if (src.pinned) {
        std::memcpy(dst, src.pinned + off, n);
        return true;
    }
    if (src.kind == OFLD_LOC_PAGEABLE) {
        if (!src.cold.pageable) return false;
        std::memcpy(dst, src.cold.pageable + off, n);
        return true;
    }
    return read_cold(src.cold, dst, off, n);
}

// ---------------------------------------------------------------------------
// Durable versions
// ---------------------------------------------------------------------------
std::string Daemon::persist_job_dir(const JobUID& uid) const {
    char b[96];
    std::snprintf(b, sizeof(b), "/j%llu_%llu_%llu", (unsigned long long)uid.tenant_id,
                  (unsigned long long)uid.job_id, (unsigned long long)uid.launch_epoch);
    return cfg_.v2_persist_dir + b;
}

void Daemon::enqueue_persist(const VersionKey& vk) {
    if (cfg_.v2_persist_dir.empty()) return;
    {
        std::lock_guard<std::mutex> g(persist_mu_);
        persist_queue_.push_back(vk);
    }
    persist_cv_.notify_one();
}

// A version whose objects are moving between tiers is retried after the
// others (every 10 ms, for up to about a minute) instead of being dropped.
void Daemon::persist_loop() {
    std::map<VersionKey, int> attempts;
    while (workers_on_.load()) {
        VersionKey vk;
        {
            std::unique_lock<std::mutex> g(persist_mu_);
            persist_cv_.wait_for(g, std::chrono::milliseconds(100),
                                 [&] { return !persist_queue_.empty() || !workers_on_.load(); });
            if (persist_queue_.empty()) continue;
            vk = persist_queue_.front();
            persist_queue_.pop_front();
        }
        const int rc = persist_version(vk);
        if (rc == 0 && ++attempts[vk] < 6000) {
            {
                std::lock_guard<std::mutex> g(persist_mu_);
                persist_queue_.push_back(vk);
            }
            sleep_us(10000);
            continue;
        }
        attempts.erase(vk);
        if (rc <= 0)
            LOG_WARN(TAG, "version job=%llu role=%u v=%llu not persisted", (unsigned long long)vk.job.job_id,
                     vk.role, (unsigned long long)vk.version);
    }
}

int Daemon::persist_version(const VersionKey& vk) {
    PersistedVersion pv;
    std::string dir;
    std::vector<uint64_t> todo;  // one object per storage not yet on disk
    {
        std::lock_guard<std::mutex> g(mu_);
        auto mit = manifests_.find(vk);
        if (mit == manifests_.end() || mit->second.state != MANIFEST_SEALED) return 1;  // dropped meanwhile
        auto jit = jobs_.find(vk.job);
        if (jit == jobs_.end()) return 1;
        const Manifest& man = mit->second;
        dir = persist_job_dir(vk.job);
        pv.job = JobKeyWire{vk.job.tenant_id, vk.job.job_id, vk.job.launch_epoch, jit->second.name};
        pv.role = vk.role;
        pv.version = vk.version;
        pv.sealed_ns = man.sealed_ns;
        pv.total_nbytes = man.total_nbytes;
        pv.hash_lo = man.hash_lo;
        pv.hash_hi = man.hash_hi;
        auto lit = latest_sealed_.find({vk.job, vk.role});
        pv.promoted = lit != latest_sealed_.end() && lit->second >= vk.version;
        std::set<uint64_t> seen;
        for (uint64_t oid : man.object_ids) {
            CanonicalObject* o = find_object(oid);
            if (!o) return -1;
            PersistedObject po;
            po.object_id = oid;
            po.nbytes = o->nbytes;
            po.hash_lo = o->hash_lo;
            po.hash_hi = o->hash_hi;
            po.storage_id = o->synthetic_tid;
            po.producer_rank = o->producer_rank;
            po.key = o->key;
            pv.objects.push_back(po);
            if (!persisted_files_.count(o->synthetic_tid) && seen.insert(o->synthetic_tid).second) todo.push_back(oid);
        }
    }
    if (!make_dirs(dir)) {
        LOG_ERR(TAG, "mkdir %s: %s", dir.c_str(), std::strerror(errno));
        return -1;
    }
    const std::string jobrec = dir + "/job.rec";
    if (::access(jobrec.c_str(), F_OK) != 0 && !write_atomically(jobrec, encode(pv.job))) return -1;

    std::vector<char> bounce;
    for (uint64_t oid : todo) {
        ReadSrc src;
        std::string why;
        uint64_t tid = 0, nbytes = 0, hlo = 0, hhi = 0;
        {
            std::lock_guard<std::mutex> g(mu_);
            CanonicalObject* o = find_object(oid);
            if (!o) return -1;
            if (persisted_files_.count(o->synthetic_tid)) continue;  // another version wrote it
            if (!begin_read(*o, &src, &why)) return why.find("retry") != std::string::npos ? 0 : -1;
            tid = o->synthetic_tid;
            nbytes = o->nbytes;
            hlo = o->hash_lo;
            hhi = o->hash_hi;
        }
        const std::string path = dir + storage_name(tid), tmp = path + ".tmp";
        bool ok = false;
        int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (fd >= 0) {
            std::vector<uint8_t> head(kDataOffset, 0);
            // reserved[0]: the coding of the stored bytes (OFLD_FLAG_FORMAT_*), written as stored
            StorageHeader h{kStorageMagic, kFormat, tid, nbytes, hlo, hhi, {src.fmt, 0, 0}};
            std::memcpy(head.data(), &h, sizeof(h));
            ok = write_fully(fd, head.data(), head.size());
            const uint64_t chunk = 8ull << 20;
            for (uint64_t off = 0; ok && off < nbytes; off += chunk) {
                const uint64_t n = std::min(chunk, nbytes - off);
                if (src.pinned) {
                    ok = write_fully(fd, src.pinned + off, n);
                } else {
                    bounce.resize(n);
                    ok = copy_out(src, bounce.data(), off, n) && write_fully(fd, bounce.data(), n);
                }
            }
            // whole pages, so O_DIRECT reads of the tail stay inside the file
            ok = ok && ::ftruncate(fd, off_t(round_up(kDataOffset + nbytes, kPage))) == 0 && ::fsync(fd) == 0;
            ::close(fd);
            ok = ok && ::rename(tmp.c_str(), path.c_str()) == 0;
        }
        if (!ok) ::unlink(tmp.c_str());
        std::lock_guard<std::mutex> g(mu_);
        end_read(oid, src);
        if (!ok) {
            LOG_ERR(TAG, "writing %s failed: %s", path.c_str(), std::strerror(errno));
            return -1;
        }
        persisted_files_[tid] = path;
        Metrics::get().add(M::kPersistedBytes, nbytes);
    }
    sync_dir(dir);
    const std::string mpath = dir + manifest_name(vk.role, vk.version);
    if (!write_atomically(mpath, encode(pv))) return -1;
    sync_dir(dir);
    std::lock_guard<std::mutex> g(mu_);
    auto mit = manifests_.find(vk);
    if (mit == manifests_.end() || mit->second.state != MANIFEST_SEALED) {
        ::unlink(mpath.c_str());  // dropped while it was being written
        return 1;
    }
    for (uint64_t oid : mit->second.object_ids)
        if (CanonicalObject* o = find_object(oid)) o->holders.insert(kPersistHolder);
    Metrics::get().inc(M::kVersionsPersisted);
    LOG_INFO(TAG, "persisted job=%llu role=%u version=%llu (%zu objects, %zu storage files written)",
             (unsigned long long)vk.job.job_id, vk.role, (unsigned long long)vk.version, pv.objects.size(),
             todo.size());
    return 1;
}

void Daemon::unlink_persisted_manifest(const VersionKey& vk) {
    if (cfg_.v2_persist_dir.empty()) return;
    ::unlink((persist_job_dir(vk.job) + manifest_name(vk.role, vk.version)).c_str());
}

void Daemon::forget_persisted_storage(uint64_t tid) {
    auto it = persisted_files_.find(tid);
    if (it == persisted_files_.end()) return;
    ::unlink(it->second.c_str());
    persisted_files_.erase(it);
}

void Daemon::recover_persisted() {
    const std::string& root = cfg_.v2_persist_dir;
    if (!make_dirs(root)) throw std::runtime_error("manifest.persist_dir: cannot create " + root);
    DIR* d = ::opendir(root.c_str());
    if (!d) return;
    std::vector<std::string> jobdirs;
    while (dirent* e = ::readdir(d))
        if (e->d_name[0] == 'j') jobdirs.push_back(root + "/" + e->d_name);
    ::closedir(d);
    std::sort(jobdirs.begin(), jobdirs.end());
    uint64_t versions = 0;
    for (const std::string& jd : jobdirs) {
        std::vector<uint8_t> buf;
        if (!read_file(jd + "/job.rec", &buf)) continue;
        JobKeyWire jk;
        try {
            jk = decode<JobKeyWire>(buf);
        } catch (const std::exception&) {
            LOG_WARN(TAG, "%s/job.rec unreadable; skipped", jd.c_str());
            continue;
        }
        const JobUID uid{jk.tenant_id, jk.job_id, jk.launch_epoch};
        if (!jobs_.count(uid)) {
            Job j;
            j.uid = uid;
            j.name = jk.job_name;
            j.created_ns = real_ns();
            init_job_quotas(j);
            jobs_[uid] = j;
        }
        next_launch_epoch_ = std::max(next_launch_epoch_, jk.launch_epoch + 1);
        Job& job = jobs_[uid];
        DIR* jdir = ::opendir(jd.c_str());
        if (!jdir) continue;
        std::vector<std::string> mans;
        while (dirent* e = ::readdir(jdir)) {
            const std::string n = e->d_name;
            if (n.size() > 4 && n[0] == 'm' && n.compare(n.size() - 4, 4, ".man") == 0) mans.push_back(jd + "/" + n);
        }
        ::closedir(jdir);
        std::sort(mans.begin(), mans.end());
        for (const std::string& mp : mans) {
            PersistedVersion pv;
            try {
                if (!read_file(mp, &buf)) continue;
                pv = decode<PersistedVersion>(buf);
            } catch (const std::exception&) {
                LOG_WARN(TAG, "%s unreadable; skipped", mp.c_str());
                continue;
            }
            if (pv.format != kFormat) continue;
            // every storage file must be present and match before anything is loaded
            bool complete = true;
            std::map<uint64_t, uint64_t> coding;  // storage id -> OFLD_FLAG_FORMAT_* of its bytes
            for (const PersistedObject& po : pv.objects) {
                if (persisted_files_.count(po.storage_id)) continue;
                StorageHeader h{};
                int fd = ::open((jd + storage_name(po.storage_id)).c_str(), O_RDONLY | O_CLOEXEC);
                struct stat st;
                complete = fd >= 0 && ::pread(fd, &h, sizeof(h), 0) == ssize_t(sizeof(h)) && ::fstat(fd, &st) == 0 &&
                           h.magic == kStorageMagic && h.storage_id == po.storage_id && h.nbytes == po.nbytes &&
                           uint64_t(st.st_size) >= kDataOffset + po.nbytes &&
                           (h.reserved[0] & ~OFLD_FLAG_FORMAT_MASK) == 0 && h.reserved[0] != OFLD_FLAG_FORMAT_MASK;
                if (complete) coding[po.storage_id] = h.reserved[0];
                if (fd >= 0) ::close(fd);
                if (!complete) break;
            }
            if (!complete) {
                LOG_WARN(TAG, "%s: storage files missing or damaged; version skipped", mp.c_str());
                continue;
            }
            VersionKey vk{uid, pv.role, pv.version};
            Manifest man;
            man.vk = vk;
            man.state = MANIFEST_SEALED;
            man.created_ns = man.sealed_ns = pv.sealed_ns;
            man.total_nbytes = pv.total_nbytes;
            man.hash_lo = pv.hash_lo;
            man.hash_hi = pv.hash_hi;
            for (const PersistedObject& po : pv.objects) {
                man.object_ids.push_back(po.object_id);
                next_object_ = std::max(next_object_, po.object_id + 1);
                next_object_ = std::max(next_object_, (po.storage_id & ~kCanonicalTidBit) + 1);
                if (objects_.count(po.object_id)) continue;
                if (!persisted_files_.count(po.storage_id)) {
                    const std::string path = jd + storage_name(po.storage_id);
                    ColdEntry c;
                    c.kind = OFLD_LOC_NVME;
                    c.nbytes = po.nbytes;
                    c.extents.push_back(Extent{path, kDataOffset, po.nbytes});
                    c.persisted = true;
                    Location loc;
                    loc.version = pv.version;
                    loc.kind = OFLD_LOC_NVME;
                    loc.cold_ref = commit_cold(std::move(c));
                    loc.nbytes = po.nbytes;
                    loc.fmt = coding[po.storage_id];
                    locations_[po.storage_id] = loc;
                    persisted_files_[po.storage_id] = path;
                }
                CanonicalObject o;
                o.object_id = po.object_id;
                o.key = po.key;
                o.key_str = key_string(po.key, cfg_.v2_cross_job_dedup);
                o.nbytes = po.nbytes;
                o.state = OBJ_SEALED;
                o.holders.insert(kPersistHolder);
                o.producer_rank = po.producer_rank;
                o.hash_lo = po.hash_lo;
                o.hash_hi = po.hash_hi;
                o.synthetic_tid = po.storage_id;
                o.created_ns = o.sealed_ns = o.last_access_ns = pv.sealed_ns;
                storage_[po.storage_id].objects++;
                object_by_key_[o.key_str] = o.object_id;
                objects_[o.object_id] = o;
                job.object_count++;
            }
            std::sort(man.object_ids.begin(), man.object_ids.end());
            manifests_[vk] = man;
            if (pv.promoted) {
                uint64_t& latest = latest_sealed_[{uid, pv.role}];
                latest = std::max(latest, pv.version);
            }
            ++versions;
            Metrics::get().inc(M::kVersionsRecovered);
        }
    }
    if (versions) LOG_INFO(TAG, "recovered %llu sealed versions from %s", (unsigned long long)versions, root.c_str());
}

}  // namespace ofld
