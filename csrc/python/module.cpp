// Python binding (`statespectre_b200._C`). No torch headers: tensors cross
// the boundary as (data pointer, byte count, CUDA stream handle) integers and
// the Python layer owns every torch object. Control-plane RPCs travel as raw
// encoded bodies (`Agent.call_raw`) that the Python schema mirror
// (statespectre_b200/_wire.py) encodes and decodes, so the binding has no
// per-message code; data-moving calls have typed bindings.
#include <cuda_runtime.h>
#include <sys/socket.h>
#include <sys/time.h>

#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <memory>
#include <thread>

#include "../agent/agent.h"
#include "../daemon/config.h"
#include "../daemon/daemon.h"
#include "../kernels/kernels.h"
#include "../kernels/timing.h"
#include "ofld/chunk_hash.h"
#include "ofld/zbf16.h"
#include "ofld/codec.h"
#include "ofld/log.h"
#include "ofld/metrics.h"
#include "ofld/transport.h"

namespace py = pybind11;
using namespace ofld;

void bind_fabric(py::module_& m);  // fabric_bind.cpp

namespace {

bool py_alive() { return Py_IsInitialized() && !_Py_IsFinalizing(); }

// Wrap a Python callable so it may run (and be destroyed) on any thread.
DoneCallback wrap_cb(py::object fn) {
    if (fn.is_none()) return {};
    std::shared_ptr<py::object> holder(new py::object(std::move(fn)), [](py::object* p) {
        if (py_alive()) {
            py::gil_scoped_acquire g;
            delete p;
        }  // interpreter gone: leak rather than touch Python
    });
    return [holder]() {
        if (!py_alive()) return;
        py::gil_scoped_acquire g;
        try {
            (*holder)();
        } catch (py::error_already_set& e) {
            e.discard_as_unraisable("statespectre_b200 completion callback");
        }
    };
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Generic raw round trip on a dedicated connection (used by RolloutWeightClient
// fallbacks and tests that drive the wire directly).
class RawConn {
 public:
    // reply_timeout_ms > 0: a call whose reply does not arrive in time fails
    // (a daemon that does not know an opcode may leave it unanswered)
    RawConn(const std::string& addr, int timeout_ms, int reply_timeout_ms) {
        if (addr.rfind("tcp://", 0) == 0) {
            std::string host;
            uint16_t port = 0;
            if (!split_host_port(addr.substr(6), &host, &port)) throw std::runtime_error("bad tcp address");
            fd_ = tcp_connect(host, port, timeout_ms);
        } else {
            fd_ = uds_connect(addr.rfind("unix://", 0) == 0 ? addr.substr(7) : addr, timeout_ms);
        }
        if (reply_timeout_ms > 0) {
            timeval tv{reply_timeout_ms / 1000, (reply_timeout_ms % 1000) * 1000};
            ::setsockopt(fd_, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
        }
    }
    ~RawConn() { close_fd(fd_); }
    py::tuple call(int op, py::bytes body, std::vector<int> fds_in) {
        std::string b = body;
        std::vector<uint8_t> frame = make_frame(Op(op), std::vector<uint8_t>(b.begin(), b.end()));
        Op rop;
        std::vector<uint8_t> reply;
        std::vector<int> fds;
        {
            py::gil_scoped_release nogil;
            send_frame(fd_, frame, fds_in);
            if (!recv_frame(fd_, &rop, &reply, &fds)) throw std::runtime_error("connection closed");
        }
        return py::make_tuple(int(rop), py::bytes(reinterpret_cast<const char*>(reply.data()), reply.size()), fds);
    }
    // Send raw bytes without waiting (fault-injection tests: truncated frames).
    void send_bytes(py::bytes data) {
        std::string s = data;
        if (!write_all(fd_, s.data(), s.size())) throw std::runtime_error("send failed");
    }
    void close() {
        close_fd(fd_);
        fd_ = -1;
    }

 private:
    int fd_ = -1;
};

class DaemonThread {
 public:
    explicit DaemonThread(const DaemonConfig& cfg) : d_(new Daemon(cfg)) {
        th_ = std::thread([this] {
            try {
                d_->run();
            } catch (const std::exception& e) {
                LOG_ERR("daemon-thread", "%s", e.what());
            }
        });
        if (!d_->wait_ready(10000)) throw std::runtime_error("daemon did not start");
    }
    ~DaemonThread() { stop(); }
    void stop() {
        if (!d_) return;
        d_->stop();
        if (th_.joinable()) {
            py::gil_scoped_release nogil;
            th_.join();
        }
        d_.reset();
    }
    void fake_host_memory(uint64_t avail) {
        if (d_) d_->fake_host_memory(avail);
    }
    void inject_io_failures(int w, int r) {
        if (d_) d_->inject_io_failures(w, r);
    }
    void pause_rings(bool p) {
        if (d_) d_->pause_rings(p);
    }
    std::string socket() const { return d_ ? d_->config().socket_path : ""; }

 private:
    std::unique_ptr<Daemon> d_;
    std::thread th_;
};

DaemonConfig config_from(py::dict kw) {
    DaemonConfig c;
    if (kw.contains("yaml")) {
        c = parse_config(kw["yaml"].cast<std::string>());
    } else {
        uint64_t mb = kw.contains("arena_mb") ? kw["arena_mb"].cast<uint64_t>() : 256;
        c = smoke_config(mb << 20, kw.contains("numa") ? kw["numa"].cast<uint32_t>() : 0,
                         kw.contains("gpu") ? kw["gpu"].cast<uint32_t>() : 0);
    }
    if (kw.contains("socket")) c.socket_path = kw["socket"].cast<std::string>();
    if (kw.contains("slot_mb")) c.allocation_granularity_bytes = kw["slot_mb"].cast<uint64_t>() << 20;
    if (kw.contains("drain_on_complete")) c.drain_on_d2h_complete = kw["drain_on_complete"].cast<bool>();
    if (kw.contains("heartbeat_timeout_ms")) c.heartbeat_timeout_ms = kw["heartbeat_timeout_ms"].cast<uint64_t>();
    if (kw.contains("tcp_port")) c.v2_control_tcp_port = kw["tcp_port"].cast<uint32_t>();
    if (kw.contains("nvme_dir")) {
        c.nvme_enabled = true;
        c.nvme_path = kw["nvme_dir"].cast<std::string>();
        c.nvme_direct_io = kw.contains("direct_io") ? kw["direct_io"].cast<bool>() : false;
    }
    if (kw.contains("drain_target")) {
        std::string t = kw["drain_target"].cast<std::string>();
        c.drain_target = t == "nvme" ? DrainTarget::kNvmeOnly
                         : t == "pageable_then_nvme" ? DrainTarget::kPageableThenNvme
                                                     : DrainTarget::kPageableOnly;
    }
    if (kw.contains("pageable_limit_mb")) c.pageable_limit_bytes = kw["pageable_limit_mb"].cast<uint64_t>() << 20;
    if (kw.contains("io_engine")) c.nvme_io_engine = kw["io_engine"].cast<std::string>();
    if (kw.contains("persist_dir")) c.v2_persist_dir = kw["persist_dir"].cast<std::string>();
    if (kw.contains("retain_sealed_versions"))
        c.v2_retain_sealed_versions = kw["retain_sealed_versions"].cast<uint32_t>();
    if (kw.contains("thresholds")) {
        auto t = kw["thresholds"].cast<std::tuple<double, double, double>>();
        c.normal_threshold = std::get<0>(t);
        c.priority_threshold = std::get<1>(t);
        c.aggressive_threshold = std::get<2>(t);
    }
    if (kw.contains("quota_max_pinned_bytes")) c.v2_quota_max_pinned_bytes = kw["quota_max_pinned_bytes"].cast<uint64_t>();
    if (kw.contains("creating_policy")) c.v2_creating_policy = kw["creating_policy"].cast<uint32_t>();
    if (kw.contains("copy_threads")) c.copy_threads = kw["copy_threads"].cast<uint32_t>();
    validate(c);
    return c;
}

py::dict stats_dict(const AgentStats& s) {
    py::dict d;
    d["rank_id"] = s.rank_id;
    d["gpu_id"] = s.gpu_id;
    d["numa_node"] = s.numa_node;
    d["registered_pinned_bytes"] = s.registered_pinned_bytes;
    d["inflight_d2h_bytes"] = s.inflight_d2h_bytes;
    d["inflight_h2d_bytes"] = s.inflight_h2d_bytes;
    d["evict_count"] = s.evict_count;
    d["restore_count"] = s.restore_count;
    d["d2h_completed"] = s.d2h_completed;
    d["h2d_completed"] = s.h2d_completed;
    d["rank_epoch"] = s.rank_epoch;
    d["num_slots"] = s.num_slots;
    d["d2h_bytes"] = s.d2h_bytes;
    d["h2d_bytes"] = s.h2d_bytes;
    d["kernel_launches"] = s.kernel_launches;
    d["rpc_count"] = s.rpc_count;
    d["d2h_ns"] = s.d2h_ns;
    d["h2d_ns"] = s.h2d_ns;
    d["registration_ns"] = s.registration_ns;
    d["coded_canonical"] = s.coded_canonical;
    return d;
}

// Agent wrapper owning the GIL discipline.
class PyAgent {
 public:
    explicit PyAgent(py::dict kw) {
        AgentOptions o;
        for (auto item : kw) {
            std::string k = item.first.cast<std::string>();
            py::handle v = item.second;
            if (k == "socket_path") o.socket_path = v.cast<std::string>();
            else if (k == "device") o.device = v.cast<int>();
            else if (k == "rank_id") o.rank_id = v.cast<uint32_t>();
            else if (k == "local_rank") o.local_rank = v.cast<uint32_t>();
            else if (k == "world_rank") o.world_rank = v.cast<uint32_t>();
            else if (k == "numa_node") o.numa_node = v.cast<int>();
            else if (k == "eager_register") o.eager_register = v.cast<bool>();
            else if (k == "heartbeat_ms") o.heartbeat_ms = v.cast<uint64_t>();
            else if (k == "progress_poll_us") o.progress_poll_us = v.cast<uint64_t>();
            else if (k == "prefetch_poll_us") o.prefetch_poll_us = v.cast<uint64_t>();
            else if (k == "engine") o.engine = v.cast<std::string>();
            else if (k == "uncoded") o.uncoded = v.cast<std::string>();
            else if (k == "coded_restore") o.coded_restore = v.cast<std::string>();
            else if (k == "coded_evict") o.coded_evict = v.cast<std::string>();
            else if (k == "evict_ctas") o.evict_ctas = v.cast<int>();
            else if (k == "restore_ctas") o.restore_ctas = v.cast<int>();
            else if (k == "hash_ctas") o.hash_ctas = v.cast<int>();
            else if (k == "stage_ctas") o.stage_ctas = v.cast<int>();
            else if (k == "stage_depth") o.stage_depth = v.cast<int>();
            else if (k == "stage_piece_chunks") o.stage_piece_chunks = v.cast<int>();
            else if (k == "hash_on_evict") o.hash_on_evict = v.cast<bool>();
            else if (k == "host_hash_max_bytes") o.host_hash_max_bytes = v.cast<uint64_t>();
            else if (k == "use_ring") o.use_ring = v.cast<bool>();
            else if (k == "fast_submit") o.fast_submit = v.cast<bool>();
            else if (k == "keep_digests") o.keep_digests = v.cast<bool>();
            else if (k == "zero_canonical_hash") o.zero_canonical_hash = v.cast<bool>();
            else if (k == "stream_priority") o.stream_priority = v.cast<int>();
            else if (k == "compress") o.compress = v.cast<bool>();
            else if (k == "compress_canonical") o.compress_canonical = v.cast<bool>();
            else if (k == "v1_only") o.v1_only = v.cast<bool>();
            else if (k == "compress_min_bytes") o.compress_min_bytes = v.cast<uint64_t>();
            else if (k == "batch_group_bytes") o.batch_group_bytes = v.cast<uint64_t>();
            else if (k == "kernel_timing") o.kernel_timing = v.cast<bool>();
            else if (k == "registration_threads") o.registration_threads = v.cast<int>();
            else if (k == "blocked_wait_ms") o.blocked_wait_ms = v.cast<uint64_t>();
            else throw std::invalid_argument("unknown agent option '" + k + "'");
        }
        py::gil_scoped_release nogil;
        a_.reset(new Agent(o));
    }
    Agent& ag() {
        if (!a_)
            throw std::runtime_error(
                "statespectre: session is closed (its offload_context exited or was garbage-collected)");
        return *a_;
    }
    void close() {
        std::unique_ptr<Agent> a = std::move(a_);
        py::gil_scoped_release nogil;
        a.reset();
    }
    std::unique_ptr<Agent> a_;
};

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "statespectre_b200 native runtime: rank agent, in-process daemon, sm_100a kernels";

    py::class_<PyAgent>(m, "Agent")
        .def(py::init<py::dict>())
        .def("close", &PyAgent::close)
        .def(
            "evict",
            [](PyAgent& self, uint64_t ptr, uint64_t nbytes, uint64_t stream, bool destructive, uint64_t tid,
               uint64_t ver, std::string name, py::object cb, bool wait, uint32_t fmt_hint) {
                DoneCallback f = wrap_cb(std::move(cb));
                EvictTicket t;
                {
                    py::gil_scoped_release nogil;
                    t = self.ag().evict(ptr, nbytes, stream, destructive, tid, ver, name, std::move(f), wait,
                                        fmt_hint);
                }
                return py::make_tuple(t.ok, t.message, t.lease_id, t.slot_id, t.hash_lo, t.hash_hi, t.coded);
            },
            py::arg("ptr"), py::arg("nbytes"), py::arg("stream"), py::arg("destructive"), py::arg("tensor_id"),
            py::arg("version"), py::arg("name"), py::arg("callback"), py::arg("wait"), py::arg("fmt_hint") = 0)
        .def(
            "evict_batch",
            [](PyAgent& self, std::vector<std::vector<uint64_t>> items, uint64_t stream, bool wait) {
                // items: (ptr, nbytes, tensor_id, version[, fmt_hint])
                std::vector<BatchItem> b;
                for (auto& t : items) {
                    if (t.size() < 4) throw std::invalid_argument("evict_batch item needs 4 or 5 fields");
                    b.push_back(BatchItem{t[0], t[1], t[2], t[3], t.size() > 4 ? uint32_t(t[4]) : 0u});
                }
                std::vector<EvictTicket> r;
                {
                    py::gil_scoped_release nogil;
                    r = self.ag().evict_batch(b, stream, wait);
                }
                py::list out;
                for (auto& t : r) out.append(py::make_tuple(t.ok, t.message, t.coded));
                return out;
            })
        .def(
            "restore",
            [](PyAgent& self, uint64_t tid, uint64_t ver, uint64_t ptr, uint64_t nbytes, uint64_t stream, bool wait,
               int cast, uint64_t scales_ptr, bool verify, bool keep_pinned) {
                RestoreOptions ro{cast, scales_ptr, verify, keep_pinned};
                RestoreOutcome r;
                {
                    py::gil_scoped_release nogil;
                    r = self.ag().restore(tid, ver, ptr, nbytes, stream, wait, ro);
                }
                return py::make_tuple(r.ok, r.message, r.mismatched_chunks);
            },
            py::arg("tensor_id"), py::arg("version"), py::arg("ptr"), py::arg("nbytes"), py::arg("stream"),
            py::arg("wait"), py::arg("cast") = 0, py::arg("scales_ptr") = 0, py::arg("verify") = false,
            py::arg("keep_pinned") = false)
        .def("restore_batch",
             [](PyAgent& self, std::vector<std::tuple<uint64_t, uint64_t, uint64_t, uint64_t>> items, uint64_t stream,
                bool wait) {
                 std::vector<BatchItem> b;
                 for (auto& t : items) b.push_back(BatchItem{std::get<0>(t), std::get<1>(t), std::get<2>(t), std::get<3>(t)});
                 std::vector<RestoreOutcome> r;
                 {
                     py::gil_scoped_release nogil;
                     r = self.ag().restore_batch(b, stream, wait);
                 }
                 py::list out;
                 for (auto& x : r) out.append(py::make_tuple(x.ok, x.message));
                 return out;
             })
        .def("is_offloaded", [](PyAgent& s, uint64_t t, uint64_t v) { return s.ag().is_offloaded(t, v); })
        .def("wait_offloaded",
             [](PyAgent& s, uint64_t t, uint64_t v) {
                 py::gil_scoped_release nogil;
                 s.ag().wait_offloaded(t, v);
             })
        .def("is_restored", [](PyAgent& s, uint64_t t, uint64_t v) { return s.ag().is_restored(t, v); })
        .def("wait_restored",
             [](PyAgent& s, uint64_t t, uint64_t v) {
                 py::gil_scoped_release nogil;
                 s.ag().wait_restored(t, v);
             })
        .def("tensor_hash",
             [](PyAgent& s, uint64_t t, uint64_t v) -> py::object {
                 uint64_t lo = 0, hi = 0;
                 if (!s.ag().tensor_hash(t, v, &lo, &hi)) return py::none();
                 return py::make_tuple(lo, hi);
             })
        .def("location",
             [](PyAgent& s, uint64_t t, uint64_t v) {
                 py::gil_scoped_release nogil;
                 return s.ag().location(t, v);
             })
        .def("discard",
             [](PyAgent& s, uint64_t t, uint64_t v) {
                 py::gil_scoped_release nogil;
                 s.ag().discard(t, v);
             })
        .def("discard_batch",
             [](PyAgent& s, std::vector<std::pair<uint64_t, uint64_t>> items) {
                 py::gil_scoped_release nogil;
                 s.ag().discard_batch(items);
             })
        .def("assert_no_inflight", [](PyAgent& s) { s.ag().assert_no_inflight(); })
        .def("synchronize",
             [](PyAgent& s) {
                 py::gil_scoped_release nogil;
                 s.ag().synchronize();
             })
        .def(
            "canonical_evict",
            [](PyAgent& self, uint64_t ptr, uint64_t nbytes, uint64_t stream, bool destructive, py::bytes req_body,
               py::object cb, bool wait) {
                std::string b = req_body;
                auto req = decode<RequestCanonicalEvictRequest>(reinterpret_cast<const uint8_t*>(b.data()), b.size());
                DoneCallback f = wrap_cb(std::move(cb));
                CanonicalOutcome r;
                {
                    py::gil_scoped_release nogil;
                    r = self.ag().canonical_evict(ptr, nbytes, stream, destructive, req, std::move(f), wait);
                }
                return py::make_tuple(r.ok, r.action, r.object_id, r.did_d2h, r.message, r.hash_lo, r.hash_hi);
            })
        .def(
            "canonical_evict_batch",
            [](PyAgent& self, py::list items, uint64_t stream, bool destructive, uint64_t max_inflight_bytes) {
                // items: (ptr, nbytes, request body, invalidate callback or None)
                std::vector<CanonicalItem> v;
                v.reserve(items.size());
                for (py::handle it : items) {
                    py::tuple t = py::reinterpret_borrow<py::tuple>(it);
                    CanonicalItem ci;
                    ci.ptr = t[0].cast<uint64_t>();
                    ci.nbytes = t[1].cast<uint64_t>();
                    std::string b = t[2].cast<py::bytes>();
                    ci.req = decode<RequestCanonicalEvictRequest>(reinterpret_cast<const uint8_t*>(b.data()), b.size());
                    ci.on_invalidate = wrap_cb(py::reinterpret_borrow<py::object>(t[3]));
                    v.push_back(std::move(ci));
                }
                std::vector<CanonicalOutcome> rs;
                {
                    py::gil_scoped_release nogil;
                    rs = self.ag().canonical_evict_batch(v, stream, destructive, max_inflight_bytes);
                }
                py::list out;
                for (const CanonicalOutcome& r : rs)
                    out.append(py::make_tuple(r.ok, r.action, r.object_id, r.did_d2h, r.message, r.hash_lo, r.hash_hi));
                return out;
            },
            py::arg("items"), py::arg("stream"), py::arg("destructive"), py::arg("max_inflight_bytes") = 0)
        .def(
            "canonical_restore",
            [](PyAgent& self, uint64_t oid, uint64_t ptr, uint64_t nbytes, uint64_t stream, bool wait, int cast,
               uint64_t scales_ptr) {
                RestoreOptions ro{cast, scales_ptr, false, false};
                RestoreOutcome r;
                {
                    py::gil_scoped_release nogil;
                    r = self.ag().canonical_restore(oid, ptr, nbytes, stream, wait, ro);
                }
                return py::make_tuple(r.ok, r.message);
            },
            py::arg("object_id"), py::arg("ptr"), py::arg("nbytes"), py::arg("stream"), py::arg("wait"),
            py::arg("cast") = 0, py::arg("scales_ptr") = 0)
        .def("call_raw",
             [](PyAgent& self, int op, py::bytes body) {
                 std::string b = body;
                 std::vector<uint8_t> out;
                 {
                     py::gil_scoped_release nogil;
                     std::vector<uint8_t> in(b.begin(), b.end());
                     Op o = Op(op);
                     // Re-encode through the C++ schema so malformed bodies fail here.
                     std::vector<uint8_t> body2 = reencode_body(o, false, in);
                     Agent& a = self.ag();
                     switch (o) {
#define RAW(OPC, METHOD)                                                                    \
    case Op::OPC:                                                                           \
        out = encode(a.METHOD(decode<OpTypes<Op::OPC>::Request>(body2)));                   \
        break;
                         RAW(kRegisterJob, register_job)
                         RAW(kSealModelVersion, seal)
                         RAW(kGetLatestSealedVersion, latest)
                         RAW(kGetManifest, manifest)
                         RAW(kPullTensor, pull)
                         RAW(kDropCanonicalVersion, drop_version)
                         RAW(kReleaseCanonical, release)
                         RAW(kExportManifest, export_manifest)
                         RAW(kGetJobStats, job_stats)
                         RAW(kCarryForward, carry_forward)
#undef RAW
                         case Op::kGetStats: out = encode(a.daemon_stats()); break;
                         default: throw std::invalid_argument("call_raw: opcode not routed through the agent");
                     }
                 }
                 return py::bytes(reinterpret_cast<const char*>(out.data()), out.size());
             })
        .def("publish_peer_buffer",
             [](PyAgent& self, py::bytes desc_body, int fd) {
                 std::string b = desc_body;
                 auto d = decode<PeerBufferDesc>(reinterpret_cast<const uint8_t*>(b.data()), b.size());
                 py::gil_scoped_release nogil;
                 StatusResponse r = self.ag().publish_peer_buffer(d, fd);
                 return std::make_tuple(r.ok, r.message);
             })
        .def("lookup_peer_buffer",
             [](PyAgent& self, std::string key, uint32_t wait_ms) {
                 int fd = -1;
                 LookupPeerBufferResponse r;
                 {
                     py::gil_scoped_release nogil;
                     r = self.ag().lookup_peer_buffer(key, wait_ms, &fd);
                 }
                 auto body = encode(r.desc);
                 return py::make_tuple(r.found, py::bytes(reinterpret_cast<const char*>(body.data()), body.size()), fd);
             })
        .def("hash_buffer",
             [](PyAgent& self, uint64_t ptr, uint64_t nbytes, uint64_t stream) {
                 uint64_t lo, hi;
                 {
                     py::gil_scoped_release nogil;
                     self.ag().hash_buffer(ptr, nbytes, stream, &lo, &hi);
                 }
                 return py::make_tuple(lo, hi);
             })
        .def("map_arena", [](PyAgent& s, uint64_t arena, uint64_t off) { return s.ag().map_arena(arena, off); })
        .def("stats", [](PyAgent& s) { return stats_dict(s.ag().stats()); })
        .def("summary_string", [](PyAgent& s) { return s.ag().summary_string(); })
        .def("device", [](PyAgent& s) { return s.ag().device(); })
        .def("numa_node", [](PyAgent& s) { return s.ag().numa_node(); })
        .def("rank_id", [](PyAgent& s) { return s.ag().rank_id(); })
        .def("rank_epoch", [](PyAgent& s) { return s.ag().rank_epoch(); })
        .def("pause_heartbeat", [](PyAgent& s, bool p) { s.ag().pause_heartbeat(p); });

    py::class_<DaemonThread>(m, "DaemonThread")
        .def(py::init([](py::kwargs kw) { return new DaemonThread(config_from(kw)); }))
        .def("stop", &DaemonThread::stop)
        .def("inject_io_failures", &DaemonThread::inject_io_failures)
        .def("fake_host_memory", &DaemonThread::fake_host_memory)
        .def("pause_rings", &DaemonThread::pause_rings)
        .def_property_readonly("socket", &DaemonThread::socket);

    py::class_<RawConn>(m, "RawConn")
        .def(py::init<std::string, int, int>(), py::arg("addr"), py::arg("timeout_ms") = 10000,
             py::arg("reply_timeout_ms") = 0)
        .def("call", &RawConn::call, py::arg("op"), py::arg("body"), py::arg("fds") = std::vector<int>{})
        .def("send_bytes", &RawConn::send_bytes)
        .def("close", &RawConn::close);

    // ---- hashing (host oracle) ----
    m.def("ssh_hash", [](py::buffer b) {
        py::buffer_info bi = b.request();
        uint64_t n = uint64_t(bi.size) * uint64_t(bi.itemsize);
        ssh::Object o;
        {
            py::gil_scoped_release nogil;
            o = ssh::host_hash(bi.ptr, n);
        }
        return py::make_tuple(o.lo, o.hi);
    });
    m.def("ssh_hash_ptr", [](uint64_t ptr, uint64_t n) {
        py::gil_scoped_release nogil;
        ssh::Object o = ssh::host_hash(reinterpret_cast<const void*>(ptr), n);
        return std::make_tuple(o.lo, o.hi);
    });
    m.def("ssh_digests", [](py::buffer b) {
        py::buffer_info bi = b.request();
        uint64_t n = uint64_t(bi.size) * uint64_t(bi.itemsize);
        std::vector<uint64_t> d(ssh::num_chunks(n));
        ssh::host_chunk_digests(bi.ptr, n, d.data());
        return d;
    });
    m.def("ssh_fold", [](std::vector<uint64_t> d, uint64_t nbytes) {
        ssh::Object o = ssh::fold_digests(d.data(), d.size(), nbytes);
        return py::make_tuple(o.lo, o.hi);
    });
    m.def("fnv1a64", [](py::bytes b) {
        std::string s = b;
        return fnv1a64(s.data(), s.size());
    });
    m.def("fnv2", [](py::bytes b) {
        std::string s = b;
        uint64_t lo, hi;
        fnv2_hash(s.data(), s.size(), &lo, &hi);
        return py::make_tuple(lo, hi);
    });

    // ---- wire ----
    m.def("reencode", [](int op, bool response, py::bytes body) {
        std::string b = body;
        auto out = reencode_body(Op(op), response, std::vector<uint8_t>(b.begin(), b.end()));
        return py::bytes(reinterpret_cast<const char*>(out.data()), out.size());
    });
    m.def("op_name", [](int op) { return std::string(op_name(Op(op))); });
    m.def("parse_config", [](std::string text) {
        DaemonConfig c = parse_config(text);
        py::dict d;
        d["socket_path"] = c.socket_path;
        d["heartbeat_timeout_ms"] = c.heartbeat_timeout_ms;
        d["allocation_granularity_bytes"] = c.allocation_granularity_bytes;
        d["registration_chunk_bytes"] = c.registration_chunk_bytes;
        py::list arenas;
        for (auto& a : c.per_numa) {
            py::dict ad;
            ad["numa_node"] = a.numa_node;
            ad["size_bytes"] = a.size_bytes;
            ad["overflow_bytes"] = a.overflow_bytes;
            py::list w;
            for (auto& g : a.gpu_windows) w.append(py::make_tuple(g.gpu, g.size_bytes));
            ad["gpu_windows"] = w;
            arenas.append(ad);
        }
        d["per_numa"] = arenas;
        d["drain_target"] = std::string(drain_target_name(c.drain_target));
        d["drain_on_d2h_complete"] = c.drain_on_d2h_complete;
        d["thresholds"] = py::make_tuple(c.normal_threshold, c.priority_threshold, c.aggressive_threshold);
        d["nvme_enabled"] = c.nvme_enabled;
        d["nvme_path"] = c.nvme_path;
        d["nvme_io_engine"] = c.nvme_io_engine;
        d["nvme_direct_io"] = c.nvme_direct_io;
        d["nvme_stripe_count"] = c.nvme_stripe_count;
        d["nvme_block_bytes"] = c.nvme_block_bytes;
        d["nvme_queue_depth"] = c.nvme_queue_depth;
        d["nvme_stripe_dirs"] = c.nvme_stripe_dirs;
        d["dedup_default_mode"] = c.v2_dedup_default_mode;
        d["creating_policy"] = c.v2_creating_policy;
        d["retain_sealed_versions"] = c.v2_retain_sealed_versions;
        d["persist_dir"] = c.v2_persist_dir;
        d["accepted_settings"] = c.accepted_settings;
        d["job_quota_overrides"] = c.v2_job_quota_overrides;
        d["default_transport"] = c.v2_default_transport;
        d["fallback_transport"] = c.v2_fallback_transport;
        d["control_tcp_port"] = c.v2_control_tcp_port;
        d["quota_max_pinned_bytes"] = c.v2_quota_max_pinned_bytes;
        d["quota_max_inflight_export_bytes"] = c.v2_quota_max_inflight_export_bytes;
        d["pageable_limit_bytes"] = c.pageable_limit_bytes;
        d["agent_options"] = c.agent_options;
        return d;
    });
    m.def("parse_size", &parse_size);
    m.def("metric_names", [] {
        std::vector<std::string> v;
        for (int i = 0; i < int(M::kCount); ++i) v.push_back(metric_name(M(i)));
        return v;
    });

    // ---- raw kernel launchers (tests, benchmarks, fabric layer) ----
    m.def("kernel_launch_count", &kern::launch_count);
    m.def(
        "kernel_timing_enable",
        [](int device, uint32_t capacity) {
            cudaError_t e = kern::timing_enable(device, capacity);
            if (e != cudaSuccess) throw std::runtime_error(std::string("timing_enable: ") + cudaGetErrorString(e));
        },
        py::arg("device"), py::arg("capacity") = 4096);
    m.def("kernel_timing_disable", &kern::timing_disable);
    m.def(
        "kernel_timings",
        [](int device, uint64_t since) {
            uint64_t next = 0;
            std::vector<kern::StampRecord> recs = kern::timing_read(device, since, &next);
            py::list out;
            for (const kern::StampRecord& r : recs) {
                py::dict d;
                d["seq"] = r.seq;
                d["kernel"] = kern::kernel_name(r.kernel);
                d["bytes"] = r.bytes;
                d["ns"] = r.t1 - r.t0;
                d["t0"] = r.t0;
                out.append(d);
            }
            return py::make_tuple(out, next);
        },
        py::arg("device"), py::arg("since") = 0);
    m.def("cuda_available", [] {
        int n = 0;
        return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
    });
    m.def("k_evict_hash", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t dig, uint64_t stream, int ctas) {
        check(kern::evict_hash(reinterpret_cast<void*>(src), reinterpret_cast<void*>(dst), n,
                               reinterpret_cast<uint64_t*>(dig), reinterpret_cast<cudaStream_t>(stream), ctas),
              "evict_hash");
    });
    m.def("k_restore_cast", [](uint64_t src, uint64_t dst, uint64_t n, int cast, uint64_t scales, uint64_t expect,
                               uint64_t mismatch, uint64_t stream, int ctas) {
        check(kern::restore_cast(reinterpret_cast<void*>(src), reinterpret_cast<void*>(dst), n, kern::Cast(cast),
                                 reinterpret_cast<float*>(scales), reinterpret_cast<const uint64_t*>(expect),
                                 reinterpret_cast<uint32_t*>(mismatch), reinterpret_cast<cudaStream_t>(stream), ctas),
              "restore_cast");
    });
    m.def("k_evict_bulk", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t dig, uint64_t err, uint64_t stream,
                             int ctas) {
        check(kern::evict_bulk(reinterpret_cast<void*>(src), reinterpret_cast<void*>(dst), n,
                               reinterpret_cast<uint64_t*>(dig), reinterpret_cast<uint32_t*>(err),
                               reinterpret_cast<cudaStream_t>(stream), ctas),
              "evict_bulk");
    });
    m.def("k_restore_bulk", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t err, uint64_t stream, int ctas) {
        check(kern::restore_bulk(reinterpret_cast<void*>(src), reinterpret_cast<void*>(dst), n,
                                 reinterpret_cast<uint32_t*>(err), reinterpret_cast<cudaStream_t>(stream), ctas),
              "restore_bulk");
    });
    m.def("k_hash_onepass", [](uint64_t src, uint64_t n, uint64_t dig, uint64_t stream, int ctas) {
        check(kern::hash_onepass(reinterpret_cast<void*>(src), n, reinterpret_cast<uint64_t*>(dig),
                                 reinterpret_cast<cudaStream_t>(stream), ctas),
              "hash_onepass");
    });
    m.def("k_hash_device", [](uint64_t src, uint64_t n, uint64_t dig, uint64_t stream, int ctas) {
        check(kern::hash_device(reinterpret_cast<void*>(src), n, reinterpret_cast<uint64_t*>(dig),
                                reinterpret_cast<cudaStream_t>(stream), ctas),
              "hash_device");
    });
    m.def("k_fold_digests", [](uint64_t dig, uint64_t n, uint64_t nbytes, uint64_t out, uint64_t stream) {
        check(kern::fold_digests(reinterpret_cast<const uint64_t*>(dig), n, nbytes, reinterpret_cast<uint64_t*>(out),
                                 reinterpret_cast<cudaStream_t>(stream)),
              "fold_digests");
    });
    m.def("k_verify_peer", [](uint64_t local, uint64_t peer, uint64_t n, uint64_t dig, uint64_t mismatch,
                              uint64_t stream, int ctas) {
        check(kern::verify_peer(reinterpret_cast<void*>(local), reinterpret_cast<void*>(peer), n,
                                reinterpret_cast<uint64_t*>(dig), reinterpret_cast<uint32_t*>(mismatch),
                                reinterpret_cast<cudaStream_t>(stream), ctas),
              "verify_peer");
    });
    m.def("k_quant_fp8", [](uint64_t src, uint64_t dst, uint64_t scales, uint64_t nelem, uint64_t stream, int ctas) {
        check(kern::quant_fp8_block(reinterpret_cast<void*>(src), reinterpret_cast<void*>(dst),
                                    reinterpret_cast<float*>(scales), nelem, reinterpret_cast<cudaStream_t>(stream),
                                    ctas),
              "quant_fp8_block");
    });
    m.def("host_register", [](uint64_t ptr, uint64_t n) {
        check(cudaHostRegister(reinterpret_cast<void*>(ptr), n, cudaHostRegisterPortable | cudaHostRegisterMapped),
              "cudaHostRegister");
        void* dev = nullptr;
        check(cudaHostGetDevicePointer(&dev, reinterpret_cast<void*>(ptr), 0), "cudaHostGetDevicePointer");
        return reinterpret_cast<uint64_t>(dev);
    });
    // zbf16 host reference codec (tests, tools)
    m.def("zbf16_encode", [](py::buffer b) -> py::object {
        py::buffer_info i = b.request();
        const uint64_t n = uint64_t(i.size) * uint64_t(i.itemsize);
        std::string out(n, '\0');
        bool ok;
        {
            py::gil_scoped_release nogil;
            ok = zbf16::encode_object(static_cast<const uint8_t*>(i.ptr), n, reinterpret_cast<uint8_t*>(&out[0]));
        }
        if (!ok) return py::none();
        return py::bytes(out);
    });
    m.def("zbf16_decode", [](py::bytes coded) {
        std::string in = coded;
        std::string out(in.size(), '\0');
        if (!zbf16::decode_object(reinterpret_cast<const uint8_t*>(in.data()), in.size(),
                                  reinterpret_cast<uint8_t*>(&out[0])))
            throw std::runtime_error("malformed zbf16 object");
        return py::bytes(out);
    });
    // The daemon's export decoder (allocation-free chunk decoding) over bytes
    // [off, off + n) of a coded object: fmt 1 = zbf16, 2 = zf32.
    m.def("zcoded_decode_range", [](int fmt, py::bytes coded, uint64_t off, uint64_t n) {
        std::string in = coded;
        if (off > in.size()) throw std::runtime_error("offset beyond the object");
        std::string out(n, '\0');
        std::vector<uint32_t> keys;
        if (!zbf16::decode_range(zbf16::Coding(fmt), reinterpret_cast<const uint8_t*>(in.data()) + off, in.size(), off,
                                 n, reinterpret_cast<uint8_t*>(&out[0]), keys))
            throw std::runtime_error("malformed coded range");
        return py::bytes(out);
    });
    m.def("zbf16_coded_bytes", [](py::bytes coded) {
        std::string in = coded;
        return zbf16::coded_bytes(reinterpret_cast<const uint8_t*>(in.data()), in.size());
    });
    m.def("k_zscan", [](uint64_t src, uint64_t n, uint64_t ebase, uint64_t fail, uint64_t stream, int ctas) {
        check(kern::zscan(reinterpret_cast<const void*>(src), n, reinterpret_cast<uint8_t*>(ebase),
                          reinterpret_cast<uint32_t*>(fail), reinterpret_cast<cudaStream_t>(stream), ctas),
              "zscan");
    });
    m.def("k_evict_z", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t ebase, uint64_t dig, uint64_t stream,
                          int ctas) {
        check(kern::evict_z(reinterpret_cast<const void*>(src), reinterpret_cast<void*>(dst), n,
                            reinterpret_cast<const uint8_t*>(ebase), reinterpret_cast<uint64_t*>(dig),
                            reinterpret_cast<cudaStream_t>(stream), ctas),
              "evict_z");
    });
    m.def("k_restore_z", [](uint64_t src, uint64_t dst, uint64_t n, int cast, uint64_t scales, uint64_t expect,
                            uint64_t mismatch, uint64_t stream, int ctas) {
        check(kern::restore_z(reinterpret_cast<const void*>(src), reinterpret_cast<void*>(dst), n, kern::Cast(cast),
                              reinterpret_cast<float*>(scales), reinterpret_cast<const uint64_t*>(expect),
                              reinterpret_cast<uint32_t*>(mismatch), reinterpret_cast<cudaStream_t>(stream), ctas),
              "restore_z");
    });
    // zf32 host reference codec (tests, tools)
    m.def("zf32_encode", [](py::buffer b) -> py::object {
        py::buffer_info i = b.request();
        const uint64_t n = uint64_t(i.size) * uint64_t(i.itemsize);
        std::string out(n, '\0');
        bool ok;
        {
            py::gil_scoped_release nogil;
            ok = zf32::encode_object(static_cast<const uint8_t*>(i.ptr), n, reinterpret_cast<uint8_t*>(&out[0]));
        }
        if (!ok) return py::none();
        return py::bytes(out);
    });
    m.def("zf32_decode", [](py::bytes coded) {
        std::string in = coded;
        std::string out(in.size(), '\0');
        if (!zf32::decode_object(reinterpret_cast<const uint8_t*>(in.data()), in.size(),
                                 reinterpret_cast<uint8_t*>(&out[0])))
            throw std::runtime_error("malformed zf32 object");
        return py::bytes(out);
    });
    m.def("zf32_coded_bytes", [](py::bytes coded) {
        std::string in = coded;
        return zf32::coded_bytes(reinterpret_cast<const uint8_t*>(in.data()), in.size());
    });
    m.def("k_zscan_f32", [](uint64_t src, uint64_t n, uint64_t ebase, uint64_t fail, uint64_t stream, int ctas,
                            uint64_t max_coded) {
        check(kern::zscan_f32(reinterpret_cast<const void*>(src), n, reinterpret_cast<uint8_t*>(ebase),
                              reinterpret_cast<uint32_t*>(fail), reinterpret_cast<cudaStream_t>(stream), ctas,
                              reinterpret_cast<uint32_t*>(max_coded)),
              "zscan_f32");
    }, py::arg("src"), py::arg("n"), py::arg("ebase"), py::arg("fail"), py::arg("stream"), py::arg("ctas"),
       py::arg("max_coded") = 0);
    m.def("k_evict_zf32", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t ebase, uint64_t stream, int ctas) {
        check(kern::evict_zf32(reinterpret_cast<const void*>(src), reinterpret_cast<void*>(dst), n,
                               reinterpret_cast<const uint8_t*>(ebase), reinterpret_cast<cudaStream_t>(stream), ctas),
              "evict_zf32");
    });
    m.def("k_restore_zf32", [](uint64_t src, uint64_t dst, uint64_t n, uint64_t stream, int ctas) {
        check(kern::restore_zf32(reinterpret_cast<const void*>(src), reinterpret_cast<void*>(dst), n,
                                 reinterpret_cast<cudaStream_t>(stream), ctas),
              "restore_zf32");
    });
    m.def("k_compare_digests", [](uint64_t got, uint64_t expect, uint64_t n, uint64_t mismatch, uint64_t stream) {
        check(kern::compare_digests(reinterpret_cast<const uint64_t*>(got), reinterpret_cast<const uint64_t*>(expect),
                                    n, reinterpret_cast<uint32_t*>(mismatch), reinterpret_cast<cudaStream_t>(stream)),
              "compare_digests");
    });
    m.def("host_unregister", [](uint64_t ptr) { check(cudaHostUnregister(reinterpret_cast<void*>(ptr)), "cudaHostUnregister"); });
    bind_fabric(m);
}
