// YAML-subset loader. Grammar: block mappings ("key: value" / "key:" + nested
// block), block sequences ("- item" / "- key: value" items), scalars, '#'
// comments. Tabs in indentation are rejected. Parsing produces a small Node
// tree; a table of binders then maps dotted paths onto DaemonConfig fields.
#include "config.h"

#include <algorithm>
#include <cctype>
#include <fstream>
#include <functional>
#include <memory>
#include <sstream>
#include <stdexcept>

#include "ofld/log.h"

namespace ofld {

namespace {

struct Node {
    enum Kind { kNull, kScalar, kMap, kSeq } kind = kNull;
    std::string scalar;
    std::vector<std::pair<std::string, std::unique_ptr<Node>>> map;
    std::vector<std::unique_ptr<Node>> seq;
    int line = 0;
    const Node* get(const std::string& k) const {
        for (auto& kv : map)
            if (kv.first == k) return kv.second.get();
        return nullptr;
    }
};

struct Line {
    int indent;
    int no;
    std::string text;
};

[[noreturn]] void fail(int line, const std::string& msg) {
    throw std::runtime_error("config line " + std::to_string(line) + ": " + msg);
}

std::string trim(const std::string& s) {
    size_t b = s.find_first_not_of(" \t\r");
    if (b == std::string::npos) return {};
    size_t e = s.find_last_not_of(" \t\r");
    return s.substr(b, e - b + 1);
}

std::string unquote(const std::string& s) {
    if (s.size() >= 2 && ((s.front() == '"' && s.back() == '"') || (s.front() == '\'' && s.back() == '\'')))
        return s.substr(1, s.size() - 2);
    return s;
}

// Remove a trailing comment: '#' at line start or preceded by whitespace,
// outside quotes.
std::string strip_comment(const std::string& s) {
    char q = 0;
    for (size_t i = 0; i < s.size(); ++i) {
        char c = s[i];
        if (q) {
            if (c == q) q = 0;
        } else if (c == '"' || c == '\'') {
            q = c;
        } else if (c == '#' && (i == 0 || s[i - 1] == ' ' || s[i - 1] == '\t')) {
            return s.substr(0, i);
        }
    }
    return s;
}

std::vector<Line> lex(const std::string& text) {
    std::vector<Line> out;
    std::istringstream in(text);
    std::string raw;
    int no = 0;
    while (std::getline(in, raw)) {
        ++no;
        std::string s = strip_comment(raw);
        if (trim(s).empty()) continue;
        size_t ind = 0;
        while (ind < s.size() && (s[ind] == ' ' || s[ind] == '\t')) {
            if (s[ind] == '\t') fail(no, "tabs are not allowed for indentation");
            ++ind;
        }
        std::string body = s.substr(ind);
        while (!body.empty() && (body.back() == ' ' || body.back() == '\r' || body.back() == '\t'))
            body.pop_back();
        if (body == "---") continue;
        out.push_back({int(ind), no, body});
    }
    return out;
}

class Parser {
 public:
    explicit Parser(std::vector<Line> lines) : L_(std::move(lines)) {}
    std::unique_ptr<Node> parse_root() {
        if (L_.empty()) {
            auto n = std::make_unique<Node>();
            n->kind = Node::kMap;
            return n;
        }
        auto n = block(L_[0].indent);
        if (i_ < L_.size()) fail(L_[i_].no, "unexpected indentation");
        return n;
    }

 private:
    static bool is_item(const std::string& t) { return t == "-" || t.rfind("- ", 0) == 0; }

    std::unique_ptr<Node> block(int indent) {
        if (is_item(L_[i_].text)) return seq(indent);
        return mapping(indent);
    }

    std::unique_ptr<Node> scalar_node(const std::string& v, int line) {
        auto n = std::make_unique<Node>();
        n->kind = Node::kScalar;
        n->scalar = unquote(v);
        n->line = line;
        return n;
    }

    // Value after "key:" -- inline scalar, inline [a, b] list, or nested block.
    std::unique_ptr<Node> value(const std::string& v, int indent, int line) {
        if (!v.empty()) {
            if (v.front() == '[' && v.back() == ']') {
                auto n = std::make_unique<Node>();
                n->kind = Node::kSeq;
                n->line = line;
                std::stringstream ss(v.substr(1, v.size() - 2));
                std::string item;
                while (std::getline(ss, item, ','))
                    if (!trim(item).empty()) n->seq.push_back(scalar_node(trim(item), line));
                return n;
            }
            return scalar_node(v, line);
        }
        if (i_ < L_.size() && (L_[i_].indent > indent || (L_[i_].indent == indent && is_item(L_[i_].text))))
            return block(L_[i_].indent);
        auto n = std::make_unique<Node>();
        n->line = line;
        return n;
    }

    std::unique_ptr<Node> mapping(int indent) {
        auto n = std::make_unique<Node>();
        n->kind = Node::kMap;
        n->line = L_[i_].no;
        while (i_ < L_.size() && L_[i_].indent == indent && !is_item(L_[i_].text)) {
            const Line& ln = L_[i_];
            size_t c = ln.text.find(':');
            if (c == std::string::npos) fail(ln.no, "expected 'key: value'");
            std::string k = trim(ln.text.substr(0, c));
            std::string v = trim(ln.text.substr(c + 1));
            ++i_;
            n->map.emplace_back(unquote(k), value(v, indent, ln.no));
        }
        if (i_ < L_.size() && L_[i_].indent > indent) fail(L_[i_].no, "bad indentation");
        return n;
    }

    std::unique_ptr<Node> seq(int indent) {
        auto n = std::make_unique<Node>();
        n->kind = Node::kSeq;
        n->line = L_[i_].no;
        while (i_ < L_.size() && L_[i_].indent == indent && is_item(L_[i_].text)) {
            Line& ln = L_[i_];
            size_t c = 1;
            while (c < ln.text.size() && ln.text[c] == ' ') ++c;
            std::string rest = ln.text.substr(c);
            if (rest.empty()) {
                ++i_;
                if (i_ < L_.size() && L_[i_].indent > indent)
                    n->seq.push_back(block(L_[i_].indent));
                else
                    n->seq.push_back(std::make_unique<Node>());
                continue;
            }
            size_t colon = rest.find(':');
            bool is_kv = colon != std::string::npos && rest.front() != '"' && rest.front() != '\'';
            if (!is_kv) {
                n->seq.push_back(scalar_node(rest, ln.no));
                ++i_;
                continue;
            }
            // "- key: value": the item is a mapping whose first key sits at
            // indent + c; rewrite the line in place and parse a mapping there.
            ln.indent = indent + int(c);
            ln.text = rest;
            n->seq.push_back(mapping(ln.indent));
        }
        return n;
    }

    std::vector<Line> L_;
    size_t i_ = 0;
};

std::string lower(std::string s) {
    std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return std::tolower(c); });
    return s;
}

const std::string& need_scalar(const Node& n, const std::string& key) {
    if (n.kind != Node::kScalar) fail(n.line, "expected a scalar for '" + key + "'");
    return n.scalar;
}

uint64_t as_u64(const Node& n, const std::string& key) {
    const std::string& s = need_scalar(n, key);
    char* end = nullptr;
    errno = 0;
    long long v = std::strtoll(s.c_str(), &end, 10);
    if (*end != '\0' || v < 0 || errno != 0) fail(n.line, "invalid integer '" + s + "' for " + key);
    return uint64_t(v);
}
double as_double(const Node& n, const std::string& key) {
    const std::string& s = need_scalar(n, key);
    char* end = nullptr;
    double v = std::strtod(s.c_str(), &end);
    if (*end != '\0') fail(n.line, "invalid number '" + s + "' for " + key);
    return v;
}
bool as_bool(const Node& n, const std::string& key) {
    std::string s = lower(need_scalar(n, key));
    if (s == "true" || s == "yes" || s == "on" || s == "1") return true;
    if (s == "false" || s == "no" || s == "off" || s == "0") return false;
    fail(n.line, "invalid bool '" + s + "' for " + key);
}
uint64_t as_size(const Node& n, const std::string& key) {
    try {
        return parse_size(need_scalar(n, key));
    } catch (const std::exception& e) {
        fail(n.line, std::string(e.what()) + " for " + key);
    }
}

uint32_t dedup_mode_of(const std::string& s) {
    if (s == "disabled") return 0;
    if (s == "semantic_trusted") return 1;
    if (s == "hash_verified") return 2;
    if (s == "sampled_hash") return 3;
    if (s == "device_hash_verified") return 4;
    if (s == "p2p_verified") return 5;
    return 1;
}
uint32_t transport_of(const std::string& s) {
    if (s == "tcp") return 1;
    if (s == "file") return 2;
    if (s == "libfabric" || s == "libfabric_send") return 3;
    if (s == "libfabric_rdma_read") return 4;
    if (s == "libfabric_rdma_write") return 5;
    return 1;
}

using Binder = std::function<void(DaemonConfig&, const Node&, const std::string&)>;

const std::map<std::string, Binder>& binders() {
    static const std::map<std::string, Binder> b = {
        // daemon
        {"daemon.socket_path", [](DaemonConfig& c, const Node& n, const std::string& k) { c.socket_path = need_scalar(n, k); }},
        {"daemon.control_shm_name", [](DaemonConfig& c, const Node& n, const std::string& k) { c.control_shm_name = need_scalar(n, k); }},
        {"daemon.heartbeat_timeout_ms", [](DaemonConfig& c, const Node& n, const std::string& k) { c.heartbeat_timeout_ms = as_u64(n, k); }},
        {"daemon.completion_ring_max_ranks", [](DaemonConfig& c, const Node& n, const std::string& k) { c.completion_ring_max_ranks = uint32_t(as_u64(n, k)); }},
        {"daemon.completion_ring_capacity", [](DaemonConfig& c, const Node& n, const std::string& k) { c.completion_ring_capacity = uint32_t(as_u64(n, k)); }},
        {"daemon.ring_poll_us", [](DaemonConfig& c, const Node& n, const std::string& k) { c.ring_poll_us = uint32_t(as_u64(n, k)); }},
        // arenas (per_numa handled separately)
        {"arenas.registration_policy", [](DaemonConfig& c, const Node& n, const std::string& k) { c.registration_policy = need_scalar(n, k); }},
        {"arenas.registration_chunk_mb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.registration_chunk_bytes = as_u64(n, k) << 20; }},
        {"arenas.allocation_granularity_mb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.allocation_granularity_bytes = as_u64(n, k) << 20; }},
        {"arenas.first_touch", [](DaemonConfig& c, const Node& n, const std::string& k) { c.numa_first_touch = as_bool(n, k); }},
        {"arenas.huge_pages", [](DaemonConfig& c, const Node& n, const std::string& k) { c.arena_huge_pages = as_bool(n, k); }},
        // drain_policy
        {"drain_policy.target_tier", [](DaemonConfig& c, const Node& n, const std::string& k) {
             std::string s = need_scalar(n, k);
             if (s == "pageable_then_nvme") c.drain_target = DrainTarget::kPageableThenNvme;
             else if (s == "pageable") c.drain_target = DrainTarget::kPageableOnly;
             else if (s == "nvme") c.drain_target = DrainTarget::kNvmeOnly;
             else fail(n.line, "unknown target_tier '" + s + "'");
         }},
        {"drain_policy.drain_on_d2h_complete", [](DaemonConfig& c, const Node& n, const std::string& k) { c.drain_on_d2h_complete = as_bool(n, k); }},
        {"drain_policy.normal_threshold", [](DaemonConfig& c, const Node& n, const std::string& k) { c.normal_threshold = as_double(n, k); }},
        {"drain_policy.priority_threshold", [](DaemonConfig& c, const Node& n, const std::string& k) { c.priority_threshold = as_double(n, k); }},
        {"drain_policy.aggressive_threshold", [](DaemonConfig& c, const Node& n, const std::string& k) { c.aggressive_threshold = as_double(n, k); }},
        {"drain_policy.pageable_limit_gb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.pageable_limit_bytes = as_u64(n, k) << 30; }},
        {"drain_policy.drain_workers", [](DaemonConfig& c, const Node& n, const std::string& k) { c.drain_workers = uint32_t(as_u64(n, k)); }},
        {"drain_policy.readback_workers", [](DaemonConfig& c, const Node& n, const std::string& k) { c.readback_workers = uint32_t(as_u64(n, k)); }},
        {"drain_policy.pageable_pool_mb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.pageable_pool_bytes = as_u64(n, k) << 20; }},
        {"drain_policy.copy_threads", [](DaemonConfig& c, const Node& n, const std::string& k) { c.copy_threads = uint32_t(as_u64(n, k)); }},
        // nvme
        {"nvme.enabled", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_enabled = as_bool(n, k); }},
        {"nvme.path", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_path = need_scalar(n, k); }},
        {"nvme.io_engine", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_io_engine = need_scalar(n, k); }},
        {"nvme.direct_io", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_direct_io = as_bool(n, k); }},
        {"nvme.stripe", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_stripe = as_bool(n, k); }},
        {"nvme.stripe_count", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_stripe_count = uint32_t(as_u64(n, k)); }},
        {"nvme.block_mb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_block_bytes = as_u64(n, k) << 20; }},
        {"nvme.queue_depth", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_queue_depth = uint32_t(as_u64(n, k)); }},
        {"nvme.workers", [](DaemonConfig& c, const Node& n, const std::string& k) { c.nvme_workers = uint32_t(as_u64(n, k)); }},
        {"nvme.stripe_dirs", [](DaemonConfig& c, const Node& n, const std::string& k) {
             if (n.kind != Node::kSeq) fail(n.line, "nvme.stripe_dirs must be a list");
             c.nvme_stripe_dirs.clear();
             for (auto& it : n.seq) c.nvme_stripe_dirs.push_back(need_scalar(*it, k));
         }},
        // python_api
        {"python_api.default_invalidate", [](DaemonConfig& c, const Node& n, const std::string& k) { c.default_invalidate = need_scalar(n, k); }},
        {"python_api.require_own_storage", [](DaemonConfig& c, const Node& n, const std::string& k) { c.require_own_storage = as_bool(n, k); }},
        {"python_api.allow_views", [](DaemonConfig& c, const Node& n, const std::string& k) { c.allow_views = as_bool(n, k); }},
        {"python_api.unsafe_autograd", [](DaemonConfig& c, const Node& n, const std::string& k) { c.unsafe_autograd = as_bool(n, k); }},
        // manager
        {"manager.enable_canonical_store", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_enable_canonical_store = as_bool(n, k); }},
        {"manager.enable_manifests", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_enable_manifests = as_bool(n, k); }},
        {"manager.enable_rollout_export", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_enable_rollout_export = as_bool(n, k); }},
        {"manager.control_tcp_port", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_control_tcp_port = uint32_t(as_u64(n, k)); }},
        {"manager.daemon_socket", [](DaemonConfig& c, const Node& n, const std::string& k) {
             std::string s = need_scalar(n, k);
             c.socket_path = s.rfind("unix://", 0) == 0 ? s.substr(7) : s;
         }},
        // namespace
        {"namespace.default_tenant_id", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_default_tenant_id = as_u64(n, k); }},
        {"namespace.require_job_registration", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_require_job_registration = as_bool(n, k); }},
        {"namespace.include_launch_epoch", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_include_launch_epoch = as_bool(n, k); }},
        {"namespace.job_name_is_identity", [](DaemonConfig&, const Node&, const std::string&) {}},
        // canonical_store
        {"canonical_store.dedup_default_mode", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_dedup_default_mode = dedup_mode_of(need_scalar(n, k)); }},
        {"canonical_store.cross_job_dedup", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_cross_job_dedup = as_bool(n, k); }},
        {"canonical_store.creating_policy", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_creating_policy = need_scalar(n, k) == "duplicate_candidate_on_pressure" ? 1 : 0; }},
        {"canonical_store.duplicate_candidate_gpu_pressure_threshold", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_duplicate_candidate_gpu_pressure_threshold = as_double(n, k); }},
        {"canonical_store.sampled_hash_bytes_per_gib", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_sampled_hash_bytes_per_gib = as_u64(n, k); }},
        {"canonical_store.object_table_capacity", [](DaemonConfig&, const Node&, const std::string&) {}},
        {"canonical_store.manifest_table_capacity", [](DaemonConfig&, const Node&, const std::string&) {}},
        // manifest
        {"manifest.seal_requires_all_objects_valid", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_seal_requires_all_objects_valid = as_bool(n, k); }},
        {"manifest.retain_sealed_versions", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_retain_sealed_versions = uint32_t(as_u64(n, k)); }},
        {"manifest.persist_dir", [](DaemonConfig& c, const Node& n, const std::string&) { c.v2_persist_dir = n.scalar; }},
        {"manifest.allow_sealed_version_mutation", [](DaemonConfig&, const Node&, const std::string&) {}},
        {"manifest.latest_pointer_update", [](DaemonConfig&, const Node&, const std::string&) {}},
        // export
        {"export.default_transport", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_default_transport = transport_of(need_scalar(n, k)); }},
        {"export.fallback_transport", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_fallback_transport = transport_of(need_scalar(n, k)); }},
        {"export.use_dedicated_export_buffers", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_use_dedicated_export_buffers = as_bool(n, k); }},
        {"export.require_export_refcount", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_require_export_refcount = as_bool(n, k); }},
        {"export.max_concurrent_exports_per_job", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_max_concurrent_exports_per_job = uint32_t(as_u64(n, k)); }},
        {"export.chunk_mb", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_export_chunk_bytes = as_u64(n, k) << 20; }},
        {"export.export_buffer_pool_bytes", [](DaemonConfig&, const Node&, const std::string&) {}},
        {"export.allow_direct_rdma_read_from_object_slot", [](DaemonConfig&, const Node&, const std::string&) {}},
        // quotas
        {"quotas.default.max_pinned_bytes", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_quota_max_pinned_bytes = as_size(n, k); }},
        {"quotas.default.max_pageable_bytes", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_quota_max_pageable_bytes = as_size(n, k); }},
        {"quotas.default.max_nvme_bytes", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_quota_max_nvme_bytes = as_size(n, k); }},
        {"quotas.default.max_inflight_d2h_bytes", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_quota_max_inflight_d2h_bytes = as_size(n, k); }},
        {"quotas.default.max_inflight_export_bytes", [](DaemonConfig& c, const Node& n, const std::string& k) { c.v2_quota_max_inflight_export_bytes = as_size(n, k); }},
        {"quotas.default.priority", [](DaemonConfig&, const Node&, const std::string&) {}},
    };
    return b;
}

const char* kKnownSections[] = {"daemon", "arenas", "drain_policy", "nvme", "python_api", "manager",
                                "namespace", "canonical_store", "manifest", "export", "quotas",
                                "roles", "libfabric", "cleanup", "metrics", "nvlink", "kernels"};

void bind_arenas(DaemonConfig& c, const Node& pn) {
    if (pn.kind != Node::kSeq) fail(pn.line, "arenas.per_numa must be a list");
    for (auto& item : pn.seq) {
        if (item->kind != Node::kMap) fail(item->line, "per_numa entry must be a mapping");
        NumaArena a;
        for (auto& kv : item->map) {
            const std::string& k = kv.first;
            const Node& v = *kv.second;
            if (k == "numa_node") a.numa_node = uint32_t(as_u64(v, k));
            else if (k == "size_gb") a.size_bytes = as_u64(v, k) << 30;
            else if (k == "size_mb") a.size_bytes = as_u64(v, k) << 20;
            else if (k == "overflow_gb") a.overflow_bytes = as_u64(v, k) << 30;
            else if (k == "overflow_mb") a.overflow_bytes = as_u64(v, k) << 20;
            else if (k == "gpu_windows") {
                if (v.kind != Node::kSeq) fail(v.line, "gpu_windows must be a list");
                for (auto& w : v.seq) {
                    if (w->kind != Node::kMap) fail(w->line, "gpu_windows entry must be a mapping");
                    GpuWindow gw;
                    for (auto& wkv : w->map) {
                        if (wkv.first == "gpu") gw.gpu = uint32_t(as_u64(*wkv.second, "gpu"));
                        else if (wkv.first == "size_gb") gw.size_bytes = as_u64(*wkv.second, "size_gb") << 30;
                        else if (wkv.first == "size_mb") gw.size_bytes = as_u64(*wkv.second, "size_mb") << 20;
                        else LOG_WARN("config", "unknown gpu_windows.%s (ignored)", wkv.first.c_str());
                    }
                    a.gpu_windows.push_back(gw);
                }
            } else {
                LOG_WARN("config", "unknown per_numa.%s (ignored)", k.c_str());
            }
        }
        c.per_numa.push_back(std::move(a));
    }
}

void walk(DaemonConfig& c, const Node& n, const std::string& path) {
    for (auto& kv : n.map) {
        std::string p = path.empty() ? kv.first : path + "." + kv.first;
        const Node& v = *kv.second;
        if (p == "arenas.per_numa") {
            bind_arenas(c, v);
            continue;
        }
        if (path == "nvlink" || path == "kernels" || p.rfind("nvlink.", 0) == 0 || p.rfind("kernels.", 0) == 0) {
            if (v.kind == Node::kScalar) c.agent_options[p] = v.scalar;
            else if (v.kind == Node::kMap) walk(c, v, p);
            continue;
        }
        if (p == "quotas.per_job_overrides") {
            for (auto& job : v.map) {
                for (auto& q : job.second->map) {
                    static const char* kKeys[] = {"max_pinned_bytes", "max_pageable_bytes", "max_nvme_bytes",
                                                  "max_inflight_d2h_bytes", "max_inflight_export_bytes"};
                    bool ok = false;
                    for (const char* k : kKeys) ok |= q.first == k;
                    if (!ok) {
                        LOG_WARN("config", "unknown key %s.%s.%s (ignored)", p.c_str(), job.first.c_str(),
                                 q.first.c_str());
                        continue;
                    }
                    c.v2_job_quota_overrides[job.first][q.first] =
                        as_size(*q.second, p + "." + job.first + "." + q.first);
                }
            }
            continue;  // `{}` (no overrides) parses as an empty map or scalar
        }
        if (p.rfind("roles.", 0) == 0 || p.rfind("libfabric.", 0) == 0 || p.rfind("cleanup.", 0) == 0 ||
            p == "metrics.labels" || p.rfind("metrics.labels.", 0) == 0) {
            if (v.kind == Node::kMap) {
                walk(c, v, p);
            } else if (v.kind == Node::kSeq) {
                std::string joined;
                for (auto& e : v.seq) joined += (joined.empty() ? "" : ",") + e->scalar;
                c.accepted_settings[p] = joined;
            } else {
                c.accepted_settings[p] = v.scalar;
            }
            continue;
        }
        auto it = binders().find(p);
        if (it != binders().end()) {
            it->second(c, v, p);
        } else if (v.kind == Node::kMap) {
            walk(c, v, p);
        } else if (path.empty()) {
            bool known = false;
            for (const char* s : kKnownSections) known |= (kv.first == s);
            if (!known) LOG_WARN("config", "unknown top-level key '%s' (ignored)", kv.first.c_str());
        } else {
            LOG_WARN("config", "unknown key %s (ignored)", p.c_str());
        }
    }
}

}  // namespace

uint64_t parse_size(const std::string& s_in) {
    std::string s = trim(s_in);
    char* end = nullptr;
    double v = std::strtod(s.c_str(), &end);
    if (end == s.c_str() || v < 0) throw std::runtime_error("invalid size '" + s_in + "'");
    std::string suf = lower(trim(std::string(end)));
    uint64_t mult = 1;
    if (suf.empty() || suf == "b") mult = 1;
    else if (suf == "k" || suf == "kb" || suf == "kib") mult = 1ull << 10;
    else if (suf == "m" || suf == "mb" || suf == "mib") mult = 1ull << 20;
    else if (suf == "g" || suf == "gb" || suf == "gib") mult = 1ull << 30;
    else if (suf == "t" || suf == "tb" || suf == "tib") mult = 1ull << 40;
    else throw std::runtime_error("unknown size suffix '" + suf + "'");
    return uint64_t(v * double(mult));
}

const char* drain_target_name(DrainTarget t) {
    switch (t) {
        case DrainTarget::kPageableOnly: return "pageable";
        case DrainTarget::kNvmeOnly: return "nvme";
        case DrainTarget::kPageableThenNvme: return "pageable_then_nvme";
    }
    return "unknown";
}

void validate(const DaemonConfig& c) {
    if (c.allocation_granularity_bytes == 0)
        throw std::runtime_error("config: allocation_granularity_mb must be > 0");
    if (c.per_numa.empty()) throw std::runtime_error("config: at least one arenas.per_numa entry required");
    for (const NumaArena& a : c.per_numa) {
        if (a.size_bytes == 0)
            throw std::runtime_error("config: numa_node " + std::to_string(a.numa_node) + " size must be > 0");
        uint64_t need = a.overflow_bytes;
        for (const GpuWindow& w : a.gpu_windows) need += w.size_bytes;
        if (need > a.size_bytes)
            throw std::runtime_error("config: numa_node " + std::to_string(a.numa_node) +
                                     " gpu_windows + overflow (" + std::to_string(need) +
                                     " bytes) exceed arena size (" + std::to_string(a.size_bytes) + " bytes)");
    }
    if (c.normal_threshold > c.priority_threshold || c.priority_threshold > c.aggressive_threshold)
        throw std::runtime_error("config: drain thresholds must be ordered normal <= priority <= aggressive");
}

DaemonConfig parse_config(const std::string& text) {
    Parser p(lex(text));
    std::unique_ptr<Node> root = p.parse_root();
    if (root->kind != Node::kMap) throw std::runtime_error("config: top level must be a mapping");
    DaemonConfig c;
    walk(c, *root, "");
    validate(c);
    return c;
}

DaemonConfig load_config(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("config: cannot open '" + path + "'");
    std::stringstream ss;
    ss << f.rdbuf();
    if (trim(ss.str()).empty()) throw std::runtime_error("config: file '" + path + "' is empty");
    return parse_config(ss.str());
}

DaemonConfig smoke_config(uint64_t arena_bytes, uint32_t numa_node, uint32_t gpu) {
    DaemonConfig c;
    c.allocation_granularity_bytes = 2ull << 20;
    c.registration_chunk_bytes = std::min<uint64_t>(arena_bytes, 512ull << 20);
    c.nvme_enabled = false;
    c.drain_workers = 1;
    c.readback_workers = 1;
    c.nvme_workers = 1;
    c.drain_target = DrainTarget::kPageableOnly;
    NumaArena a;
    a.numa_node = numa_node;
    a.size_bytes = arena_bytes;
    uint64_t overflow = std::max<uint64_t>(arena_bytes / 8, 16ull << 20);
    if (overflow >= arena_bytes) overflow = arena_bytes / 2;
    a.gpu_windows.push_back(GpuWindow{gpu, arena_bytes - overflow});
    a.overflow_bytes = overflow;
    c.per_numa.push_back(a);
    return c;
}

}  // namespace ofld
