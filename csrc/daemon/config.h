// Daemon configuration: defaults, the YAML-subset loader and validation.
//
// Every key of StateSpectre's config files is accepted with the same meaning
// (reference: src/daemon/config.h:35-137, config.cpp:399-679), so existing
// config/*.yaml files load unchanged. Keys this runtime adds:
//   drain_policy.pageable_limit_gb    pageable tier budget before NVMe spill
//   drain_policy.readback_workers     readback thread count
//   nvme.workers                      pwrite engine worker threads
//   nvlink.*, kernels.*               forwarded to rank agents via GetStats keys
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ofld {

enum class DrainTarget { kPageableOnly, kNvmeOnly, kPageableThenNvme };

struct GpuWindow {
    uint32_t gpu = 0;
    uint64_t size_bytes = 0;
};

struct NumaArena {
    uint32_t numa_node = 0;
    uint64_t size_bytes = 0;
    std::vector<GpuWindow> gpu_windows;
    uint64_t overflow_bytes = 0;
};

struct DaemonConfig {
    // daemon
    std::string socket_path = "/tmp/state_spectre.sock";
    std::string control_shm_name = "/state_spectre_ctrl";
    uint64_t heartbeat_timeout_ms = 5000;
    uint32_t completion_ring_max_ranks = 64;
    uint32_t completion_ring_capacity = 1024;
    uint32_t ring_poll_us = 50;

    // arenas
    std::string registration_policy = "lazy_chunked";
    uint64_t registration_chunk_bytes = 512ull << 20;
    uint64_t allocation_granularity_bytes = 16ull << 20;
    std::vector<NumaArena> per_numa;
    bool numa_first_touch = true;
    // Ask for transparent huge pages on the arena mappings (madvise): 2 MiB
    // pages cut IOMMU translation misses of GPU DMA into host memory.
    bool arena_huge_pages = true;

    // drain_policy
    DrainTarget drain_target = DrainTarget::kPageableThenNvme;
    bool drain_on_d2h_complete = true;
    double normal_threshold = 0.60;
    double priority_threshold = 0.80;
    double aggressive_threshold = 0.95;
    uint64_t pageable_limit_bytes = 0;  // 0 = unlimited
    // 4 + 4 workers and 8 pool threads: a 40 GB KV cache cycling 20 GB per
    // iteration through a 24 GB window restored at 52.0 GB/s with 2 + 2 and 4
    // pool threads, 58.7 GB/s (the evict rate) with these.
    uint32_t drain_workers = 4;
    uint32_t readback_workers = 4;
    // Freed pageable buffers kept for reuse (bytes), so tensors that cycle
    // through the pageable tier copy into memory that is already faulted in.
    uint64_t pageable_pool_bytes = 4ull << 30;
    // Pool threads that share pinned <-> pageable copies (1 MiB pieces) with
    // the drain and readback workers.
    uint32_t copy_threads = 8;

    // nvme
    bool nvme_enabled = true;
    std::string nvme_path = "/nvme/state_spectre";
    std::string nvme_io_engine = "io_uring";
    bool nvme_direct_io = true;
    bool nvme_stripe = true;
    uint32_t nvme_stripe_count = 4;
    uint64_t nvme_block_bytes = 16ull << 20;
    uint32_t nvme_queue_depth = 8;
    std::vector<std::string> nvme_stripe_dirs;
    uint32_t nvme_workers = 2;

    // python_api (rank-side policy, informational for the daemon)
    std::string default_invalidate = "set_empty";
    bool require_own_storage = true;
    bool allow_views = false;
    bool unsafe_autograd = false;

    // v2 manager / namespace / canonical_store / manifest / export / quotas
    bool v2_enable_canonical_store = true;
    bool v2_enable_manifests = true;
    bool v2_enable_rollout_export = true;
    uint32_t v2_control_tcp_port = 0;
    uint64_t v2_default_tenant_id = 0;
    bool v2_require_job_registration = true;
    bool v2_include_launch_epoch = true;
    uint32_t v2_dedup_default_mode = 1;
    bool v2_cross_job_dedup = false;
    uint32_t v2_creating_policy = 0;
    double v2_duplicate_candidate_gpu_pressure_threshold = 0.90;
    uint64_t v2_sampled_hash_bytes_per_gib = 1ull << 20;
    bool v2_seal_requires_all_objects_valid = true;
    uint32_t v2_retain_sealed_versions = 4;
    // Directory where sealed versions are made durable (empty: off). A daemon
    // started on the same directory serves them again after a restart.
    std::string v2_persist_dir;
    uint32_t v2_default_transport = 3;
    uint32_t v2_fallback_transport = 1;
    bool v2_use_dedicated_export_buffers = true;
    bool v2_require_export_refcount = true;
    uint32_t v2_max_concurrent_exports_per_job = 8;
    uint64_t v2_export_chunk_bytes = 8ull << 20;
    uint64_t v2_quota_max_pinned_bytes = 0;
    uint64_t v2_quota_max_pageable_bytes = 0;
    uint64_t v2_quota_max_nvme_bytes = 0;
    uint64_t v2_quota_max_inflight_d2h_bytes = 0;
    uint64_t v2_quota_max_inflight_export_bytes = 0;
    // quotas.per_job_overrides: job name -> {max_pinned_bytes, max_pageable_bytes,
    // max_nvme_bytes, max_inflight_d2h_bytes, max_inflight_export_bytes}
    std::map<std::string, std::map<std::string, uint64_t>> v2_job_quota_overrides;
    // Sections StateSpectre's config files carry that this daemon accepts and
    // keeps without acting on them (roles:, libfabric:, cleanup:,
    // metrics.labels), flattened to dotted keys; sequences joined with ','.
    std::map<std::string, std::string> accepted_settings;

    // Sections forwarded verbatim to rank agents (nvlink.*, kernels.*).
    std::map<std::string, std::string> agent_options;
};

// Load a config file (throws std::runtime_error with the offending line).
DaemonConfig load_config(const std::string& path);
// Parse config text (same rules as load_config).
DaemonConfig parse_config(const std::string& text);
// Single-arena config for tests and smoke runs: one GPU window plus overflow
// of max(arena/8, 16 MiB), 2 MiB slots, pageable drain, no NVMe.
DaemonConfig smoke_config(uint64_t arena_bytes, uint32_t numa_node, uint32_t gpu);
// Throws when the arena plan is inconsistent.
void validate(const DaemonConfig& c);
const char* drain_target_name(DrainTarget t);
// Parse "256GiB", "512MiB", "1.5 GB", "4096" into bytes (throws on junk).
uint64_t parse_size(const std::string& s);

}  // namespace ofld
