"""Daemon configuration: the YAML subset, defaults, validation, CLI."""

import os
import subprocess

import pytest

from statespectre_b200._native import bin_path, native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

V1_STYLE = """
daemon:
  socket_path: /tmp/x.sock
  control_shm_name: /ctrl
  heartbeat_timeout_ms: 7000

arenas:
  registration_policy: lazy_chunked
  registration_chunk_mb: 512
  allocation_granularity_mb: 16
  per_numa:
    - numa_node: 0
      size_gb: 384
      gpu_windows:
        - gpu: 0
          size_gb: 80
        - gpu: 1
          size_gb: 80
      overflow_gb: 64   # trailing comment
    - numa_node: 1
      size_gb: 200
      gpu_windows:
        - gpu: 4
          size_gb: 80
      overflow_gb: 64

drain_policy:
  target_tier: pageable_then_nvme
  drain_on_d2h_complete: true
  normal_threshold: 0.60
  priority_threshold: 0.80
  aggressive_threshold: 0.95

nvme:
  enabled: true
  path: /nvme/ss
  io_engine: io_uring
  direct_io: true
  stripe: true
  stripe_dirs:
    - /nvme0/ss
    - /nvme1/ss
"""

V2_STYLE = """
manager:
  daemon_socket: unix:///tmp/y.sock
  enable_canonical_store: true
  control_tcp_port: 7070
namespace:
  default_tenant_id: 3
  job_name_is_identity: false
canonical_store:
  object_table_capacity: 1048576
  dedup_default_mode: hash_verified
  creating_policy: duplicate_candidate_on_pressure
roles:
  rollout_visible_roles:
    - POLICY_ROLLOUT
quotas:
  default:
    max_pinned_bytes: 256GiB
    max_inflight_export_bytes: 1.5 GB
  per_job_overrides: {}
manifest:
  retain_sealed_versions: 6
export:
  default_transport: libfabric_send
  fallback_transport: file
arenas:
  per_numa:
    - numa_node: 0
      size_gb: 8
kernels:
  evict_ctas: 32
nvlink:
  weight_sync: multicast
"""


def test_v1_style_config():
    c = native().parse_config(V1_STYLE)
    assert c["socket_path"] == "/tmp/x.sock"
    assert c["heartbeat_timeout_ms"] == 7000
    assert c["allocation_granularity_bytes"] == 16 << 20
    assert len(c["per_numa"]) == 2
    a0 = c["per_numa"][0]
    assert a0["size_bytes"] == 384 << 30 and a0["overflow_bytes"] == 64 << 30
    assert a0["gpu_windows"] == [(0, 80 << 30), (1, 80 << 30)]
    assert c["per_numa"][1]["gpu_windows"] == [(4, 80 << 30)]
    assert c["drain_target"] == "pageable_then_nvme"
    assert c["thresholds"] == (0.6, 0.8, 0.95)
    assert c["nvme_io_engine"] == "io_uring" and c["nvme_direct_io"]
    assert c["nvme_stripe_dirs"] == ["/nvme0/ss", "/nvme1/ss"]


def test_v2_overlay_keys():
    c = native().parse_config(V2_STYLE)
    assert c["socket_path"] == "/tmp/y.sock"
    assert c["control_tcp_port"] == 7070
    assert c["dedup_default_mode"] == 2 and c["creating_policy"] == 1
    assert c["quota_max_pinned_bytes"] == 256 << 30
    assert c["quota_max_inflight_export_bytes"] == int(1.5 * (1 << 30))
    assert c["retain_sealed_versions"] == 6
    assert c["default_transport"] == 3 and c["fallback_transport"] == 2
    assert c["agent_options"] == {"kernels.evict_ctas": "32", "nvlink.weight_sync": "multicast"}


def test_defaults_and_sizes():
    c = native().parse_config("arenas:\n  per_numa:\n    - numa_node: 0\n      size_gb: 1\n")
    assert c["heartbeat_timeout_ms"] == 5000
    assert c["allocation_granularity_bytes"] == 16 << 20
    assert c["drain_target"] == "pageable_then_nvme"
    p = native().parse_size
    assert p("4096") == 4096 and p("2KiB") == 2048 and p("1TiB") == 1 << 40 and p("1.5 GB") == 3 << 29


@pytest.mark.parametrize("text, msg", [
    ("daemon:\n\tsocket_path: x\n", "tabs"),
    ("arenas:\n  per_numa:\n    - numa_node: 0\n      size_gb: 1\n      overflow_gb: 2\n", "exceed"),
    ("arenas:\n  allocation_granularity_mb: 0\n  per_numa:\n    - numa_node: 0\n      size_gb: 1\n", "granularity"),
    ("daemon:\n  heartbeat_timeout_ms: soon\n", "invalid integer"),
    ("drain_policy:\n  target_tier: tape\narenas:\n  per_numa:\n    - numa_node: 0\n      size_gb: 1\n", "target_tier"),
    ("nvme:\n  enabled: maybe\n", "invalid bool"),
    ("daemon:\n  socket_path: x\n", "per_numa"),
])
def test_invalid_configs_rejected(text, msg):
    with pytest.raises(Exception, match=msg):
        native().parse_config(text)


def test_shipped_configs_parse():
    for name in os.listdir(os.path.join(ROOT, "config")):
        if name.endswith(".yaml"):
            with open(os.path.join(ROOT, "config", name)) as f:
                native().parse_config(f.read())


def test_offloadd_print_config_and_bad_args(tmp_path):
    cfg = tmp_path / "c.yaml"
    cfg.write_text(V1_STYLE)
    out = subprocess.run([bin_path("offloadd"), "--config", str(cfg), "--socket", "/tmp/z.sock", "--print-config"],
                         capture_output=True, text=True, check=True).stdout
    assert "socket_path=/tmp/z.sock" in out and "arenas=2" in out and "drain_target=pageable_then_nvme" in out
    r = subprocess.run([bin_path("offloadd"), "--bogus"], capture_output=True, text=True)
    assert r.returncode == 2
    bad = tmp_path / "bad.yaml"
    bad.write_text("daemon:\n\tx: 1\n")
    r = subprocess.run([bin_path("offloadd"), "--config", str(bad)], capture_output=True, text=True)
    assert r.returncode == 1 and "tabs" in r.stderr


def test_offload_stat_cli(tmp_path):
    from statespectre_b200 import launch_daemon

    sock = str(tmp_path / "d.sock")
    with launch_daemon(sock, arena_mb=64):
        out = subprocess.run([bin_path("offload-stat"), "--socket", sock], capture_output=True, text=True,
                             check=True).stdout
        assert "d2h_bytes" in out and "canonical_objects_created_total" in out
        prom = subprocess.run([bin_path("offload-stat"), "--socket", sock, "--prometheus"], capture_output=True,
                              text=True, check=True).stdout
        assert "# TYPE offload_jobs_registered_total counter" in prom
        assert "offload_used_pinned_bytes 0" in prom
        # labelled series: one family per metric, a sample per GPU window and per job
        import torch

        from statespectre_b200 import offload_context

        with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name="prom-job") as off:
            off.copy(torch.randn(300000), wait=True)
            prom = subprocess.run([bin_path("offload-stat"), "--socket", sock, "--prometheus"],
                                  capture_output=True, text=True, check=True).stdout
        assert prom.count("# TYPE offload_window_used_bytes gauge") == 1
        assert 'offload_window_used_bytes{gpu="0"}' in prom
        assert 'offload_gpu_live_sessions' not in prom
        assert 'job="prom-job"' in prom and "# TYPE offload_job_pinned_bytes gauge" in prom
        jobs = subprocess.run([bin_path("offload-stat"), "--socket", sock, "--jobs"], capture_output=True, text=True,
                              check=True).stdout
        assert "job_id" in jobs
        sd = subprocess.run([bin_path("offload-stat"), "--socket", sock, "--shutdown"], capture_output=True,
                            text=True)
        assert sd.returncode == 0 and "shutting down" in sd.stdout


def test_daemon_forwards_kernels_and_nvlink_sections(tmp_path):
    """`kernels:` and `nvlink:` reach every session (GetAgentOptions, op 48);
    explicit session options win."""
    from statespectre_b200 import in_process_daemon, offload_context
    from statespectre_b200.api import _daemon_agent_options

    sock = str(tmp_path / "d.sock")
    text = f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 128
nvlink:
  weight_sync: multicast
kernels:
  evict_ctas: 40
  timing: true
nvme:
  enabled: false
"""
    d = in_process_daemon(yaml=text, socket=sock)
    try:
        opts = _daemon_agent_options(sock, 0, 0)
        assert opts == {"kernels.evict_ctas": "40", "kernels.timing": "true", "nvlink.weight_sync": "multicast"}
        with offload_context(daemon_addr=sock, device="cpu", rank=0, evict_ctas=8) as off:
            assert off.nvlink_options == {"weight_sync": "multicast"}
            t = __import__("torch").randn(1000)
            h = off.copy(t, wait=True)
            assert __import__("torch").equal(h.restore(), t)
    finally:
        d.stop()
    assert _daemon_agent_options(sock + ".missing", 0, 0) == {}


def test_per_job_quota_overrides_and_accepted_sections(tmp_path):
    """quotas.per_job_overrides applies to the named job only; roles:,
    libfabric:, cleanup: and metrics.labels are accepted and kept."""
    import torch

    from statespectre_b200 import ModelRole, in_process_daemon, offload_context

    sock = str(tmp_path / "d.sock")
    text = f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 64
roles:
  rollout_visible_roles:
    - POLICY_ROLLOUT
  immutable_roles:
    - POLICY_REFERENCE
    - REWARD_MODEL
quotas:
  default:
    max_pinned_bytes: 1GiB
  per_job_overrides:
    small:
      max_pinned_bytes: 1MiB
libfabric:
  provider: auto
cleanup:
  on_job_terminate: release
metrics:
  labels:
    cluster: b200
nvme:
  enabled: false
"""
    c = native().parse_config(text)
    assert c["job_quota_overrides"] == {"small": {"max_pinned_bytes": 1 << 20}}
    assert c["accepted_settings"]["roles.immutable_roles"] == "POLICY_REFERENCE,REWARD_MODEL"
    assert c["accepted_settings"]["libfabric.provider"] == "auto"
    assert c["accepted_settings"]["metrics.labels.cluster"] == "b200"
    d = in_process_daemon(yaml=text, socket=sock)
    try:
        t = torch.randn(1 << 20)  # 4 MiB
        for job, ok in (("small", False), ("big", True)):
            with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name=job) as off:
                k = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1, param_name="w", tensor=t)
                if ok:
                    assert off.canonical_evict(t.clone(), k).did_d2h
                else:
                    with pytest.raises(RuntimeError, match="quota"):
                        off.canonical_evict(t.clone(), k)
    finally:
        d.stop()
