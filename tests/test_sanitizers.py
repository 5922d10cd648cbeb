"""Host-code sanitizers on the CUDA-free daemon (no GPU).

The daemon and the native self-test are rebuilt with AddressSanitizer +
UndefinedBehaviorSanitizer and with ThreadSanitizer; the self-test runs under
ASan, and each daemon build serves a multi-session host-mode workload (v1
evict/restore, batches, tier drains and readbacks, canonical evict, seal,
file pull, discard, a session that dies without closing) before a clean
shutdown. Any sanitizer report fails the test.
"""

import os
import subprocess
import threading
import time

import pytest
import torch

from statespectre_b200 import ModelRole, RolloutWeightClient, _build, offload_context
from statespectre_b200._native import bin_path
from statespectre_b200.daemon import launch_daemon

REPORTS = ("ERROR: AddressSanitizer", "runtime error:", "WARNING: ThreadSanitizer", "ERROR: LeakSanitizer")


@pytest.fixture(scope="module")
def sanitizer_builds():
    _build.build(sanitizers=True)
    return True


def _clean(text: str) -> bool:
    return not any(r in text for r in REPORTS)


def test_selftest_under_asan(sanitizer_builds):
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([bin_path("ofld_selftest_asan")], capture_output=True, text=True, timeout=300, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert _clean(out), out[-4000:]


def _workload(sock: str, rank: int, tmp_path) -> None:
    g = torch.Generator().manual_seed(rank)
    with offload_context(daemon_addr=sock, device="cpu", rank=rank, job_name=f"san{rank}") as off:
        ts = [torch.randn(n, generator=g) for n in (1000, 65536, 300000, 17)]
        refs = [t.clone() for t in ts]
        hs = [off.copy(t, wait=True) for t in ts]
        for h, r in zip(hs, refs):
            assert torch.equal(h.restore(), r)
        hb = off.evict_batch([t.clone() for t in refs])
        outs = [torch.empty_like(r) for r in refs]
        off.restore_batch(hb, outs)
        for o, r in zip(outs, refs):
            assert torch.equal(o, r)
        for h in hs + hb:
            h.discard()
        for i in range(3):
            w = torch.randn(4096, generator=g)
            key = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1, param_name=f"w{i}",
                                    tensor=w)
            off.canonical_evict(w, key)
        off.promote_rollout_version(1)
        client = RolloutWeightClient(sock, off.job_id, off.launch_epoch, job_name=off.job_name)
        res = client.sync_latest(transport="file")
        assert len(res["pulled"]) == 3
        client.close()
        off.daemon_stats()


@pytest.mark.parametrize("variant", ["asan", "tsan"])
def test_daemon_under_sanitizer(sanitizer_builds, tmp_path, variant):
    sock = str(tmp_path / "d.sock")
    log = str(tmp_path / f"offloadd_{variant}.log")
    env = dict(os.environ)
    if variant == "asan":
        env["ASAN_OPTIONS"] = "detect_leaks=1:abort_on_error=0"
        env["UBSAN_OPTIONS"] = "print_stacktrace=1"
    else:
        env["TSAN_OPTIONS"] = "halt_on_error=0:second_deadlock_stack=1"
    cfg = tmp_path / "offloadd.yaml"
    cfg.write_text(f"""
daemon:
  socket_path: {sock}
  heartbeat_timeout_ms: 1500
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 64
drain_policy:
  drain_on_d2h_complete: true
manifest:
  persist_dir: {tmp_path / "versions"}
nvme:
  enabled: false
""")
    d = launch_daemon(sock, config=str(cfg), log_path=log, env=env, binary=f"offloadd_{variant}")
    try:
        errs = []

        def run(rank):
            try:
                _workload(sock, rank, tmp_path)
            except Exception as e:  # noqa: BLE001
                errs.append(repr(e))

        ths = [threading.Thread(target=run, args=(r,)) for r in range(3)]
        for t in ths:
            t.start()
        for t in ths:
            t.join(240)
        assert not errs, errs
        deadline = time.time() + 30  # the persist worker wrote every sealed version
        while time.time() < deadline and d.stats()["versions_persisted_total"] < 3:
            time.sleep(0.05)
        assert d.stats()["versions_persisted_total"] == 3
        # a zbf16-coded canonical object pulled by three receivers at once: the
        # export decodes it over the copy pool from several connection threads
        from test_canonical import _coded_canonical_object, _pull_all

        raw = (torch.randn(3 << 19, generator=torch.Generator().manual_seed(1)) * 0.02).to(torch.bfloat16)
        raw = raw.view(torch.uint8).numpy().tobytes()
        rr, job, oid = _coded_canonical_object(sock, raw, "sanitized-coded")
        got = []
        pulls = [threading.Thread(target=lambda: got.append(_pull_all(sock, job))) for _ in range(3)]
        for t in pulls:
            t.start()
        for t in pulls:
            t.join(120)
        assert len(got) == 3 and all(g[k][oid] == raw for g in got for k in g)
        rr.close()
        # a session that stops heartbeating: the daemon reclaims it by timeout
        s = offload_context(daemon_addr=sock, device="cpu", rank=9)
        s.off.copy(torch.randn(5000), wait=True)
        s._agent.pause_heartbeat(True)
        time.sleep(2.5)
        assert d.stats()["rank_sessions_invalidated"] >= 1
        try:
            s.close()
        except Exception:  # noqa: BLE001 - its epoch is gone
            pass
    finally:
        rc = d.stop()
    text = open(log, errors="replace").read()
    assert _clean(text), text[-6000:]
    assert rc == 0, text[-3000:]


def test_daemon_under_asan_with_a_rank_that_corrupts_shared_memory(sanitizer_builds, tmp_path):
    """The ASan daemon serves a rank that rewrites its ring header (another
    rank's identity, a huge capacity, a tail a billion entries ahead) and
    another tensor's slot entry (arena, offset, size) while that tensor is
    drained and read back: no sanitizer report, the bytes come back intact."""
    from rawclient import RawRank

    from statespectre_b200._wire import Op

    sock = str(tmp_path / "d.sock")
    log = str(tmp_path / "offloadd_asan.log")
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    cfg = tmp_path / "offloadd.yaml"
    cfg.write_text(f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 8
drain_policy:
  drain_on_d2h_complete: false
nvme:
  enabled: false
""")
    d = launch_daemon(sock, config=str(cfg), log_path=log, env=env, binary="offloadd_asan")
    try:
        victim = RawRank(sock, 1)
        g = victim.reserve(77, 1, 4096)
        assert g["ok"] and victim.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 77, 1, g["slot_id"])["ok"]
        atk = RawRank(sock, 2, map_control=True)
        atk.write_ring_header(owner_rank=1, rank_epoch=victim.epoch, capacity=1 << 30)
        atk.ring_push(g["lease_id"], 77, 1, g["slot_id"])
        head, _ = atk.ring_head_tail()
        atk.set_ring_tail(head + 10 ** 9)
        deadline = time.time() + 20
        while time.time() < deadline and atk.ring_head_tail()[0] != head + 10 ** 9:
            time.sleep(0.01)
        assert atk.ring_head_tail()[0] == head + 10 ** 9
        assert victim.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], 77, 1, g["slot_id"])["ok"]
        with offload_context(daemon_addr=sock, device="cpu", rank=0) as off:
            x = torch.randn(1 << 18)
            h = off.copy(x, wait=True)
            slot = atk.location(h.tensor_id, h.version)["slot_id"]
            atk.scribble_slot(slot, arena_id=999, arena_offset=1 << 50, nbytes=1 << 40)
            hs = [off.copy(torch.randn(1 << 18), wait=True) for _ in range(10)]
            assert torch.equal(h.restore(), x)
            off.discard_batch(hs + [h])
        atk.close()
        victim.close()
    finally:
        rc = d.stop()
    text = open(log, errors="replace").read()
    assert _clean(text), text[-6000:]
    assert rc == 0, text[-3000:]
