"""Daemon state machine over the wire, no GPU and no data movement.

Covers what StateSpectre's test_daemon_rpc suite covers (lifecycle, epoch
rejection, re-register invalidation, stale versions, invalid transitions,
concurrent writers never overlapping; reference: tests/cpp/test_daemon_rpc.cpp:136-291)
plus the extensions (submit-on-grant, batch reservations, discard).
"""

import threading

import pytest

from statespectre_b200 import in_process_daemon
from statespectre_b200._native import native
from statespectre_b200._wire import Op

from rawclient import RawRank

MB = 1 << 20


@pytest.fixture
def d64(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    yield sock_path
    d.stop()


def test_lifecycle_offload_prefetch_h2d_release(d64):
    r = RawRank(d64, 1)
    assert r.heartbeat()["ok"]
    g = r.offload(100, 1, 3 * MB)
    assert g["capacity"] == 4 * MB  # 2 MiB slots
    loc = r.location(100)
    assert loc["ok"] and loc["location_kind"] == 2 and loc["nbytes"] == 3 * MB
    p = r.prefetch(100)
    assert p["ok"] and p["ready"] and p["slot_id"] == g["slot_id"]
    assert r.mark(Op.MARK_H2D_SUBMITTED, p["lease_id"], 100, 1, p["slot_id"])["ok"]
    assert r.h2d_complete(p["lease_id"], 100, 1, p["slot_id"])["ok"]
    # no cold copy: the pinned copy stays readable
    assert r.location(100)["location_kind"] == 2
    assert r.release(g["lease_id"])["ok"]
    assert r.location(100)["location_kind"] == 0
    assert r.release(g["lease_id"])["message"] == "already released"  # idempotent


def test_epoch_rejection_and_reregister_invalidates(d64):
    r = RawRank(d64, 2)
    old = r.epoch
    done = r.offload(1, 1, MB)
    pending = r.reserve(2, 1, MB)  # never completed
    assert pending["ok"]
    r2 = RawRank(d64, 2)  # same rank id: a restarted process
    assert r2.epoch != old
    assert not r.heartbeat(epoch=old)["ok"]
    assert not r2.reserve(3, 1, MB, epoch=old)["ok"]
    # completed data survives the restart, the orphaned reservation is reclaimed
    assert r2.location(1)["location_kind"] == 2
    stats = r2.stats()
    assert stats["rank_sessions_invalidated"] >= 1
    assert stats["rank_epoch_mismatch_rejected"] >= 2
    # the reclaimed run is reusable
    assert r2.reserve(4, 1, MB)["ok"]
    assert done["ok"]


def test_stale_version_and_invalid_transition(d64):
    r = RawRank(d64, 3)
    g2 = r.reserve(7, 2, MB)
    g1 = r.reserve(7, 1, MB)
    for g, v in ((g2, 2), (g1, 1)):
        assert r.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 7, v, g["slot_id"])["ok"]
    assert r.mark(Op.MARK_D2H_COMPLETE, g2["lease_id"], 7, 2, g2["slot_id"])["latest_version"]
    c1 = r.mark(Op.MARK_D2H_COMPLETE, g1["lease_id"], 7, 1, g1["slot_id"])
    assert c1["ok"] and not c1["latest_version"]
    assert r.location(7)["version"] == 2
    # complete without submitted -> invalid transition
    g = r.reserve(8, 1, MB)
    bad = r.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], 8, 1, g["slot_id"])
    assert not bad["ok"]
    # wrong tensor identity on a valid lease
    assert r.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 8, 1, g["slot_id"])["ok"]
    assert not r.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], 9, 1, g["slot_id"])["ok"]
    s = r.stats()
    assert s["stale_version_completion_rejected"] >= 1
    assert s["invalid_transition_rejected"] >= 2


def test_lease_owner_mismatch(d64):
    a, b = RawRank(d64, 10), RawRank(d64, 11)
    g = a.reserve(1, 1, MB)
    assert not b.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 1, 1, g["slot_id"])["ok"]
    assert not b.release(g["lease_id"])["ok"]
    assert b.stats()["lease_owner_mismatch_rejected"] >= 2


def test_blocked_when_full_and_no_overlap_under_concurrency(d64):
    granted = []
    lock = threading.Lock()
    errors = []

    def writer(rank):
        try:
            r = RawRank(d64, 20 + rank)
            for i in range(40):
                g = r.reserve(rank * 1000 + i, 1, 2 * MB)
                if not g["ok"]:
                    assert g["blocked"]
                    continue
                with lock:
                    granted.append((g["slot_id"], rank, i))
                assert r.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], rank * 1000 + i, 1, g["slot_id"])["ok"]
                if i % 3 == 0:  # release some so slots recycle
                    assert r.release(g["lease_id"])["ok"]
                    with lock:
                        granted.remove((g["slot_id"], rank, i))
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=writer, args=(k,)) for k in range(6)]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert not errors, errors
    live_slots = [g[0] for g in granted]
    assert len(live_slots) == len(set(live_slots)), "two live leases share a slot"
    r = RawRank(d64, 99)
    s = r.stats()
    assert s["blocked_reservation_count"] > 0
    assert s["slot_overlap_prevented"] == 0


def test_submit_on_grant_and_ready_flags(d64):
    r = RawRank(d64, 4)
    g = r.reserve(50, 1, MB, flags=1 << 16)
    assert g["ok"] and g["state"] == 2  # D2H_IN_FLIGHT straight away
    assert r.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], 50, 1, g["slot_id"])["ok"]
    p = r.prefetch(50, flags=1 << 17)
    assert p["ready"] and p["state"] == 8  # H2D_IN_FLIGHT straight away
    assert r.h2d_complete(p["lease_id"], 50, 1, p["slot_id"])["ok"]


def test_batch_reserve_and_batch_complete(d64):
    r = RawRank(d64, 5)
    items = [dict(tensor_id=600 + i, version=1, nbytes=MB, gpu_id=0, numa_node=0, flags=1 << 16) for i in range(8)]
    b = r.call(Op.BATCH_REQUEST_OFFLOAD, rank_id=5, rank_epoch=r.epoch, items=items)
    assert b["ok"] and all(g["ok"] for g in b["grants"])
    comps = [dict(event_type=1, lease_id=g["lease_id"], tensor_id=600 + i, version=1, slot_id=g["slot_id"])
             for i, g in enumerate(b["grants"])]
    c = r.call(Op.BATCH_COMPLETE, rank_id=5, rank_epoch=r.epoch, completions=comps)
    assert c["accepted"] == 8 and c["rejected"] == 0
    pf = r.call(Op.BATCH_REQUEST_PREFETCH, rank_id=5, rank_epoch=r.epoch,
                items=[dict(tensor_id=600 + i, version=1) for i in range(8)])
    assert all(x["ready"] for x in pf["results"])


def test_discard_frees_everything(d64):
    r = RawRank(d64, 6)
    used0 = r.stats()["used_slots"]
    r.offload(70, 1, 5 * MB)
    assert r.stats()["used_slots"] == used0 + 3
    d = r.call(Op.DISCARD_TENSOR, rank_id=6, rank_epoch=r.epoch, tensor_id=70, version=1)
    assert d["ok"]
    assert r.stats()["used_slots"] == used0
    assert not r.location(70)["ok"]


def test_stats_cover_every_metric_name(d64):
    r = RawRank(d64, 7)
    s = r.stats()
    for name in native().metric_names():
        assert name in s
    for k in ("bandwidth_mbps_p50", "bandwidth_mbps_p90", "bandwidth_mbps_p99", "total_slots"):
        assert k in s
    assert s["total_slots"] == 32


def test_control_plane_benchmark_runs():
    from statespectre_b200.benchmarks import control

    res = control.run(seconds=0.3, rank_counts=(2,))
    assert res["single"]["round_trips_per_s"] > 100
    assert res["batch"]["items_per_s"] > 1000
    assert res["ranks"]["2"]["round_trips_per_s"] > 100


def test_discard_batch_frees_everything(sock_path):
    import torch

    from statespectre_b200 import in_process_daemon, offload_context

    d = in_process_daemon(socket=sock_path, arena_mb=64, slot_mb=1, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            ts = [torch.randn(n) for n in (10, 1000, 300000, 17)]
            hs = off.evict_batch(ts) + [off.copy(torch.randn(5000), wait=True)]
            assert off.daemon_stats()["used_slots"] > 0
            off.discard_batch(hs)
            off.discard_batch(hs)  # idempotent
            st = off.daemon_stats()
            assert st["used_slots"] == 0 and st["pageable_resident_bytes"] == 0
    finally:
        d.stop()
