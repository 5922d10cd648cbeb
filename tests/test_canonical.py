"""Canonical model-state store through the public API (host-mode ranks).

Mirrors StateSpectre's canonical suite (job namespaces, DP attach vs TP /
expert distinct, creating race, hash mismatch, duplicate candidate, seal +
pull, seal failure, canonical restore, drop, multi-consumer refcount, pull of
an unsealed version, quota; reference: tests/cpp/test_canonical.cpp:226-727).
"""

import os
import struct
import time

import pytest
import torch

from statespectre_b200 import (DedupPolicy, ModelRole, RolloutWeightClient, in_process_daemon, offload_context)
from statespectre_b200._wire import Op

from rawclient import RawRank

ROLL = ModelRole.POLICY_ROLLOUT


@pytest.fixture
def cdaemon(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False)
    yield sock_path
    d.stop()


def session(sock, rank, job="train", **kw):
    return offload_context(daemon_addr=sock, device="cpu", rank=rank, job_name=job, **kw)


def test_dp_replicas_attach_and_tp_shards_stay_distinct(cdaemon):
    w = torch.randn(256, 64)
    with session(cdaemon, 0) as r0, session(cdaemon, 1) as r1, session(cdaemon, 2) as r2:
        assert r0.job_id == r1.job_id and r0.launch_epoch == r1.launch_epoch  # one namespace per job
        k0 = r0.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=w, tp_rank=0)
        h0 = r0.canonical_evict(w.clone(), k0)
        assert h0.action_name == "NEED_D2H_CREATE" and h0.did_d2h
        k1 = r1.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=w, tp_rank=0)
        h1 = r1.canonical_evict(w.clone(), k1)  # DP replica: same identity, no copy
        assert h1.action_name == "ATTACHED_EXISTING" and not h1.did_d2h and h1.object_id == h0.object_id
        k2 = r2.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=w, tp_rank=1)
        h2 = r2.canonical_evict(w.clone(), k2)  # different TP shard: distinct object
        assert h2.did_d2h and h2.object_id != h0.object_id
        ke = r2.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=w, tp_rank=0, expert_id=3)
        he = r2.canonical_evict(w.clone(), ke)
        assert he.object_id not in (h0.object_id, h2.object_id)
        s = r0.daemon_stats()
        assert s["canonical_attach_existing_total"] == 1
        assert s["canonical_d2h_bytes_avoided"] == w.numel() * 4


def test_relaunch_gets_fresh_epoch_and_jobs_are_isolated(cdaemon):
    with session(cdaemon, 0, job="a") as a, session(cdaemon, 1, job="b") as b:
        assert a.job_id != b.job_id
        w = torch.ones(128)
        ka = a.canonical_key(model_role=ROLL, model_version=1, param_name="x", tensor=w)
        kb = b.canonical_key(model_role=ROLL, model_version=1, param_name="x", tensor=w)
        assert a.canonical_evict(w.clone(), ka).did_d2h
        assert b.canonical_evict(w.clone(), kb).did_d2h  # other job: no cross-job dedup


def test_hash_verified_detects_corrupt_replica(cdaemon):
    w = torch.randn(1024)
    with session(cdaemon, 0) as r0, session(cdaemon, 1) as r1:
        pol = DedupPolicy("hash_verified")
        k = r0.canonical_key(model_role=ROLL, model_version=3, param_name="w", tensor=w)
        r0.canonical_evict(w.clone(), k, dedup_policy=pol)
        ok = r1.canonical_evict(w.clone(), k, dedup_policy=pol)
        assert ok.action_name == "DUPLICATE_CANDIDATE" and ok.did_d2h
        bad = w.clone()
        bad[17] += 1.0
        with pytest.raises(RuntimeError, match="mismatch"):
            r1.canonical_evict(bad, k, dedup_policy=pol)
        assert r0.daemon_stats()["canonical_hash_mismatch_total"] == 1


def test_device_hash_verified_needs_no_copy(cdaemon):
    w = torch.randn(4096)
    with session(cdaemon, 0) as r0, session(cdaemon, 1) as r1:
        pol = DedupPolicy("device_hash_verified")
        k = r0.canonical_key(model_role=ROLL, model_version=4, param_name="w", tensor=w)
        c = r0.canonical_evict(w.clone(), k, dedup_policy=pol)
        assert c.did_d2h
        used = r0.daemon_stats()["used_slots"]
        v = r1.canonical_evict(w.clone(), k, dedup_policy=pol)
        assert v.action_name == "VERIFIED_BY_DEVICE_HASH" and not v.did_d2h
        assert r0.daemon_stats()["used_slots"] == used  # no candidate slot reserved
        bad = w.clone()
        bad[0] = 7
        with pytest.raises(RuntimeError, match="mismatch"):
            r1.canonical_evict(bad, k, dedup_policy=pol)


def test_creating_race_waits_then_attaches(cdaemon):
    """A second rank arriving while the creator has not committed gets WAIT."""
    r0 = RawRank(cdaemon, 0)
    job = r0.call(Op.REGISTER_JOB, tenant_id=0, job_name="race")["job"]
    key = {"job": job, "model_role": ROLL, "model_version": 1, "param_id": 5, "nbytes": 4096, "shard_nbytes": 4096,
           "expert_id": -1}
    req = dict(rank_id=0, rank_epoch=r0.epoch, key=key, destructive=True, attach_if_exists=True,
               create_if_missing=True, dedup_mode=1)
    c = r0.call(Op.REQUEST_CANONICAL_EVICT, **req)
    assert c["action"] == 1
    r1 = RawRank(cdaemon, 1)
    w = r1.call(Op.REQUEST_CANONICAL_EVICT, **dict(req, rank_id=1, rank_epoch=r1.epoch))
    assert w["action"] == 2 and w["object_id"] == c["object_id"]
    dup = r1.call(Op.REQUEST_CANONICAL_EVICT, **dict(req, rank_id=1, rank_epoch=r1.epoch,
                                                     allow_duplicate_candidate=True))
    assert dup["action"] == 3 and dup["synthetic_tid"] >> 62 == 3
    # creator finishes: D2H complete + commit
    assert r0.mark(Op.MARK_D2H_SUBMITTED, c["lease_id"], c["synthetic_tid"], 1, c["slot_id"])["ok"]
    assert r0.mark(Op.MARK_D2H_COMPLETE, c["lease_id"], c["synthetic_tid"], 1, c["slot_id"])["ok"]
    cm = r0.call(Op.COMMIT_CANONICAL_OBJECT, rank_id=0, rank_epoch=r0.epoch, object_id=c["object_id"],
                 lease_id=c["lease_id"], slot_id=c["slot_id"])
    assert cm["ok"] and cm["won"]
    # the candidate loser commits and attaches; its slot is freed
    lose = r1.call(Op.COMMIT_CANONICAL_OBJECT, rank_id=1, rank_epoch=r1.epoch, object_id=c["object_id"],
                   lease_id=dup["lease_id"], slot_id=dup["slot_id"])
    assert lose["ok"] and not lose["won"]
    again = r1.call(Op.REQUEST_CANONICAL_EVICT, **dict(req, rank_id=1, rank_epoch=r1.epoch))
    assert again["action"] == 0


def test_seal_pull_tcp_and_file_restore_drop(cdaemon, tmp_path):
    tensors = {f"layer{i}.w": torch.randn(100 + i, 33) for i in range(3)}
    with session(cdaemon, 0) as off:
        handles = {}
        for name, t in tensors.items():
            k = off.canonical_key(model_role=ROLL, model_version=5, param_name=name, tensor=t)
            handles[name] = off.canonical_evict(t.clone(), k)
        # pulling an unsealed version is refused
        c = RolloutWeightClient(cdaemon, off.job_id, off.launch_epoch, job_name=off.job_name)
        man_req_failed = False
        try:
            c.get_manifest(5)
        except IOError:
            man_req_failed = True
        assert man_req_failed
        info = off.promote_rollout_version(5)
        assert info["tensor_count"] == 3
        for transport in ("tcp", "file"):
            c2 = RolloutWeightClient(cdaemon, off.job_id, off.launch_epoch, job_name=off.job_name)
            res = c2.sync_latest(transport=transport, workers=2)
            assert len(res["pulled"]) == 3
            man = c2.get_manifest(5)
            for e in man["tensors"]:
                name = e["key"]["param_fqn_debug"]
                assert res["data"][e["object_id"]] == tensors[name].numpy().tobytes()
                assert e["location_hint"] == "pinned"
            c2.close()
        # canonical restore by object id
        for name, h in handles.items():
            out = torch.empty_like(tensors[name])
            h.restore_into(out)
            assert torch.equal(out, tensors[name])
        # manifest export in fixed record format
        path = str(tmp_path / "m.bin")
        r = off.export_manifest(ROLL, 5, path)
        assert r["tensor_count"] == 3 and os.path.getsize(path) == 192 + 3 * 384
        with open(path, "rb") as f:
            hdr = f.read(192)
        tenant, job_id, epoch, role, state, ver, ntens = struct.unpack("<QQQIIQQ", hdr[:48])
        assert (job_id, role, state, ver, ntens) == (off.job_id, ROLL, 2, 5, 3)
        # writes into a sealed version are rejected
        t = torch.randn(8)
        k = off.canonical_key(model_role=ROLL, model_version=5, param_name="late", tensor=t)
        with pytest.raises(RuntimeError, match="REJECTED_STALE_VERSION"):
            off.canonical_evict(t, k)
        d = off.drop_canonical_version(ROLL, 5)
        assert d["dropped"] == 3 and d["skipped_inflight"] == 0
        assert off.daemon_stats()["canonical_objects"] == 0


def test_seal_fails_when_expected_params_missing(cdaemon):
    with session(cdaemon, 0) as off:
        t = torch.randn(64)
        k = off.canonical_key(model_role=ROLL, model_version=2, param_name="a", tensor=t)
        off.canonical_evict(t, k)
        with pytest.raises(RuntimeError, match="missing"):
            off.seal_model_version(ROLL, 2, expected_param_ids=[k.param_id, 12345])
        assert off.seal_model_version(ROLL, 2, expected_param_ids=[k.param_id])["tensor_count"] == 1


def test_multi_consumer_refcount_release(cdaemon):
    w = torch.randn(512)
    with session(cdaemon, 0) as a, session(cdaemon, 1) as b:
        k = a.canonical_key(model_role=ROLL, model_version=9, param_name="w", tensor=w)
        ha = a.canonical_evict(w.clone(), k)
        hb = b.canonical_evict(w.clone(), k)
        assert hb.attached
        r1 = ha.release()
        assert r1 == {"released": 1, "freed": 0, "bytes_freed": 0, "message": "ok"}
        out = torch.empty_like(w)
        hb.restore_into(out)  # still alive for the other holder
        assert torch.equal(out, w)
        r2 = b.release_canonical_version(ROLL, 9)
        assert r2["freed"] == 1 and r2["bytes_freed"] == w.numel() * 4


def test_pinned_quota_rejects(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False, quota_max_pinned_bytes=1 << 20)
    try:
        with session(sock_path, 0) as off:
            t = torch.randn(1 << 18)  # exactly 1 MiB
            off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=1, param_name="a", tensor=t))
            t2 = torch.randn(16)
            with pytest.raises(RuntimeError, match="QUOTA"):
                off.canonical_evict(t2, off.canonical_key(model_role=ROLL, model_version=1, param_name="b",
                                                          tensor=t2))
            jobs = off.job_stats()
            assert jobs[0]["pinned_bytes"] == 1 << 20
    finally:
        d.stop()


def test_sealed_retention_drops_old_versions(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False, retain_sealed_versions=2)
    try:
        with session(sock_path, 0) as off:
            for v in range(1, 5):
                t = torch.full((256,), float(v))
                off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=v, param_name="w", tensor=t))
                off.promote_rollout_version(v)
            c = RolloutWeightClient(sock_path, off.job_id, off.launch_epoch)
            assert c.get_latest_sealed_version() == 4
            with pytest.raises(IOError):
                c.get_manifest(1)
            assert len(c.get_manifest(3)["tensors"]) == 1
            c.close()
    finally:
        d.stop()


def test_diff_skips_unchanged_tensors_across_versions(cdaemon):
    """A tensor whose bytes did not change between versions is not re-pulled."""
    a, b = torch.randn(300), torch.randn(300)
    with session(cdaemon, 0) as off:
        c = RolloutWeightClient(cdaemon, off.job_id, off.launch_epoch)
        for v, tensors in ((1, (a, b)), (2, (a, b + 1))):
            for name, t in zip(("a", "b"), tensors):
                off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=v, param_name=name,
                                                                 tensor=t))
            off.promote_rollout_version(v)
            res = c.sync_latest()
            assert len(res["pulled"]) == (2 if v == 1 else 1)
        c.close()


def test_carry_forward_shares_storage_and_survives_retention(sock_path):
    """Unchanged params of a new version share the old version's storage; the
    storage outlives the version that created it and is pulled byte-exact."""
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False, retain_sealed_versions=2)
    try:
        a, b = torch.randn(4096), torch.randn(4096)
        with session(sock_path, 0) as off:
            keys = {}
            for name, t in (("a", a), ("b", b)):
                k = off.canonical_key(model_role=ROLL, model_version=1, param_name=name, tensor=t)
                keys[name] = k
                off.canonical_evict(t.clone(), k)
            off.promote_rollout_version(1)
            used1 = off.daemon_stats()["used_slots"]
            cur_b = b
            for v in range(2, 6):
                cur_b = cur_b + 1
                k = off.canonical_key(model_role=ROLL, model_version=v, param_name="b", tensor=cur_b)
                off.canonical_evict(cur_b.clone(), k)
                r = off.carry_forward_version(ROLL, v - 1, v, [keys["a"].param_id])
                assert r["carried"] == 1 and r["missing"] == 0 and r["bytes_shared"] == a.numel() * 4
                again = off.carry_forward_version(ROLL, v - 1, v, [keys["a"].param_id])
                assert again["existing"] == 1 and again["carried"] == 0
                off.promote_rollout_version(v)
            # v1 and v2.. v3 dropped by retention; "a" still lives in v4/v5 without a copy
            stats = off.daemon_stats()
            assert stats["used_slots"] <= used1 + 2  # one slot run for a, and b of v4 + v5 (64 MiB slots)
            c = RolloutWeightClient(sock_path, off.job_id, off.launch_epoch)
            man = c.get_manifest(5)
            names = {e["object_id"]: e["key"]["param_fqn_debug"] for e in man["tensors"]}
            assert set(names.values()) == {"a", "b"}
            res = c.sync_latest()
            want = {"a": a, "b": cur_b}
            for oid, data in res["data"].items():
                assert data == want[names[oid]].numpy().tobytes()
            c.close()
            off.drop_canonical_version(ROLL, 4)
            off.drop_canonical_version(ROLL, 5)
            assert off.daemon_stats()["used_slots"] == 0
    finally:
        d.stop()


def test_carry_forward_rejects_sealed_target_and_unknown_job(cdaemon):
    with session(cdaemon, 0) as off:
        t = torch.ones(64)
        off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=t))
        off.promote_rollout_version(1)
        with pytest.raises(RuntimeError, match="already sealed"):
            off.carry_forward_version(ROLL, 2, 1)
        r = off.carry_forward_version(ROLL, 1, 2, [12345])
        assert r["missing"] == 1 and r["carried"] == 0


def test_export_cancelled_when_receiver_disconnects(cdaemon):
    """A rollout receiver that hangs up mid-stream: the daemon's export fails
    cleanly (error counted, in-flight bytes released, object unpinned), the
    object stays pullable and the version can be dropped."""
    import socket
    import threading

    from statespectre_b200 import _wire

    big = torch.randn(8 << 20)  # 32 MiB: far more than the socket buffers hold
    with session(cdaemon, 0) as off:
        k = off.canonical_key(model_role=ROLL, model_version=1, param_name="big", tensor=big)
        off.canonical_evict(big.clone(), k)
        off.promote_rollout_version(1)
        c = RolloutWeightClient(cdaemon, off.job_id, off.launch_epoch, job_name=off.job_name)
        entry = c.get_manifest(1)["tensors"][0]
        lsock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        lsock.bind(("127.0.0.1", 0))
        lsock.listen(1)
        lsock.settimeout(30)
        result = {}
        base = {"job": c._job(), "model_role": int(ROLL), "model_version": 1, "object_id": int(entry["object_id"])}

        def rpc():
            result["resp"] = c._conn_for_pull().call(Op.PULL_TENSOR, base, transport=_wire.TK_TCP,
                                                      target_descriptor=f"127.0.0.1:{lsock.getsockname()[1]}")

        th = threading.Thread(target=rpc)
        th.start()
        conn, _ = lsock.accept()
        conn.recv(1 << 20)
        conn.setsockopt(socket.SOL_SOCKET, socket.SO_LINGER, struct.pack("ii", 1, 0))  # reset, not FIN
        conn.close()
        lsock.close()
        th.join(60)
        assert not th.is_alive()
        assert result["resp"]["ok"] is False and "transport failed" in result["resp"]["message"]
        st = off.daemon_stats()
        assert st["export_transport_errors_total"] >= 1
        assert st["export_inflight_bytes"] == 0
        # the object is intact and exports again
        res = c.sync_latest(transport="tcp")
        assert res["data"][entry["object_id"]] == big.numpy().tobytes()
        c.close()
        d = off.drop_canonical_version(ROLL, 1)
        assert d["dropped"] == 1 and d["skipped_inflight"] == 0


def test_cold_tier_and_inflight_quotas(tmp_path):
    """max_pageable_bytes sends a job's drains to NVMe once its pageable share
    is used up; max_inflight_d2h_bytes caps what a job may copy at once; job
    accounting follows the bytes out when objects are dropped."""
    import time

    sock = str(tmp_path / "q.sock")
    text = f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 64
drain_policy:
  drain_on_d2h_complete: true
nvme:
  enabled: true
  path: {tmp_path / "nvme"}
  direct_io: false
quotas:
  per_job_overrides:
    capped:
      max_pageable_bytes: 6MiB
    narrow:
      max_inflight_d2h_bytes: 1MiB
"""
    d = in_process_daemon(yaml=text, socket=sock)
    try:
        with session(sock, 0, job="capped") as off:
            hs = []
            for i in range(3):  # 4 MiB each: the first fits the 6 MiB pageable quota, the others spill
                t = torch.randn(1 << 20)
                hs.append(off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=1,
                                                                   param_name=f"w{i}", tensor=t)))
            deadline = time.time() + 10
            while time.time() < deadline and off.job_stats()[0]["pageable_bytes"] < (4 << 20):
                time.sleep(0.01)
            time.sleep(0.2)
            js = [j for j in off.job_stats() if j["job"]["job_name"] == "capped"][0]
            assert js["pageable_bytes"] == 4 << 20 and js["nvme_bytes"] == 8 << 20, js
            off.drop_canonical_version(ROLL, 1)
            js = [j for j in off.job_stats() if j["job"]["job_name"] == "capped"][0]
            assert js["pageable_bytes"] == 0 and js["nvme_bytes"] == 0 and js["pinned_bytes"] == 0, js
        with session(sock, 1, job="narrow") as off:
            t = torch.randn(1 << 20)  # 4 MiB > 1 MiB in flight
            with pytest.raises(RuntimeError, match="QUOTA"):
                off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=t))
            small = torch.randn(1000)
            h = off.canonical_evict(small, off.canonical_key(model_role=ROLL, model_version=1, param_name="s",
                                                             tensor=small))
            assert h.did_d2h
            js = [j for j in off.job_stats() if j["job"]["job_name"] == "narrow"][0]
            assert js["inflight_d2h_bytes"] == 0  # settled at commit
    finally:
        d.stop()


def test_carry_forward_of_one_tensor_parallel_shard(sock_path):
    """Two TP ranks hold shards of the same parameters (same param_id): each
    carries forward only its own partition, so a version where rank 0 changed
    "w" and rank 1 did not has rank 0's new object and rank 1's old one."""
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False)
    try:
        shards = {0: torch.randn(4096), 1: torch.randn(4096)}
        with session(sock_path, 0) as off:
            def key(v, r, t):
                return off.canonical_key(model_role=ROLL, model_version=v, param_name="w", tensor=t, tp_rank=r)

            for r, t in shards.items():
                off.canonical_evict(t.clone(), key(1, r, t))
            off.promote_rollout_version(1)
            new0 = shards[0] + 1
            off.canonical_evict(new0.clone(), key(2, 0, new0))            # rank 0 changed w
            pid = key(2, 1, shards[1]).param_id
            c1 = off.carry_forward_version(ROLL, 1, 2, [pid], tp_rank=1)  # rank 1 did not
            assert c1["carried"] == 1 and c1["existing"] == 0
            c0 = off.carry_forward_version(ROLL, 1, 2, [pid], tp_rank=0)  # rank 0 already has its v2 object
            assert c0["carried"] == 0 and c0["existing"] == 1
            off.promote_rollout_version(2)
            c = RolloutWeightClient(sock_path, off.job_id, off.launch_epoch)
            res = c.sync_latest()
            man = c.get_manifest(2)
            by_tp = {e["key"]["tp_rank"]: e["object_id"] for e in man["tensors"]}
            assert sorted(by_tp) == [0, 1]
            assert res["data"][by_tp[0]] == new0.numpy().tobytes()
            assert res["data"][by_tp[1]] == shards[1].numpy().tobytes()
            c.close()
            # without a shard filter every partition of the parameter is carried
            everything = off.carry_forward_version(ROLL, 2, 3, [pid])
            assert everything["carried"] == 2
    finally:
        d.stop()


def test_p2p_verified_replica_attaches_with_its_own_action(cdaemon):
    """Dedup mode 5: a replica that compared its bytes with the owner's GPU
    copy (statespectre_b200.parallel.dp_dedup) attaches without any copy and
    is counted separately from trusted attaches."""
    w = torch.randn(300, 40)
    pol = DedupPolicy("p2p_verified")
    with session(cdaemon, 0) as r0, session(cdaemon, 1) as r1:
        k = r0.canonical_key(model_role=ROLL, model_version=1, param_name="w", tensor=w)
        h0 = r0.canonical_evict(w.clone(), k, dedup_policy=pol)
        assert h0.action_name == "NEED_D2H_CREATE" and h0.did_d2h
        before = r1.daemon_stats()
        h1 = r1.canonical_evict(w.clone(), r1.canonical_key(model_role=ROLL, model_version=1, param_name="w",
                                                            tensor=w), dedup_policy=pol)
        assert h1.action_name == "VERIFIED_BY_P2P" and not h1.did_d2h and h1.object_id == h0.object_id
        after = r1.daemon_stats()
        assert after["canonical_p2p_verified_total"] == before["canonical_p2p_verified_total"] + 1
        assert after["canonical_d2h_bytes_avoided"] - before["canonical_d2h_bytes_avoided"] == w.numel() * 4
        out = torch.empty_like(w)
        h1.restore_into(out)
        assert torch.equal(out, w)


def test_non_destructive_canonical_evict_of_a_view_in_a_flat_buffer(cdaemon):
    """Parameters that are views of one flat buffer (a data-parallel trainer's
    layout) are copied in place by a non-destructive canonical evict; a
    destructive one still refuses a view that does not own its storage."""
    flat = torch.randn(10000)
    a, b = flat[:4000].view(40, 100), flat[4000:]
    with session(cdaemon, 0) as off:
        ha = off.canonical_evict(a, off.canonical_key(model_role=ROLL, model_version=1, param_name="a", tensor=a),
                                 destructive=False)
        hb = off.canonical_evict(b, off.canonical_key(model_role=ROLL, model_version=1, param_name="b", tensor=b),
                                 destructive=False)
        assert ha.did_d2h and hb.did_d2h and flat.numel() == 10000
        out = torch.empty(40, 100)
        ha.restore_into(out)
        assert torch.equal(out, a)
        with pytest.raises(RuntimeError, match="does not own"):
            off.canonical_evict(a, off.canonical_key(model_role=ROLL, model_version=2, param_name="a", tensor=a))


@pytest.mark.parametrize("max_inflight", [0, 5000])
def test_canonical_evict_batch_matches_one_by_one(cdaemon, max_inflight):
    """canonical_evict_batch records the same objects, hashes and manifest as
    one canonical_evict per tensor; a DP replica's batch attaches; the
    in-flight bound only changes when copies are awaited."""
    torch.manual_seed(3)
    tensors = {f"l{i}.w": torch.randn(40 + 7 * i, 31) for i in range(6)}
    with session(cdaemon, 0) as a, session(cdaemon, 1) as b:
        one = {}
        for name, t in tensors.items():
            k = a.canonical_key(model_role=ROLL, model_version=1, param_name=name, tensor=t)
            one[name] = a.canonical_evict(t.clone(), k, destructive=False)
        man1 = a.promote_rollout_version(1)
        items = [(t.clone(), a.canonical_key(model_role=ROLL, model_version=2, param_name=n, tensor=t))
                 for n, t in tensors.items()]
        hs = a.canonical_evict_batch(items, destructive=False, max_inflight_bytes=max_inflight)
        assert [h.action_name for h in hs] == ["NEED_D2H_CREATE"] * len(tensors)
        assert all(h.did_d2h for h in hs)
        assert [h.content_hash for h in hs] == [one[n].content_hash for n in tensors]
        man2 = a.promote_rollout_version(2)
        assert man2["tensor_count"] == man1["tensor_count"] == len(tensors)
        def entries(v):
            man = a.get_manifest(ROLL, v)
            return sorted((e["key"]["param_fqn_debug"], e["content_hash_lo"], e["content_hash_hi"], e["nbytes"])
                          for e in man["tensors"])

        assert entries(2) == entries(1)
        # a DP replica (another rank, same identity) attaches without copying
        rep = [(t.clone(), b.canonical_key(model_role=ROLL, model_version=3, param_name=n, tensor=t))
               for n, t in tensors.items()]
        own = [(t.clone(), a.canonical_key(model_role=ROLL, model_version=3, param_name=n, tensor=t))
               for n, t in tensors.items()]
        a.canonical_evict_batch(own, destructive=False)
        hb = b.canonical_evict_batch(rep, destructive=False)
        assert all(h.action_name == "ATTACHED_EXISTING" and not h.did_d2h for h in hb)
        # bytes come back exactly
        for (name, t), h in zip(tensors.items(), hs):
            out = torch.empty_like(t)
            h.restore_into(out)
            assert torch.equal(out, t)
        assert a.canonical_evict_batch([]) == []


def test_canonical_evict_batch_destructive_releases_storage(cdaemon):
    with session(cdaemon, 0) as off:
        ts = [torch.randn(64, 16) for _ in range(3)]
        refs = [t.clone() for t in ts]
        items = [(t, off.canonical_key(model_role=ROLL, model_version=1, param_name=f"p{i}", tensor=t))
                 for i, t in enumerate(ts)]
        hs = off.canonical_evict_batch(items)
        assert all(t.numel() == 0 for t in ts)
        for h, r in zip(hs, refs):
            out = torch.empty_like(r)
            h.restore_into(out)
            assert torch.equal(out, r)


def _coded_canonical_object(sock, raw: bytes, job_name: str, version: int = 1, fmt: str = "zbf16"):
    """Create a canonical object whose pinned run holds `raw` coded (zbf16 or
    zf32, the host codec's bytes, as a GPU agent's coded evict stores them),
    record its coding with SetRunFormat, commit it with the raw bytes' hash
    and promote the version. Returns (rank, job, object id)."""
    import numpy as np

    from statespectre_b200._native import native

    C = native()
    arr = np.frombuffer(raw, dtype=np.uint8)
    coded = C.zbf16_encode(arr) if fmt == "zbf16" else C.zf32_encode(arr)
    assert coded is not None and len(coded) == len(raw) and coded != raw
    r = RawRank(sock, 0, map_control=True)
    job = r.call(Op.REGISTER_JOB, tenant_id=0, job_name=job_name)["job"]
    key = {"job": job, "model_role": ROLL, "model_version": version, "param_id": 77, "param_fqn_debug": "coded.w",
           "nbytes": len(raw), "shard_nbytes": len(raw), "expert_id": -1, "dtype": 15 if fmt == "zbf16" else 6}
    c = r.call(Op.REQUEST_CANONICAL_EVICT, rank_id=0, rank_epoch=r.epoch, key=key, destructive=False,
               attach_if_exists=True, create_if_missing=True, dedup_mode=1, alignment=256)
    assert c["ok"] and c["action"] == 1, c
    r.write_arena(c["arena_id"], c["arena_offset"], coded)
    bit = (1 << 18) if fmt == "zbf16" else (1 << 19)
    bad = r.call(Op.SET_RUN_FORMAT, rank_id=0, rank_epoch=r.epoch, lease_id=c["lease_id"] + 99, slot_id=c["slot_id"],
                 format=bit)
    assert not bad["ok"]  # only the lease holder records a coding
    assert not r.call(Op.SET_RUN_FORMAT, rank_id=0, rank_epoch=r.epoch, lease_id=c["lease_id"], slot_id=c["slot_id"],
                      format=3 << 18)["ok"]  # both codings at once is no coding
    assert r.call(Op.SET_RUN_FORMAT, rank_id=0, rank_epoch=r.epoch, lease_id=c["lease_id"], slot_id=c["slot_id"],
                  format=bit)["ok"]
    assert r.mark(Op.MARK_D2H_SUBMITTED, c["lease_id"], c["synthetic_tid"], 1, c["slot_id"])["ok"]
    assert r.mark(Op.MARK_D2H_COMPLETE, c["lease_id"], c["synthetic_tid"], 1, c["slot_id"])["ok"]
    lo, hi = C.ssh_hash(arr)
    cm = r.call(Op.COMMIT_CANONICAL_OBJECT, rank_id=0, rank_epoch=r.epoch, object_id=c["object_id"],
                lease_id=c["lease_id"], slot_id=c["slot_id"], content_hash_lo=lo, content_hash_hi=hi)
    assert cm["ok"], cm
    s = r.call(Op.SEAL_MODEL_VERSION, job=job, model_role=ROLL, model_version=version, fail_if_missing=True,
               expected_param_ids=[], promote=True)
    assert s["ok"], s
    # once complete, the coding of the run is fixed
    assert not r.call(Op.SET_RUN_FORMAT, rank_id=0, rank_epoch=r.epoch, lease_id=c["lease_id"],
                      slot_id=c["slot_id"], format=0)["ok"]
    return r, job, c["object_id"]


def _pull_all(sock, job, transports=("tcp", "file")):
    out = {}
    for transport in transports:
        cl = RolloutWeightClient(sock, job["job_id"], job["launch_epoch"], job_name=job["job_name"])
        res = cl.sync_latest(transport=transport)
        out[transport] = res["data"]
        cl.close()
    return out


@pytest.mark.parametrize("fmt", ["zbf16", "zf32"])
def test_coded_canonical_object_is_served_raw_from_pinned(sock_path, fmt):
    """A canonical object whose run is coded is exported decoded: TCP and
    FILE pulls (and the reference-format receiver's hash check) see the raw
    bytes; the export counts the decoded bytes."""
    d = in_process_daemon(socket=sock_path, arena_mb=128, drain_on_complete=False)
    try:
        g = torch.Generator().manual_seed(5)
        if fmt == "zbf16":
            raw = (torch.randn((3 << 20) // 2 + 8 * 1000, generator=g) * 0.02).to(torch.bfloat16)
        else:
            raw = torch.randn(5 * 32768, generator=g) * 0.02
        raw = raw.view(torch.uint8).numpy().tobytes()
        r, job, oid = _coded_canonical_object(sock_path, raw, f"coded-{fmt}", fmt=fmt)
        before = r.stats().get("export_decoded_bytes_total", 0)
        for transport, data in _pull_all(sock_path, job).items():
            assert data[oid] == raw, transport
        assert r.stats()["export_decoded_bytes_total"] - before == 2 * len(raw)
        r.close()
    finally:
        d.stop()


def test_coded_canonical_object_drained_and_persisted_stays_exact(tmp_path):
    """The coding follows the bytes: drained to pageable memory, written to
    the persist directory verbatim and reloaded by a restarted daemon, the
    object still pulls as its raw bytes."""
    sock = str(tmp_path / "d.sock")
    pdir = str(tmp_path / "persist")
    raw = (torch.randn(1 << 20, generator=torch.Generator().manual_seed(9))).to(torch.bfloat16)
    raw = raw.view(torch.uint8).numpy().tobytes()
    d = in_process_daemon(socket=sock, arena_mb=128, drain_on_complete=True, persist_dir=pdir)
    try:
        r, job, oid = _coded_canonical_object(sock, raw, "coded-tiers")
        man = RolloutWeightClient(sock, job["job_id"], job["launch_epoch"], job_name=job["job_name"])
        for _ in range(500):
            if man.get_manifest(1)["tensors"][0]["location_hint"] != "pinned":
                break
            time.sleep(0.01)
        assert man.get_manifest(1)["tensors"][0]["location_hint"] in ("pageable", "nvme")
        man.close()
        assert _pull_all(sock, job)["tcp"][oid] == raw
        for _ in range(500):
            if r.stats().get("versions_persisted_total", 0) >= 1:
                break
            time.sleep(0.01)
        assert r.stats()["versions_persisted_total"] >= 1
        r.close()
    finally:
        d.stop()
    d = in_process_daemon(socket=sock, arena_mb=128, drain_on_complete=False, persist_dir=pdir)
    try:
        data = _pull_all(sock, job)
        assert data["tcp"][oid] == raw and data["file"][oid] == raw
    finally:
        d.stop()


def test_host_mode_consumer_decodes_a_coded_object(cdaemon):
    """A CPU (host-mode) session restoring an object that a GPU rank stored
    coded gets the raw bytes, whole or as a 64 KiB-multiple prefix."""
    raw_t = (torch.randn(3 << 19, generator=torch.Generator().manual_seed(4)) * 0.02).to(torch.bfloat16)
    raw = raw_t.view(torch.uint8).numpy().tobytes()
    r, job, oid = _coded_canonical_object(cdaemon, raw, "coded-host")
    with session(cdaemon, 5, job="coded-host") as off:
        out = torch.empty_like(raw_t)
        ok, msg = off._agent.canonical_restore(oid, out.data_ptr(), len(raw), 0, True)
        assert ok, msg
        assert out.view(torch.uint8).numpy().tobytes() == raw
        part = torch.empty(65536, dtype=torch.uint8)
        ok, msg = off._agent.canonical_restore(oid, part.data_ptr(), 65536, 0, True)
        assert ok, msg
        assert part.numpy().tobytes() == raw[:65536]
        odd = torch.empty(1000, dtype=torch.uint8)
        ok, msg = off._agent.canonical_restore(oid, odd.data_ptr(), 1000, 0, True)
        assert not ok and "64 KiB" in msg
    r.close()


def test_corrupt_coded_object_fails_its_export_and_the_daemon_survives(cdaemon):
    """Coded bytes that no longer decode (a rank scribbled over its run after
    the commit) make that pull fail with a message; other objects and later
    pulls are unaffected."""
    raw = (torch.randn(1 << 20, generator=torch.Generator().manual_seed(2))).to(torch.bfloat16)
    raw = raw.view(torch.uint8).numpy().tobytes()
    r, job, oid = _coded_canonical_object(cdaemon, raw, "coded-corrupt")
    cl = RolloutWeightClient(cdaemon, job["job_id"], job["launch_epoch"], job_name=job["job_name"])
    man = cl.get_manifest(1)
    entry = man["tensors"][0]
    assert cl.pull_tensor(entry, 1) == raw
    # find the run and overwrite the escape count of its third chunk header
    arena_id, off = None, None
    for s in range(r.num_slots):
        state, a, o, n, tid = r.slot_fields(s)
        if n == len(raw) and tid >> 63:
            arena_id, off = a, o
            break
    assert arena_id is not None
    r.write_arena(arena_id, off + 2 * 65536 + 4, b"\xff\xff\x00\x00")
    with pytest.raises(Exception, match="decode|transport|export|failed"):
        cl.pull_tensor(entry, 1)
    cl.close()
    assert r.stats()["export_transport_errors_total"] >= 1
    r.close()
