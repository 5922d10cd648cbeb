"""Durable sealed versions (manifest.persist_dir), no GPU.

A trainer session seals two versions (the second carries two of three tensors
forward), the daemon is killed with SIGKILL, a new daemon on the same
directory reloads both versions, and a rollout client pulls them byte for
byte with unchanged manifests. Dropping a version removes its manifest and the
storage only it used; carried-forward storage stays with the surviving
version.
"""

import os
import time

import pytest
import torch

from statespectre_b200 import ModelRole, RolloutWeightClient, _wire, launch_daemon, offload_context
from statespectre_b200._native import native

ROLL = ModelRole.POLICY_ROLLOUT


def _config(tmp_path, sock, persist):
    cfg = tmp_path / "offloadd.yaml"
    cfg.write_text(f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 96
manifest:
  retain_sealed_versions: 0
  persist_dir: {persist}
nvme:
  enabled: false
""")
    return str(cfg)


def _wait_stat(d, key, want, timeout=30.0):
    deadline = time.time() + timeout
    while time.time() < deadline:
        if d.stats().get(key, 0) >= want:
            return True
        time.sleep(0.02)
    return False


def _pull_all(sock, job, version):
    c = RolloutWeightClient(sock, job["job_id"], job["launch_epoch"], job_name=job["job_name"])
    man = c.get_manifest(version)
    data = {}
    for e in man["tensors"]:
        data[e["key"]["param_fqn_debug"]] = c.pull_tensor(e, version, transport="tcp")
    latest = c.get_latest_sealed_version()
    c.close()
    return man, data, latest


def test_sealed_versions_survive_daemon_kill(tmp_path):
    sock = str(tmp_path / "d.sock")
    persist = str(tmp_path / "versions")
    cfg = _config(tmp_path, sock, persist)
    g = torch.Generator().manual_seed(3)
    v1 = {"embed": torch.randn(300000, generator=g), "w": torch.randn(1000, 33, generator=g),
          "norm": torch.randn(17, generator=g)}
    v2 = dict(v1, w=v1["w"] + 1.0)
    d = launch_daemon(sock, config=cfg, log_path=str(tmp_path / "d1.log"))
    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name="trainer") as off:
            for n, t in v1.items():
                off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=1, param_name=n,
                                                                 tensor=t))
            off.promote_rollout_version(1)
            off.canonical_evict(v2["w"].clone(), off.canonical_key(model_role=ROLL, model_version=2, param_name="w",
                                                                   tensor=v2["w"]))
            pids = [off.canonical_key(model_role=ROLL, model_version=2, param_name=n, tensor=v1[n]).param_id
                    for n in ("embed", "norm")]
            off.carry_forward_version(ROLL, 1, 2, pids)
            off.promote_rollout_version(2)
            job = {"job_id": off.job_id, "launch_epoch": off.launch_epoch, "job_name": off.job_name}
            assert _wait_stat(d, "versions_persisted_total", 2)
            man1, data1, _ = _pull_all(sock, job, 1)
            man2, data2, latest = _pull_all(sock, job, 2)
            assert latest == 2
            # v2 wrote one new storage file: the carried-forward tensors share v1's
            jd = [os.path.join(persist, x) for x in os.listdir(persist)]
            assert len(jd) == 1
            files = sorted(os.listdir(jd[0]))
            assert sum(f.endswith(".obj") for f in files) == 4 and sum(f.endswith(".man") for f in files) == 2
            d.kill()  # crash: no shutdown path runs
    finally:
        d.kill()

    d = launch_daemon(sock, config=cfg, log_path=str(tmp_path / "d2.log"))
    try:
        st = d.stats()
        assert st["versions_recovered_total"] == 2 and st["canonical_objects"] == 6
        for version, before, want in ((1, man1, v1), (2, man2, v2)):
            man, data, latest = _pull_all(sock, job, version)
            assert latest == 2
            # the manifest is unchanged except where the bytes live now
            strip = [{k: v for k, v in e.items() if not k.startswith("location")} for e in man["tensors"]]
            was = [{k: v for k, v in e.items() if not k.startswith("location")} for e in before["tensors"]]
            assert strip == was and man["state"] == before["state"]
            assert all(e["location_hint"] == "nvme" for e in man["tensors"])
            for n, t in want.items():
                assert data[n] == t.numpy().tobytes(), (version, n)
                e = next(e for e in man["tensors"] if e["key"]["param_fqn_debug"] == n)
                assert (e["content_hash_lo"], e["content_hash_hi"]) == native().ssh_hash(t.numpy()) or \
                    (e["content_hash_lo"], e["content_hash_hi"]) == (0, 0)
        # the restarted trainer continues the same job namespace: sealed versions stay
        # read-only, the next version gets fresh object ids
        with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name="trainer") as off:
            assert (off.job_id, off.launch_epoch) == (job["job_id"], job["launch_epoch"])
            t = torch.randn(64)
            with pytest.raises(RuntimeError, match="REJECTED_STALE_VERSION"):
                off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=2, param_name="w",
                                                                 tensor=v2["w"]))
            # a recovered object restores through the agent (file -> pinned readback -> copy)
            from statespectre_b200 import CanonicalHandle

            e = next(e for e in man2["tensors"] if e["key"]["param_fqn_debug"] == "embed")
            out = torch.empty_like(v2["embed"])
            CanonicalHandle(e["object_id"], 0, False, None, "", off=off).restore_into(out)
            assert torch.equal(out, v2["embed"])
            h = off.canonical_evict(t, off.canonical_key(model_role=ROLL, model_version=3, param_name="x", tensor=t))
            assert h.object_id > max(e["object_id"] for e in man2["tensors"])
            off.seal_model_version(ROLL, 3)
        # drop version 1 of the recovered job: its manifest and its own "w" storage go, shared storage stays
        c = _wire.Connection(sock)
        r = c.call(_wire.Op.DROP_CANONICAL_VERSION, job={"tenant_id": 0, "job_id": job["job_id"],
                                                         "launch_epoch": job["launch_epoch"],
                                                         "job_name": job["job_name"]},
                   model_role=int(ROLL), model_version=1)
        c.close()
        assert r["ok"] and r["dropped_count"] == 3
        assert _wait_stat(d, "versions_persisted_total", 1)  # version 3
        files = sorted(os.listdir(jd[0]))
        assert sum(f.endswith(".man") for f in files) == 2  # versions 2 and 3
        assert sum(f.endswith(".obj") for f in files) == 4  # v2's three storages + v3's one
        _, data, _ = _pull_all(sock, job, 2)
        for n, t in v2.items():
            assert data[n] == t.numpy().tobytes()
    finally:
        d.stop()
    # and again after a clean restart: versions 2 and 3
    d = launch_daemon(sock, config=cfg, log_path=str(tmp_path / "d3.log"))
    try:
        assert d.stats()["versions_recovered_total"] == 2
        _, data, _ = _pull_all(sock, job, 2)
        assert data["w"] == v2["w"].numpy().tobytes()
    finally:
        d.stop()


def test_persisted_version_outlives_trainer_and_damaged_files_are_skipped(tmp_path):
    sock = str(tmp_path / "d.sock")
    persist = str(tmp_path / "versions")
    cfg = _config(tmp_path, sock, persist)
    t1, t2 = torch.randn(5000), torch.randn(7000)
    d = launch_daemon(sock, config=cfg, log_path=str(tmp_path / "d1.log"))
    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=0, job_name="trainer") as off:
            for v, t in ((1, t1), (2, t2)):
                off.canonical_evict(t.clone(), off.canonical_key(model_role=ROLL, model_version=v, param_name="w",
                                                                 tensor=t))
                off.promote_rollout_version(v)
            job = {"job_id": off.job_id, "launch_epoch": off.launch_epoch, "job_name": off.job_name}
            assert _wait_stat(d, "versions_persisted_total", 2)
        # the trainer's session is gone; the persisted versions stay pullable
        _, data, latest = _pull_all(sock, job, 1)
        assert latest == 2 and data["w"] == t1.numpy().tobytes()
    finally:
        d.stop()
    # damage version 1's storage file: only version 1 is skipped at recovery
    jd = os.path.join(persist, os.listdir(persist)[0])
    import struct

    # the storage of version 1 is the file whose header records t1's size
    for f in [f for f in os.listdir(jd) if f.endswith(".obj")]:
        with open(os.path.join(jd, f), "r+b") as fh:
            _magic, _fmt, _sid, nbytes = struct.unpack("<IIQQ", fh.read(24))
            if nbytes == t1.numel() * 4:
                fh.seek(0)
                fh.write(b"XXXX")  # bad magic
    d = launch_daemon(sock, config=cfg, log_path=str(tmp_path / "d2.log"))
    try:
        assert d.stats()["versions_recovered_total"] == 1
        _, data, latest = _pull_all(sock, job, 2)
        assert latest == 2 and data["w"] == t2.numpy().tobytes()
        c = RolloutWeightClient(sock, job["job_id"], job["launch_epoch"], job_name=job["job_name"])
        with pytest.raises(IOError):
            c.get_manifest(1)
        c.close()
    finally:
        d.stop()
