"""CPU-only end-to-end: the plumbing workload of the north-star spec.

A host-mode session evicts and restores 64 fp32 CPU tensors whose shapes are
drawn by seed from {(1024,1024),(4096,256),(17,333)} with N(0,1) values, then
canonical-evicts 4 of them under job 'j0', seals version 1 and pulls them with
the file transport into a RolloutWeightClient. Every round trip must be
byte-identical.
"""

import random

import numpy as np
import torch

from statespectre_b200 import ModelRole, RolloutWeightClient, in_process_daemon, offload_context
from statespectre_b200._native import native


def test_cpu_plumbing_config(sock_path, tmp_path):
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False, tcp_port=0)
    try:
        rng = random.Random(7)
        g = torch.Generator().manual_seed(7)
        shapes = [rng.choice([(1024, 1024), (4096, 256), (17, 333)]) for _ in range(64)]
        with offload_context(daemon_addr=sock_path, device="cpu", job_name="j0") as off:
            tensors = [torch.randn(s, generator=g) for s in shapes]
            refs = [t.clone() for t in tensors]
            for t, r in zip(tensors, refs):
                h = off.evict(t, wait=True)
                assert t.numel() == 0
                back = h.restore()
                assert torch.equal(back, r)
                assert h.content_hash == native().ssh_hash(r.numpy())
                h.discard()
            handles = []
            for i in range(4):
                w = refs[i].clone()
                key = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1,
                                        param_name=f"w{i}", tensor=w)
                handles.append(off.canonical_evict(w, key))
            assert all(h.did_d2h for h in handles)
            sealed = off.promote_rollout_version(1)
            assert sealed["tensor_count"] == 4
            client = RolloutWeightClient(sock_path, off.job_id, off.launch_epoch, job_name=off.job_name)
            res = client.sync_latest(transport="file")
            assert res["version"] == 1 and len(res["pulled"]) == 4
            by_name = {}
            man = client.get_manifest(1)
            for e in man["tensors"]:
                by_name[e["key"]["param_fqn_debug"]] = res["data"][e["object_id"]]
            for i in range(4):
                assert by_name[f"w{i}"] == refs[i].numpy().tobytes()
            # nothing changed: a second sync pulls nothing
            again = client.sync_latest(transport="file")
            assert again["pulled"] == [] and len(again["skipped"]) == 4
            client.close()
    finally:
        d.stop()


def test_host_copy_restore_into_and_location(host_session):
    off = host_session
    x = torch.arange(1 << 16, dtype=torch.float32)
    h = off.copy(x, wait=True)
    assert h.ready() and h.location() == "pinned"
    y = torch.empty_like(x)
    h.restore_into(y, verify=True)
    assert torch.equal(x, y)
    h.discard()
    assert h.location() == "none"


def test_host_hash_oracle_properties():
    C = native()
    a = np.random.default_rng(0).integers(0, 256, 200_000, dtype=np.uint8)
    b = a.copy()
    assert C.ssh_hash(a) == C.ssh_hash(b)
    b[12345] ^= 1
    assert C.ssh_hash(a) != C.ssh_hash(b)
    assert C.ssh_hash(a[:0]) != (0, 0)
    # digests fold to the object hash
    assert C.ssh_fold(C.ssh_digests(a), a.nbytes) == C.ssh_hash(a)


def test_aliased_flat_buffer_restore_into(sock_path):
    """Parameters that are views of one flat buffer: the buffer is offloaded
    and restored in place, and every view sees the restored bytes (views keep
    aliasing); a destructive evict of a single view is refused."""
    import pytest

    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            flat = torch.randn(10000, generator=torch.Generator().manual_seed(1))
            views = {"a": flat[:1000].view(10, 100), "b": flat[1000:5000], "c": flat[5000:].view(50, 100)}
            ref = flat.clone()
            h = off.copy(flat, wait=True)
            flat.zero_()
            assert float(views["a"].abs().sum()) == 0.0
            h.restore_into(flat)
            assert torch.equal(flat, ref)
            assert torch.equal(views["a"].reshape(-1), ref[:1000])
            assert torch.equal(views["c"].reshape(-1), ref[5000:])
            views["b"][0] = 123.0
            assert float(flat[1000]) == 123.0
            with pytest.raises(RuntimeError):
                off.evict(views["b"])  # does not own its storage
            hv = off.evict(views["b"], allow_views=True, compact=True, wait=True)
            assert torch.equal(hv.restore(), flat[1000:5000])
            h.discard()
            hv.discard()
    finally:
        d.stop()


def test_session_trace_writes_chrome_json(sock_path, tmp_path):
    import json

    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=3) as off:
            path = str(tmp_path / "t.json")
            with off.trace(path):
                h = off.copy(torch.randn(1000), wait=True)
                h.restore()
                h.discard()
            evs = json.load(open(path))["traceEvents"]
            assert [e["ph"] for e in evs] == ["B", "E", "i"]
            delta = evs[2]["args"]
            assert delta["d2h_completed"] == 1 and delta["h2d_completed"] == 1 and delta["rpc_count"] > 0
            assert evs[0]["pid"] == 3
    finally:
        d.stop()
