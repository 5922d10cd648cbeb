"""Two processes on two GPUs: peer-buffer broker, K4 push over NVLink, K3
P2P byte verification, and a sealed version the rollout can check.

The trainer (this process, cuda:0) hosts the daemon; the rollout is a spawned
child on cuda:1 that publishes its receive buffer and checks what arrives.
Every wait between the processes has a timeout.
"""

import multiprocessing as mp

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

TIMEOUT = 120


def _specs():
    return [("w0", (1024, 1024), "bfloat16"), ("w1", (4096, 256), "bfloat16"), ("b", (256,), "bfloat16"),
            ("w2", (3000, 512), "bfloat16")]


def _rollout(sock, mode, transport, q_in, q_out):
    import torch

    from statespectre_b200 import offload_context
    from statespectre_b200.parallel.weight_sync import RolloutWeights, WeightLayout

    torch.cuda.set_device(1)
    try:
        with offload_context(daemon_addr=sock, device="cuda:1", rank=1, job_name="fabric2") as off:
            layout = WeightLayout([(n, s, getattr(torch, d)) for n, s, d in _specs()], mode)
            rw = RolloutWeights(layout, "cuda:1")
            rw.publish(off, f"rollout/{mode}/{transport}")
            q_out.put(("published", layout.fingerprint))
            q_out.put(("connected", rw.connect(off, TIMEOUT * 1000)))
            while True:
                msg = q_in.get(timeout=TIMEOUT)
                if msg[0] == "done":
                    break
                _, version, hashes, host = msg
                torch.cuda.synchronize()
                ok = True
                if mode == "bf16":
                    ok = rw.content_hashes() == hashes
                    for n, t in host.items():
                        ok &= torch.equal(rw.get(n).cpu(), t)
                else:
                    for n, t in host.items():
                        ok &= torch.allclose(rw.dequantized(n).float().cpu(), t.float(), rtol=0.07, atol=1e-6)
                q_out.put(("checked", version, bool(ok)))
            rw.close(TIMEOUT * 1000)
    except Exception as e:  # noqa: BLE001
        q_out.put(("error", repr(e)))


@pytest.fixture
def two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


@pytest.mark.parametrize("transport", ["p2p", "multicast"])
@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_push_across_gpus_and_verify_peer(two_gpus, sock_path, mode, transport):
    from statespectre_b200 import in_process_daemon, offload_context
    from statespectre_b200._native import native
    from statespectre_b200.parallel import fabric
    from statespectre_b200.parallel.weight_sync import TrainerWeightSync

    if transport == "multicast" and not (fabric.multicast_supported(0) and fabric.multicast_supported(1)):
        pytest.skip("no switch multicast on these GPUs")
    d = in_process_daemon(socket=sock_path, arena_mb=1024, drain_on_complete=False)
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_rollout, args=(sock_path, mode, transport, q_in, q_out))
    child.start()
    tr = None
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="fabric2") as off:
            try:
                torch.manual_seed(0)
                params = {n: (torch.randn(s, device="cuda:0") * 0.02).to(getattr(torch, dt))
                          for n, s, dt in _specs()}
                tag, fp = q_out.get(timeout=TIMEOUT)
                assert tag == "published"
                tr = TrainerWeightSync(off, params, [f"rollout/{mode}/{transport}"], mode=mode, transport=transport)
                assert tr.layout.fingerprint == fp
                assert tr.transport == transport
                assert q_out.get(timeout=TIMEOUT) == ("connected", transport)
                for version in (1, 2):
                    if version == 2:
                        params["w1"].add_(0.5)
                    r = tr.publish_version(version)
                    assert r["changed"] == (len(params) if version == 1 else 1)
                    q_in.put(("check", version, tr.pushers[0].hashes(), {n: t.cpu() for n, t in params.items()}))
                    msg = q_out.get(timeout=TIMEOUT)
                    assert msg == ("checked", version, True), msg
                if mode == "bf16" and transport == "p2p":
                    # K3: compare the local parameter with the rollout's copy by P2P loads
                    C = native()
                    peer = tr.peers[0]
                    e = tr.layout.by_name["w2"]
                    n = e.nbytes
                    dig = torch.zeros((n + 65535) // 65536, dtype=torch.int64, device="cuda:0")
                    mism = torch.zeros(1, dtype=torch.int32, device="cuda:0")
                    s = torch.cuda.current_stream().cuda_stream
                    C.k_verify_peer(params["w2"].data_ptr(), peer.ptr + e.dst_offset, n, dig.data_ptr(),
                                    mism.data_ptr(), s, 0)
                    torch.cuda.synchronize()
                    assert mism.item() == 0
                man = off.get_manifest("policy_rollout", 2)
                assert len(man["tensors"]) == len(params)
            finally:
                # Team teardown and the 'closed' signal come first, on every path: the
                # rollout leaves the team only after that, never while bound to it.
                if tr is not None:
                    tr.close()
                q_in.put(("done",))
        child.join(TIMEOUT)
        assert child.exitcode == 0
    finally:
        if child.is_alive():
            child.join(TIMEOUT)
        if child.is_alive() and transport == "p2p":
            # Only a point-to-point child may be killed; a child that may still be bound
            # to a multicast object is left to exit on its own queue timeout.
            child.kill()
            child.join(10)
        d.stop()
        assert not child.is_alive(), "rollout child did not exit"


@pytest.mark.parametrize("mode", ["bf16", "fp8"])
def test_multicast_team_in_one_process(two_gpus, sock_path, mode):
    """Trainer on cuda:0 and two rollout buffers (cuda:1 and a second one on
    cuda:0) in one process: a two-GPU team, one K4 launch with multimem.st
    stores fills both."""
    from statespectre_b200 import in_process_daemon, offload_context
    from statespectre_b200.parallel import fabric
    from statespectre_b200.parallel.weight_sync import RolloutWeights, TrainerWeightSync, WeightLayout

    if not (fabric.multicast_supported(0) and fabric.multicast_supported(1)):
        pytest.skip("no switch multicast on these GPUs")
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="wsync-mc2") as off:
            torch.manual_seed(1)
            params = {n: (torch.randn(s, device="cuda:0") * 0.02).to(getattr(torch, dt)) for n, s, dt in _specs()}
            layout = WeightLayout.from_params(params, mode)
            rws = [RolloutWeights(layout, "cuda:1"), RolloutWeights(layout, "cuda:0")]
            keys = [f"rollout/mc2/{mode}/{i}" for i in range(2)]
            for rw, k in zip(rws, keys):
                rw.publish(off, k)
            tr = TrainerWeightSync(off, params, keys, mode=mode, persist=False)  # auto: 2 replicas -> multicast
            assert tr.transport == "multicast" and tr.team.ndevices == 2 and tr.team.scratch is None
            assert len(tr.pushers) == 1
            tr.publish_version(1)
            full = tr.pushers[0].result()["bytes_stored"]
            params["w1"].add_(0.5)
            r2 = tr.publish_version(2)
            assert r2["changed"] == 1
            assert tr.pushers[0].result()["bytes_stored"] - full == params["w1"].numel() * 2
            torch.cuda.synchronize(0)
            torch.cuda.synchronize(1)
            for rw in rws:
                for n, t in params.items():
                    if mode == "bf16" or not layout.by_name[n].quant:
                        assert torch.equal(rw.get(n).to("cuda:0"), t), n
                    else:
                        got = rw.dequantized(n).float().to("cuda:0")
                        assert torch.allclose(got, t.float(), rtol=0.07, atol=1e-6), n
                if mode == "bf16":
                    assert rw.content_hashes() == tr.pushers[0].hashes()
            tr.close()
            for rw in rws:
                rw.close()
    finally:
        d.stop()


def _dedup_rank(rank, sock, pg_file, q_out):
    import torch
    import torch.distributed as dist

    from statespectre_b200 import DedupPolicy, offload_context
    from statespectre_b200.parallel.dp_dedup import dedup_evict_params

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{pg_file}", rank=rank, world_size=2)
    res = {}
    try:
        with offload_context(daemon_addr=sock, device=f"cuda:{rank}", rank=rank, job_name="dp2") as off:
            g = torch.Generator(device=f"cuda:{rank}").manual_seed(0)  # same weights on both replicas
            params = {f"w{i}": torch.randn(1000 + 333 * i, 96, device=f"cuda:{rank}", generator=g)
                      .to(torch.bfloat16) for i in range(6)}
            pol = DedupPolicy("p2p_verified")
            hs = dedup_evict_params(off, params, model_role="policy_trainable", model_version=1, policy=pol,
                                    destructive=False)
            res["actions"] = {n: h.action_name for n, h in hs.items()}
            res["restored_equal"] = all(
                torch.equal(hs[n].restore_into(torch.empty_like(t)), t) for n, t in params.items())
            res["p2p_verified"] = off.daemon_stats().get("canonical_p2p_verified_total")
            if rank == 1:
                params["w0"].view(-1)[12345] += 1  # w0 is owned by rank 0: rank 1's copy now differs
            try:
                dedup_evict_params(off, params, model_role="policy_trainable", model_version=2, policy=pol,
                                   destructive=False)
                res["mismatch"] = None
            except RuntimeError as e:
                res["mismatch"] = str(e)
        q_out.put((rank, res))
    except Exception as e:  # noqa: BLE001
        q_out.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_dp_dedup_verifies_replicas_by_peer_byte_compare(two_gpus, sock_path, tmp_path):
    """p2p_verified: the owner of each parameter copies it to the host; the
    other replica compares its bytes with the owner's GPU copy over NVLink
    (K3) and attaches. A replica whose bytes differ is reported on both
    ranks, by name."""
    from statespectre_b200 import in_process_daemon

    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    procs = [ctx.Process(target=_dedup_rank, args=(r, sock_path, str(tmp_path / "pg"), q_out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = dict(q_out.get(timeout=TIMEOUT) for _ in range(2))
        for p in procs:
            p.join(TIMEOUT)
            assert p.exitcode == 0
    finally:
        for p in procs:  # point-to-point only (no multicast object): a stuck child may be killed
            if p.is_alive():
                p.kill()
                p.join(10)
        d.stop()
    for r in (0, 1):
        assert "error" not in got[r], got[r]
        acts = got[r]["actions"]
        for i in range(6):
            want = "NEED_D2H_CREATE" if i % 2 == r else "VERIFIED_BY_P2P"
            assert acts[f"w{i}"] == want, (r, acts)
        assert got[r]["restored_equal"]
        assert got[r]["mismatch"] is not None and "w0" in got[r]["mismatch"]
    assert max(got[0]["p2p_verified"], got[1]["p2p_verified"]) == 6  # every parameter verified once
