"""Several rank processes share one daemon without cross-talk
(the shape of StateSpectre's multi-process test, reference:
tests/python/test_multiproc.py:57-90), plus a gloo process group exercising
the rank-coordinated canonical flow."""

import multiprocessing as mp
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(sock, rank, n, q):
    sys.path.insert(0, ROOT)
    import torch

    from statespectre_b200 import offload_context

    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=rank) as off:
            xs = [torch.full((4096 + i,), float(rank * 1000 + i)) for i in range(n)]
            hs = [off.copy(x) for x in xs]  # asynchronous
            off.wait(hs)
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
                h.discard()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_four_processes_twenty_tensors_each(tmp_path):
    from statespectre_b200 import launch_daemon

    sock = str(tmp_path / "d.sock")
    with launch_daemon(sock, arena_mb=128, drain_on_complete=False) as d:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_worker, args=(sock, r, 20, q)) for r in range(4)]
        [p.start() for p in ps]
        res = dict(q.get(timeout=120) for _ in ps)
        [p.join(timeout=60) for p in ps]
        assert res == {r: "ok" for r in range(4)}
        s = d.stats()
        assert s["d2h_bytes"] == sum(4 * (4096 + i) for i in range(20)) * 4
        assert s["used_slots"] == 0


def _dp_worker(rank, world, port, sock, q):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from statespectre_b200 import DedupPolicy, ModelRole, offload_context

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        from statespectre_b200.parallel.dp_dedup import dedup_evict_params

        torch.manual_seed(0)  # every DP replica holds identical weights
        params = {f"layer{i}.w": torch.randn(256, 64) for i in range(6)}
        with offload_context(daemon_addr=sock, device="cpu", rank=rank, job_name="dp") as off:
            out = dedup_evict_params(off, params, model_role=ModelRole.POLICY_TRAINABLE, model_version=1,
                                     policy=DedupPolicy("device_hash_verified"), group=None, owner="rank0")
            q.put((rank, sorted(h.action_name for h in out.values())))
            dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 3])
def test_dp_dedup_over_gloo(tmp_path, world):
    from statespectre_b200 import launch_daemon

    sock = str(tmp_path / "d.sock")
    import socket as s

    with s.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    with launch_daemon(sock, arena_mb=128, drain_on_complete=False) as d:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_dp_worker, args=(r, world, port, sock, q)) for r in range(world)]
        [p.start() for p in ps]
        res = dict(q.get(timeout=180) for _ in ps)
        [p.join(timeout=60) for p in ps]
        owners = [r for r, acts in res.items() if acts == ["NEED_D2H_CREATE"] * 6]
        verifiers = [r for r, acts in res.items() if acts == ["VERIFIED_BY_DEVICE_HASH"] * 6]
        assert owners == [0] and len(verifiers) == world - 1, res
        st = d.stats()
        assert st["canonical_objects_created_total"] == 6
        assert st["d2h_bytes"] == 6 * 256 * 64 * 4  # only the owner copied
