"""Control-plane throughput of the daemon (no GPU needed).

Host-mode sessions move small tensors so that the daemon's request handling,
not the data copy, is what is measured:

  single   evict + restore + discard of a 4 KiB tensor, one call each
           (reservation, completion, prefetch and discard round trips):
           round trips per second and p50 / p99 latency
  batch    evict_batch + restore_batch + discard_batch of 256 x 4 KiB
           tensors: items per second, per phase
  ranks    the single loop in 1, 4 and 16 rank processes at once: aggregate rate
  vs_reference  the single loop against StateSpectre's own daemon (built in
           baseline/_ref) and this one, both as separate processes, with
           the same client (held to StateSpectre's opcodes for the first two)
  kv       8 rank processes, each moving its own 64 blocks of 256 KiB per
           iteration with evict_batch + restore_batch, against a pinned
           window half the size of the blocks in flight, so background
           pressure drains and readbacks run under the request load: items per
           second in aggregate, per-iteration p50 / p99, drains and readbacks

StateSpectre needs two RPCs per evict and one per restore on its one-mutex
daemon; the paged KV-cache workload (about 10k block moves per GPU per
iteration on 8 GPUs) is what these numbers have to carry.

    python -m statespectre_b200.benchmarks.control [--seconds 2] [--out control.json]
"""

from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import tempfile
import time

import torch

from .. import DaemonClient, in_process_daemon, offload_context


def _single(sock: str, rank: int, seconds: float, lat: list, barrier=None) -> int:
    n = 0
    with offload_context(daemon_addr=sock, device="cpu", rank=rank) as off:
        t = torch.randn(1024)
        out = torch.empty_like(t)
        if barrier is not None:
            barrier.wait(120)  # every rank's session is open: start together
        deadline = time.perf_counter() + seconds
        while time.perf_counter() < deadline:
            t0 = time.perf_counter()
            h = off.copy(t, wait=True)
            h.restore_into(out)
            h.discard()
            lat.append(time.perf_counter() - t0)
            n += 1
    return n


def run(seconds: float = 2.0, rank_counts=(1, 4, 16)) -> dict:
    tmp = tempfile.mkdtemp(prefix="ofld-control-")
    sock = os.path.join(tmp, "d.sock")
    d = in_process_daemon(socket=sock, arena_mb=256, slot_mb=1, drain_on_complete=False)
    out = {}
    try:
        lat: list = []
        n = _single(sock, 0, seconds, lat)
        lat.sort()
        out["single"] = {"round_trips_per_s": round(n / seconds, 1),
                         "p50_us": round(lat[len(lat) // 2] * 1e6, 1),
                         "p99_us": round(lat[min(len(lat) - 1, int(0.99 * len(lat)))] * 1e6, 1)}
        with offload_context(daemon_addr=sock, device="cpu", rank=0) as off:
            ts = [torch.randn(1024) for _ in range(256)]
            outs = [torch.empty_like(t) for t in ts]
            items = 0
            t_ev = t_rs = t_dc = 0.0
            deadline = time.perf_counter() + seconds
            while time.perf_counter() < deadline:
                t0 = time.perf_counter()
                hs = off.evict_batch(ts)
                t1 = time.perf_counter()
                off.restore_batch(hs, outs)
                t2 = time.perf_counter()
                off.discard_batch(hs)
                t3 = time.perf_counter()
                t_ev += t1 - t0
                t_rs += t2 - t1
                t_dc += t3 - t2
                items += len(ts)
            out["batch"] = {"batch": len(ts), "items_per_s": round(items / (t_ev + t_rs + t_dc), 1),
                            "evict_items_per_s": round(items / t_ev, 1),
                            "restore_items_per_s": round(items / t_rs, 1),
                            "discard_items_per_s": round(items / t_dc, 1)}
        # ranks in separate processes (one Python interpreter each, like real ranks)
        ctx = mp.get_context("spawn")
        ranks = {}
        for r in rank_counts:
            q = ctx.Queue()
            bar = ctx.Barrier(r)
            procs = [ctx.Process(target=_rank_proc, args=(sock, 100 + i, seconds, q, bar)) for i in range(r)]
            for p in procs:
                p.start()
            res = [q.get(timeout=seconds + 120) for _ in procs]
            for p in procs:
                p.join(30)
            ranks[str(r)] = {"round_trips_per_s": round(sum(n for n, _ in res) / seconds, 1),
                             "p50_us": round(statistics.median([m for _, m in res]) * 1e6, 1)}
        out["ranks"] = ranks
    finally:
        d.stop()
    return out


def _kv_rank(sock: str, rank: int, seconds: float, nblocks: int, block: int, q, barrier) -> None:
    try:
        _kv_loop(sock, rank, seconds, nblocks, block, q, barrier)
    except Exception as e:  # noqa: BLE001
        q.put((0, [], repr(e)))


def _kv_loop(sock: str, rank: int, seconds: float, nblocks: int, block: int, q, barrier) -> None:
    lat = []
    n = 0
    with offload_context(daemon_addr=sock, device="cpu", rank=rank) as off:
        g = torch.Generator().manual_seed(rank)
        blocks = [torch.randn(block // 4, generator=g) for _ in range(nblocks)]
        ref = [b.clone() for b in blocks]
        barrier.wait(120)
        deadline = time.perf_counter() + seconds
        while time.perf_counter() < deadline:
            t0 = time.perf_counter()
            hs = off.evict_batch(blocks)
            off.restore_batch(hs, blocks)
            off.discard_batch(hs)
            lat.append(time.perf_counter() - t0)
            n += nblocks
        ok = all(torch.equal(a, b) for a, b in zip(blocks, ref))
    q.put((n, lat, ok))


def run_kv(seconds: float = 3.0, ranks: int = 8, nblocks: int = 64, block: int = 256 << 10) -> dict:
    tmp = tempfile.mkdtemp(prefix="ofld-control-kv-")
    sock = os.path.join(tmp, "d.sock")
    window_mb = max(4, ranks * nblocks * block // 2 >> 20)
    d = in_process_daemon(socket=sock, arena_mb=window_mb, slot_mb=1, drain_on_complete=False)
    try:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        bar = ctx.Barrier(ranks)
        procs = [ctx.Process(target=_kv_rank, args=(sock, 200 + i, seconds, nblocks, block, q, bar))
                 for i in range(ranks)]
        for p in procs:
            p.start()
        res = [q.get(timeout=seconds + 180) for _ in procs]
        for p in procs:
            p.join(30)
        c = DaemonClient(sock)
        stats = c.stats()
        c.close()
    finally:
        d.stop()
    lat = sorted(x for _, ls, _ in res for x in ls)
    items = sum(n for n, _, _ in res)
    return {"ranks": ranks, "blocks_per_rank": nblocks, "block_bytes": block, "pinned_window_mb": window_mb,
            "items_per_s": round(items / seconds, 1),
            "iteration_p50_ms": round(lat[len(lat) // 2] * 1e3, 2) if lat else None,
            "iteration_p99_ms": round(lat[min(len(lat) - 1, int(0.99 * len(lat)))] * 1e3, 2) if lat else None,
            "drains": stats.get("drains_completed"), "readbacks": stats.get("readbacks_completed"),
            "byte_exact": all(ok is True for _, _, ok in res),
            "errors": [ok for _, _, ok in res if ok is not True and ok is not False]}


REF_DAEMON = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                          "baseline", "_ref", "bin", "offloadd")


def _external_daemon(binary: str, tag: str):
    """`binary` as its own process on a 1 GiB window, no drain on completion."""
    import subprocess

    d = tempfile.mkdtemp(prefix=f"ofld-control-{tag}-")
    sock, cfg = os.path.join(d, "d.sock"), os.path.join(d, "offloadd.yaml")
    with open(cfg, "w") as f:
        f.write("\n".join(["daemon:", f"  socket_path: {sock}", f"  control_shm_name: /ofld_cp_{os.getpid()}_{tag}",
                           "arenas:", "  allocation_granularity_mb: 1", "  per_numa:", "    - numa_node: 0",
                           "      size_gb: 1", "      overflow_gb: 0", "      gpu_windows:", "        - gpu: 0",
                           "          size_gb: 1", "drain_policy:", "  drain_on_d2h_complete: false", "nvme:",
                           "  enabled: false"]) + "\n")
    p = subprocess.Popen([binary, "--config", cfg, "--socket", sock], stdout=subprocess.DEVNULL,
                         stderr=subprocess.DEVNULL)
    deadline = time.time() + 30
    while not os.path.exists(sock) and time.time() < deadline and p.poll() is None:
        time.sleep(0.05)
    return p, sock


def run_vs_reference(seconds: float = 2.0) -> dict:
    """The single-tensor cycle (copy, restore_into, discard of 4 KiB) with the
    same client against StateSpectre's own daemon (the session speaks its
    opcodes only), against this daemon with the session held to the same
    opcodes, and against this daemon with everything on (reservation and
    submit in one round trip, completions through the shared ring)."""
    from .._native import bin_path

    if not os.path.exists(REF_DAEMON):
        return {"unavailable": "reference build not present (python baseline/build_reference.py)"}
    out = {}
    for name, binary, v1 in (("reference_daemon", REF_DAEMON, True), ("this_daemon_v1_only", bin_path("offloadd"), True),
                             ("this_daemon", bin_path("offloadd"), False)):
        p, sock = _external_daemon(binary, name)
        try:
            with offload_context(daemon_addr=sock, device="cpu", rank=0, v1_only=v1) as off:
                t = torch.randn(1024)
                dst = torch.empty_like(t)
                lat = []
                deadline = time.perf_counter() + seconds
                while time.perf_counter() < deadline:
                    t0 = time.perf_counter()
                    h = off.copy(t, wait=True)
                    h.restore_into(dst)
                    h.discard()
                    lat.append(time.perf_counter() - t0)
                # 256 blocks of 4 KiB per batch call (KV-cache style); against
                # StateSpectre's daemon each batch call is one call per block
                blocks = [torch.randn(1024) for _ in range(256)]
                outs = [torch.empty_like(b) for b in blocks]
                items, t_total = 0, 0.0
                deadline = time.perf_counter() + seconds
                while time.perf_counter() < deadline:
                    t0 = time.perf_counter()
                    hs = off.evict_batch(blocks)
                    off.restore_batch(hs, outs)
                    off.discard_batch(hs)
                    t_total += time.perf_counter() - t0
                    items += len(blocks)
            lat.sort()
            out[name] = {"cycles_per_s": round(len(lat) / seconds, 1), "p50_us": round(lat[len(lat) // 2] * 1e6, 1),
                         "p99_us": round(lat[min(len(lat) - 1, int(0.99 * len(lat)))] * 1e6, 1),
                         "batch_items_per_s": round(items / t_total, 1)}
        finally:
            p.terminate()
            p.wait(30)
    return out


def _rank_proc(sock: str, rank: int, seconds: float, q, barrier) -> None:
    lat: list = []
    n = _single(sock, rank, seconds, lat, barrier)
    q.put((n, statistics.median(lat) if lat else 0.0))


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--seconds", type=float, default=2.0)
    p.add_argument("--out", default="")
    a = p.parse_args(argv)
    res = run(a.seconds)
    res["kv"] = run_kv(max(a.seconds, 3.0))
    res["vs_reference"] = run_vs_reference(a.seconds)
    line = json.dumps({"benchmark": "control_plane", **res})
    print(line)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
