"""Control-plane throughput of the daemon (no GPU needed).

Host-mode sessions move small tensors so that the daemon's request handling,
not the data copy, is what is measured:

  single   evict + restore + discard of a 4 KiB tensor, one call each
           (reservation, completion, prefetch and discard round trips):
           round trips per second and p50 / p99 latency
  batch    evict_batch + restore_batch + discard_batch of 256 x 4 KiB
           tensors: items per second, per phase
  ranks    the single loop in 1, 4 and 16 rank processes at once: aggregate rate

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

from .. import in_process_daemon, offload_context


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
    line = json.dumps({"benchmark": "control_plane", **res})
    print(line)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
