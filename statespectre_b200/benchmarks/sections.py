"""Per-subsystem sections of the offload path on one GPU.

The same sections StateSpectre's C++ benchmark reports (reference:
tests/cpp/bench.cpp; its numbers: docs/PERFORMANCE.md), each timed here on
this runtime's real path:

  reg    eager CUDA registration of an 8 GiB pinned window, one thread and
         ``registration_threads`` pieces in parallel (ms per GiB)
  d2h    evict / restore of bf16 N(0,1) tensors of 1 and 8 GiB (device time;
         zbf16-coded K1/K2)
  drain  pinned -> pageable drain of 8 x 1 GiB by the daemon's workers, then
         restore through readback (pageable -> pinned -> device)
  nvme   spill of 4 x 1 GiB to ``--nvme-dir`` (io_uring, O_DIRECT where the
         filesystem allows it) and restore through NVMe readback
  burst  four sessions on this GPU evicting 4 x 1 GiB each at once
  numa   local vs remote NUMA arena (skipped on a single-node host)

Every section prints a ``BENCH,<section>,key=value,...`` line on stderr; the
JSON line carries them all. ``value`` is the 1 GiB evict+restore round trip.

    python bench.py --workload sections [--nvme-dir /nvme/ofld]
"""

from __future__ import annotations

import shutil
import sys
import threading
import time

import torch

from .. import offload_context
from .._native import native
from ..utils.clocks import ClockSampler
from ..utils.topology import gpu_numa_nodes, host_numa_nodes
from .common import DeviceTimer, node_daemon, setup

GiB = 1 << 30


def _emit(section: str, **kv) -> dict:
    print("BENCH," + section + "," + ",".join(f"{k}={v}" for k, v in kv.items()), file=sys.stderr, flush=True)
    return kv


def _wait_location(hs, want: str, timeout: float) -> bool:
    deadline = time.time() + timeout
    while time.time() < deadline:
        if all(h.location() == want for h in hs):
            return True
        time.sleep(0.002)
    return False


def _bf16(n_bytes: int, device, seed: int) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(n_bytes // 2, dtype=torch.bfloat16, device=device, generator=g)


def run(args, metric: str) -> dict:
    env = setup()
    if env.world != 1:
        raise SystemExit("sections runs on one GPU")
    dev = env.device
    out = {}
    launches0 = native().kernel_launch_count()
    sampler = ClockSampler([env.local_rank]).start().wait_first()
    sampler.mark_start()

    # ---- reg ----
    reg = {}
    for threads in (1, 8):
        sock, d = node_daemon(env, 8, f"/tmp/ofld_sec_reg{threads}", slot_mb=64)
        s = offload_context(daemon_addr=sock, device=dev, rank=0, eager_register=True, registration_threads=threads)
        st = s.off._agent.stats()
        gib = st["registered_pinned_bytes"] / GiB
        reg[f"threads_{threads}_ms_per_gib"] = round(st["registration_ns"] / 1e6 / max(gib, 1e-9), 2)
        s.close()
        d.stop()
    reg["window_gib"] = round(gib, 2)
    out["reg"] = _emit("reg", **reg)

    # ---- d2h / h2d ----
    sock, d = node_daemon(env, 20, "/tmp/ofld_sec_xfer", slot_mb=64)
    s = offload_context(daemon_addr=sock, device=dev, rank=0, eager_register=True, stream_priority=-1)
    stream = torch.cuda.Stream(device=dev, priority=-1)
    rows = []
    for gib_n in (1, 8):
        x = _bf16(gib_n * GiB, dev, 10 + gib_n)
        ev, rs = [], []
        for i in range(4):
            with DeviceTimer(stream) as te:
                h = s.off.copy(x, stream=stream, wait=True)
            with DeviceTimer(stream) as tr:
                h.restore_into(x, stream=stream, wait=True)
            h.discard()
            if i:
                ev.append(te.ms())
                rs.append(tr.ms())
        rows.append(_emit("d2h", gib=gib_n, d2h_gbs=round(gib_n * GiB / (min(ev) / 1e3) / 1e9, 2),
                          h2d_gbs=round(gib_n * GiB / (min(rs) / 1e3) / 1e9, 2), coded=h.coded))
        del x
    out["d2h"] = rows
    s.close()
    d.stop()

    # ---- drain (pinned -> pageable) and readback ----
    sock, d = node_daemon(env, 10, "/tmp/ofld_sec_drain", slot_mb=64, drain_on_complete=True)
    s = offload_context(daemon_addr=sock, device=dev, rank=0, eager_register=True, compress=False)
    xs = [_bf16(GiB, dev, 100 + i) for i in range(8)]
    refs = [s.off.hash_tensor(x) for x in xs]
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    hs = [s.off.copy(x, wait=True) for x in xs]
    t1 = time.perf_counter()
    ok = _wait_location(hs, "pageable", 300)
    t2 = time.perf_counter()
    for x, h in zip(xs, hs):
        h.restore_into(x, wait=True)
    torch.cuda.synchronize(dev)
    t3 = time.perf_counter()
    exact = all(s.off.hash_tensor(x) == r for x, r in zip(xs, refs))
    stats = s.off.daemon_stats()
    out["drain"] = _emit("drain", gib=8, drained=ok, evict_gbs=round(8 * GiB / (t1 - t0) / 1e9, 2),
                         drain_gbs=round(8 * GiB / (t2 - t0) / 1e9, 2),
                         readback_restore_gbs=round(8 * GiB / (t3 - t2) / 1e9, 2),
                         pageable_bytes=stats.get("pinned_to_pageable_bytes"),
                         readback_bytes=stats.get("pageable_to_pinned_bytes"), byte_exact=exact)
    for h in hs:
        h.discard()
    del xs
    s.close()
    d.stop()

    # ---- nvme ----
    nvme_dir = args.nvme_dir or "/tmp/ofld_sec_nvme"
    shutil.rmtree(nvme_dir, ignore_errors=True)
    sock, d = node_daemon(env, 6, "/tmp/ofld_sec_nvme_run", slot_mb=64, drain_on_complete=True,
                          drain_target="nvme", nvme_dir=nvme_dir)
    s = offload_context(daemon_addr=sock, device=dev, rank=0, eager_register=True, compress=False)
    xs = [_bf16(GiB, dev, 200 + i) for i in range(4)]
    refs = [s.off.hash_tensor(x) for x in xs]
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    hs = [s.off.copy(x, wait=True) for x in xs]
    ok = _wait_location(hs, "nvme", 600)
    t1 = time.perf_counter()
    for x, h in zip(xs, hs):
        h.restore_into(x, wait=True)
    torch.cuda.synchronize(dev)
    t2 = time.perf_counter()
    exact = all(s.off.hash_tensor(x) == r for x, r in zip(xs, refs))
    stats = s.off.daemon_stats()
    out["nvme"] = _emit("nvme", gib=4, dir=nvme_dir, spilled=ok, write_gbs=round(4 * GiB / (t1 - t0) / 1e9, 2),
                        read_restore_gbs=round(4 * GiB / (t2 - t1) / 1e9, 2),
                        nvme_write_bytes=stats.get("nvme_write_bytes"), nvme_read_bytes=stats.get("nvme_read_bytes"),
                        io_failures=stats.get("io_failure"), byte_exact=exact)
    for h in hs:
        h.discard()
    del xs
    s.close()
    d.stop()
    shutil.rmtree(nvme_dir, ignore_errors=True)

    # ---- burst: four sessions on one GPU ----
    sock, d = node_daemon(env, 20, "/tmp/ofld_sec_burst", slot_mb=64)
    # every session maps and registers the arena before the timed burst
    sessions = [offload_context(daemon_addr=sock, device=dev, rank=r, eager_register=True) for r in range(4)]
    data = [[_bf16(GiB, dev, 300 + 4 * r + i) for i in range(4)] for r in range(4)]
    torch.cuda.synchronize(dev)
    handles = [[] for _ in range(4)]
    errs = []

    def burst(r):
        try:
            torch.cuda.set_device(dev)
            st = torch.cuda.Stream(device=dev)
            for x in data[r]:
                handles[r].append(sessions[r].off.copy(x, stream=st, wait=True))
        except Exception as e:  # noqa: BLE001
            errs.append(repr(e))

    t0 = time.perf_counter()
    ths = [threading.Thread(target=burst, args=(r,)) for r in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    t1 = time.perf_counter()
    out["burst"] = _emit("burst", ranks=4, gib_per_rank=4, aggregate_d2h_gbs=round(16 * GiB / (t1 - t0) / 1e9, 2),
                         wall_s=round(t1 - t0, 3), errors=len(errs))
    for hl in handles:
        for h in hl:
            h.discard()
    del data
    for ss in sessions:
        ss.close()
    d.stop()

    # ---- numa ----
    nodes = host_numa_nodes()
    if len(nodes) < 2:
        out["numa"] = _emit("numa", skipped="single NUMA node", nodes=len(nodes))
    else:
        local = gpu_numa_nodes(1)[0]
        remote = next(n for n in nodes if n != local)
        res = {}
        for tag, node in (("local", local), ("remote", remote)):
            sock, d = node_daemon(env, 4, f"/tmp/ofld_sec_numa_{tag}", slot_mb=64)
            s = offload_context(daemon_addr=sock, device=dev, rank=0, eager_register=True, numa_node=node)
            x = _bf16(GiB, dev, 400)
            st = torch.cuda.Stream(device=dev)
            with DeviceTimer(st) as te:
                h = s.off.copy(x, stream=st, wait=True)
            with DeviceTimer(st) as tr:
                h.restore_into(x, stream=st, wait=True)
            res[f"{tag}_d2h_gbs"] = round(GiB / (te.ms() / 1e3) / 1e9, 2)
            res[f"{tag}_h2d_gbs"] = round(GiB / (tr.ms() / 1e3) / 1e9, 2)
            h.discard()
            s.close()
            d.stop()
        out["numa"] = _emit("numa", **res)

    sampler.mark_end()
    clocks = sampler.stop()
    launches = native().kernel_launch_count() - launches0
    head = out["d2h"][0]
    rt = 2 / (1 / head["d2h_gbs"] + 1 / head["h2d_gbs"])
    return {
        "metric": metric, "workload": "sections", "value": round(rt, 3),
        "unit": "GB/s (1 GiB evict+restore round trip; per-section results below)",
        "n_gpus": 1, "steps": 3, "warmup": 1, "ms_per_step": round(2 * GiB / (rt * 1e9) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: bf16 N(0,1) tensors, seeded",
        "config": {"model": "offload path sections: reg, d2h, drain, nvme, burst, numa", "global_batch": 1,
                   "seq_len": 0, "parallelism": "dp1", "slot_mb": 64,
                   "l2": "GiB-sized transfers; no flush needed"},
        "sections": out, "gpu_launches": int(launches), "clocks": clocks,
    }
