"""Evict/restore size sweep on every GPU of the job.

Workload: bf16 tensors with N(0,1) values (``--dtype fp32``: fp32 with
N(0, 0.02) values, zf32-coded), sizes powers of two from 4 KB to
8 GB (``--max-size-mb``), evicted into the GPU's pinned window (fused content
hash; bf16 payloads zbf16-coded) and restored, ``--steps`` repeats per size,
while an 8192x8192 bf16 GEMM loop runs on the same GPU. Each direction is
timed with CUDA events on the copy stream (the agent's kernels and its
waits are inside the timed region); the reported rate per size is the median
over repeats of the slowest rank. ``value`` is the round-trip rate at the
1 GiB point (the headline size).

    python bench.py --workload sweep --steps 20 --warmup 3 --arena-gb 64 [--compress 0]
    python bench.py --impl reference --workload sweep ...   # the reference, same sizes and timing
"""

from __future__ import annotations

import statistics

import torch

from .. import offload_context
from .._native import native
from ..utils.clocks import ClockSampler
from ..utils.load import GemmLoad
from .common import DeviceTimer, node_daemon, setup

GiB = 1 << 30


def run(args, metric: str) -> dict:
    env = setup()
    max_bytes = (args.max_size_mb or 8192) << 20
    sizes = []
    s = 4096
    while s <= max_bytes:
        sizes.append(s)
        s <<= 1
    window_gb = max(int(getattr(args, "arena_gb", 0) or 0), int(3 * max_bytes / GiB) + 2)
    sock, daemon = node_daemon(env, window_gb, "/tmp/ofld_sweep", slot_mb=64)
    sess = offload_context(daemon_addr=sock, device=env.device, rank=env.rank, local_rank=env.local_rank,
                           world_rank=env.rank, eager_register=True, compress=bool(args.compress),
                           hash_on_evict=bool(getattr(args, "hash", 1)),
                           stream_priority=-1, stage_ctas=int(getattr(args, "stage_ctas", 0) or 0),
                           stage_depth=int(getattr(args, "stage_depth", 0) or 0),
                           stage_piece_chunks=int(getattr(args, "stage_piece_chunks", 0) or 0),
                           **({"host_hash_max_bytes": int(args.host_hash_kb) << 10}
                              if getattr(args, "host_hash_kb", -1) >= 0 else {}))
    off = sess.off
    stream = torch.cuda.Stream(device=env.device, priority=-1)
    load = GemmLoad(env.device).start() if args.matmul else None
    g = torch.Generator(device=env.device).manual_seed(1234 + env.rank)
    rows = []
    fp32 = getattr(args, "dtype", "bf16") == "fp32"
    launches0 = native().kernel_launch_count()
    sampler = ClockSampler([env.local_rank]).start().wait_first()
    sampler.mark_start()
    for nbytes in sizes:
        if fp32:
            x = torch.randn(nbytes // 4, dtype=torch.float32, device=env.device, generator=g) * 0.02
        else:
            x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=env.device, generator=g)
        ref = off.hash_tensor(x)
        ev, rs = [], []
        coded = False
        for i in range(args.warmup + args.steps):
            env.barrier()
            with DeviceTimer(stream) as te:
                h = off.copy(x, stream=stream, wait=True)
            with DeviceTimer(stream) as tr:
                h.restore_into(x, stream=stream, wait=True)
            coded = h.coded
            h.discard()
            if i >= args.warmup:
                ev.append(env.max(te.ms()))
                rs.append(env.max(tr.ms()))
        torch.cuda.synchronize(env.device)
        ok = off.hash_tensor(x) == ref
        e_ms, r_ms = statistics.median(ev), statistics.median(rs)
        rows.append({"bytes": nbytes, "evict_gbs": round(nbytes / (e_ms / 1e3) / 1e9, 3),
                     "restore_gbs": round(nbytes / (r_ms / 1e3) / 1e9, 3),
                     "evict_ms": round(e_ms, 4), "restore_ms": round(r_ms, 4), "coded": coded, "byte_exact": ok})
        del x
    sampler.mark_end()
    clocks = sampler.stop()
    launches = env.sum(native().kernel_launch_count() - launches0)
    mm = load.stop() if load else 0
    sess.close()
    env.barrier()
    if daemon is not None:
        daemon.stop()
    env.close()
    if env.rank != 0:
        return None
    head = next((r for r in rows if r["bytes"] == GiB), rows[-1])
    rt = 2 * head["bytes"] / ((head["evict_ms"] + head["restore_ms"]) / 1e3) / 1e9
    return {
        "metric": metric, "workload": "sweep", "value": round(rt * env.world, 3),
        "unit": "GB/s (aggregate round trip at the 1 GiB point; per-size rows below)",
        "n_gpus": env.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(head["evict_ms"] + head["restore_ms"], 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32" if fp32 else "bf16",
        "data": "synthetic: fp32 N(0, 0.02) per size, seeded per rank" if fp32
                else "synthetic: bf16 N(0,1) per size, seeded per rank",
        "config": {"model": f"evict/restore size sweep 4 KB - max size, {'fp32' if fp32 else 'bf16'}", "max_bytes": max_bytes,
                   "arena_gb_per_gpu": window_gb, "transfer_coding": ("zf32" if fp32 else "zbf16") + " where it codes" if args.compress
                   else "none (--compress 0)",
                   "concurrent_matmul": load.describe() if load else "none", "global_batch": env.world,
                   "seq_len": 0, "parallelism": f"dp{env.world}", "slot_mb": 64,
                   "l2": "sizes above 126 MB stream from HBM; smaller ones may hit L2 (reported as measured)"},
        "sweep": rows, "all_byte_exact": all(r["byte_exact"] for r in rows),
        "gpu_launches": int(launches), "clocks": clocks, "matmul_iters": mm,
    }
