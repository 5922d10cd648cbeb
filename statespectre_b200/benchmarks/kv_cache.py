"""Paged KV-cache offload under load, on every GPU of the job.

Workload: a paged KV cache of 16-token blocks x 64 layers x 8 KV heads x
head_dim 128, bf16 N(0,1) (4 MiB per block), ``--kv-gb`` per GPU (default
40 GB). Every iteration a seeded random ``--evict-fraction`` of the blocks is
evicted and restored into place with one ``evict_batch``/``restore_batch``
call each (``--kv-batch`` splits it; the agent reserves and launches in
groups of 256 MiB, one round trip and one kernel launch per group) while a
bf16 GEMM loop stands in for the training step. The pinned
window per GPU is ``--pinned-gb``: when it is smaller than the evicted set,
the daemon drains to pageable DRAM (and NVMe when enabled) and restores read
back, exercising the tiers. Device time per iteration is the max over ranks.

    python bench.py --workload kv_cache --steps 10 --warmup 2 --kv-gb 40
"""

from __future__ import annotations

import statistics

import torch

from .. import offload_context
from .._native import native
from ..models.shapes import KVCacheSpec
from ..utils.clocks import ClockSampler
from ..utils.load import GemmLoad
from .common import DeviceTimer, node_daemon, setup

GiB = 1 << 30


def run(args, metric: str) -> dict:
    env = setup()
    spec = KVCacheSpec()
    kv_bytes = int(args.kv_gb * GiB)
    nblocks = spec.blocks_for(kv_bytes)
    per_iter = max(1, int(round(args.evict_fraction * nblocks)))
    batch = args.kv_batch if args.kv_batch > 0 else per_iter
    pinned_gb = args.pinned_gb or int(per_iter * spec.block_bytes * 1.2 / GiB) + 2
    sock, daemon = node_daemon(env, pinned_gb, "/tmp/ofld_kv", slot_mb=4,
                               tier_threads=getattr(args, "tier_threads", ""))
    sess = offload_context(daemon_addr=sock, device=env.device, rank=env.rank, local_rank=env.local_rank,
                           world_rank=env.rank, eager_register=True, stream_priority=-1,
                           kernel_timing=bool(getattr(args, "kernel_timing", 0)),
                           evict_ctas=int(getattr(args, "evict_ctas", 0)),
                           restore_ctas=int(getattr(args, "restore_ctas", 0)),
                           compress=bool(getattr(args, "compress", 1)),
                           uncoded=getattr(args, "uncoded", "copy_engine"),
                           **({"batch_group_bytes": int(args.kv_group_mb) << 20}
                              if getattr(args, "kv_group_mb", 0) else {}))
    off = sess.off
    stream = torch.cuda.Stream(device=env.device, priority=-1)
    g = torch.Generator(device=env.device).manual_seed(99 + env.rank)
    cache = torch.randn(nblocks, spec.block_bytes // 2, dtype=torch.bfloat16, device=env.device, generator=g)
    ref = off.hash_tensor(cache)
    load = GemmLoad(env.device).start() if args.matmul else None
    host_gen = torch.Generator().manual_seed(7 + env.rank)

    def iteration():
        idx = torch.randperm(nblocks, generator=host_gen)[:per_iter].tolist()
        blocks = [cache[i] for i in idx]
        with DeviceTimer(stream) as te:
            handles = []
            for j in range(0, len(blocks), batch):
                handles += off.evict_batch(blocks[j:j + batch], stream=stream, wait=True)
        with DeviceTimer(stream) as tr:
            for j in range(0, len(blocks), batch):
                off.restore_batch(handles[j:j + batch], blocks[j:j + batch], stream=stream, wait=True)
        off.discard_batch(handles)
        return te.ms(), tr.ms()

    for _ in range(args.warmup):
        iteration()
    env.barrier()
    ev, rs = [], []
    launches0 = native().kernel_launch_count()
    _, stamp0 = off.kernel_timings()
    sampler = ClockSampler([env.local_rank]).start().wait_first()
    sampler.mark_start()
    for _ in range(args.steps):
        env.barrier()
        e, r = iteration()
        ev.append(env.max(e))
        rs.append(env.max(r))
    sampler.mark_end()
    clocks = sampler.stop()
    torch.cuda.synchronize(env.device)
    byte_exact = off.hash_tensor(cache) == ref
    ok_all = env.sum(0 if byte_exact else 1) == 0
    stats = off.daemon_stats()
    kernels = off.kernel_profile(stamp0) if getattr(args, "kernel_timing", 0) else None
    launches = env.sum(native().kernel_launch_count() - launches0)
    mm = load.stop() if load else 0
    sess.close()
    env.barrier()
    if daemon is not None:
        daemon.stop()
    env.close()
    if env.rank != 0:
        return None
    moved = per_iter * spec.block_bytes
    e_ms, r_ms = statistics.median(ev), statistics.median(rs)
    step_ms = e_ms + r_ms
    return {
        "metric": metric, "workload": "kv_cache",
        "value": round(env.world * 2 * moved / (step_ms / 1e3) / 1e9, 3),
        "unit": "GB/s (aggregate evict+restore of KV blocks / device time, max over ranks)",
        "n_gpus": env.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: bf16 N(0,1) KV cache, seeded per rank; seeded random block selection",
        "config": {"model": "paged KV cache: 16-token blocks x 64 layers x 8 KV heads x 128 dims",
                   "block_bytes": spec.block_bytes, "kv_bytes_per_gpu": nblocks * spec.block_bytes,
                   "blocks_per_iter": per_iter, "batch": batch, "pinned_window_gb": pinned_gb,
                   "concurrent_matmul": load.describe() if load else "none", "global_batch": env.world,
                   "seq_len": 16, "parallelism": f"dp{env.world}", "slot_mb": 4,
                   "evict_ctas": int(getattr(args, "evict_ctas", 0)) or "default",
                   "restore_ctas": int(getattr(args, "restore_ctas", 0)) or "default",
                   "group_mb": int(getattr(args, "kv_group_mb", 0)) or 256,
                   "l2": "GBs per iteration; no flush needed"},
        "evict_gbs_per_gpu": round(moved / (e_ms / 1e3) / 1e9, 3),
        "restore_gbs_per_gpu": round(moved / (r_ms / 1e3) / 1e9, 3),
        "byte_exact": ok_all,
        "tiers": {k: stats.get(k) for k in ("pinned_to_pageable_bytes", "pageable_to_pinned_bytes",
                                            "drains_completed", "readbacks_completed")},
        "gpu_launches": int(launches), "clocks": clocks, "matmul_iters": mm,
        **({"kernels": kernels} if kernels is not None else {}),
    }
