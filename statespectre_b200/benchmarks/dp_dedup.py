"""Data-parallel canonical dedup with ZeRO-1 optimizer-state spill.

Workload: every rank of a DP group holds the same Llama-3-8B-shaped bf16
weights (random-init N(0, 0.02), identical seed) in one flat parameter
buffer. ``canonical_evict`` has one owner per parameter (round robin) copy it
to pinned memory (K1, fused hash) while every other rank confirms its replica
without PCIe traffic: ``--dedup-mode p2p_verified`` (default) compares its
bytes with the owner's GPU copy over NVLink (K3), ``device_hash_verified``
hashes its own HBM copy for the daemon to compare.
Then each rank evicts its ZeRO-1 shard of fp32 Adam m and v (1/N of the
parameters each), the daemon spills it to NVMe (``--nvme-dir``, O_DIRECT
io_uring striped files), and the shard is restored back from NVMe.

Reported (max over ranks): dedup time for the whole model, the logical
eviction rate (N replicas x model bytes / time), PCIe bytes per rank, and the
m/v evict, spill and restore rates.

    torchrun --nproc-per-node 8 bench.py --gpus 8 --workload dp_dedup --nvme-dir /nvme/ofld
"""

from __future__ import annotations

import time

import torch

from .. import DedupPolicy, offload_context
from .._native import native
from ..models.shapes import LLAMA3_8B, MODELS, num_params, param_shapes, random_init_flat
from ..parallel.dp_dedup import dedup_evict_params
from ..utils.clocks import ClockSampler
from .common import node_daemon, setup

GiB = 1 << 30


def _sync_wall(env, fn):
    torch.cuda.synchronize(env.device)
    env.barrier()
    t0 = time.perf_counter()
    out = fn()
    torch.cuda.synchronize(env.device)
    dt = time.perf_counter() - t0
    return out, env.max(dt * 1e3)


def run(args, metric: str) -> dict:
    env = setup()
    spec = MODELS.get(args.model or "llama-3-8b", LLAMA3_8B)
    shapes = param_shapes(spec, layers=args.layers or None)
    model_bytes = num_params(shapes) * 2
    shard_elems = (num_params(shapes) + env.world - 1) // env.world
    mv_bytes = 2 * shard_elems * 4
    # pinned: owned weights (1/N of the model) + the m/v shard + slack
    window_gb = int((model_bytes / env.world + mv_bytes) * 1.3 / GiB) + 4
    nvme_dir = args.nvme_dir or "/tmp/ofld_nvme"
    sock, daemon = node_daemon(env, window_gb, "/tmp/ofld_dp", slot_mb=2, drain_on_complete=True,
                               drain_target="nvme", nvme_dir=nvme_dir)
    sess = offload_context(daemon_addr=sock, device=env.device, rank=env.rank, local_rank=env.local_rank,
                           world_rank=env.rank, job_name="dp-dedup", eager_register=True)
    off = sess.off
    _flat, params = random_init_flat(shapes, env.device, seed=0)  # identical on every replica
    mode = getattr(args, "dedup_mode", "p2p_verified")
    ref = {n: off.hash_tensor(t) for n, t in list(params.items())[:4]}
    launches0 = native().kernel_launch_count()
    sampler = ClockSampler([env.local_rank]).start().wait_first()
    sampler.mark_start()

    # ---- phase 1: canonical dedup of the replicated weights ----
    handles, dedup_ms = _sync_wall(env, lambda: dedup_evict_params(
        off, params, model_role="policy_trainable", model_version=1,
        policy=DedupPolicy(mode), owner="round_robin", destructive=False))
    actions = {}
    copied = 0
    for n, h in handles.items():
        actions[h.action_name] = actions.get(h.action_name, 0) + 1
        if h.did_d2h:
            copied += params[n].numel() * 2
    pcie_bytes = env.max(copied)
    # a replica's restore of an object another rank created is byte-exact
    ok = True
    for n in list(ref):
        dst = torch.empty_like(params[n])
        handles[n].restore_into(dst)
        ok &= off.hash_tensor(dst) == ref[n]

    # ---- phase 2: ZeRO-1 m/v shard: evict, spill to NVMe, restore ----
    g = torch.Generator(device=env.device).manual_seed(100 + env.rank)
    piece = 64 << 20  # 256 MiB fp32 tensors
    mv = [torch.randn(min(piece, shard_elems - i), dtype=torch.float32, device=env.device, generator=g)
          for _ in range(2) for i in range(0, shard_elems, piece)]
    mv_ref = [off.hash_tensor(t) for t in mv]
    hs, mv_evict_ms = _sync_wall(env, lambda: [off.copy(t, wait=True) for t in mv])

    def spilled():
        deadline = time.time() + args.spill_timeout
        while time.time() < deadline:
            if all(h.location() == "nvme" for h in hs):
                return True
            time.sleep(0.05)
        return False

    spilled_ok, spill_ms = _sync_wall(env, spilled)
    outs, mv_restore_ms = _sync_wall(env, lambda: [h.restore() for h in hs])
    mv_ok = all(off.hash_tensor(o) == r for o, r in zip(outs, mv_ref))
    sampler.mark_end()
    clocks = sampler.stop()
    ok_all = env.sum(0 if (ok and mv_ok) else 1) == 0
    spill_all = env.sum(0 if spilled_ok else 1) == 0
    launches = env.sum(native().kernel_launch_count() - launches0)
    stats = off.daemon_stats()
    for h in hs:
        h.discard()
    sess.close()
    env.barrier()
    if daemon is not None:
        daemon.stop()
    env.close()
    if env.rank != 0:
        return None
    return {
        "metric": metric, "workload": "dp_dedup",
        "value": round(env.world * model_bytes / (dedup_ms / 1e3) / 1e9, 3),
        "unit": "GB/s (logical: N replicas x model bytes canonically evicted / wall time, max over ranks)",
        "n_gpus": env.world, "steps": 1, "warmup": 0, "ms_per_step": round(dedup_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init N(0,0.02) weights (same seed on every replica); fp32 N(0,1) m/v shards",
        "config": {"model": f"{spec.name}-shaped" + (f" ({args.layers} layers)" if args.layers else ""),
                   "model_bytes": model_bytes, "parallelism": f"dp{env.world}", "dedup": mode,
                   "owner": "round_robin", "zero1_mv_bytes_per_rank": mv_bytes, "nvme_dir": nvme_dir,
                   "global_batch": env.world, "seq_len": 0, "slot_mb": 2,
                   "l2": "whole-model passes; no flush needed"},
        "dedup_ms": round(dedup_ms, 3), "pcie_bytes_per_rank_max": int(pcie_bytes),
        "actions_on_rank0": actions,
        "mv_evict_gbs_per_rank": round(mv_bytes / (mv_evict_ms / 1e3) / 1e9, 3),
        "mv_spill_ms": round(spill_ms, 1), "mv_spilled_to_nvme": spill_all,
        "mv_spill_gbs_per_rank": round(mv_bytes / (spill_ms / 1e3) / 1e9, 3) if spill_all else None,
        "mv_restore_gbs_per_rank": round(mv_bytes / (mv_restore_ms / 1e3) / 1e9, 3),
        "byte_exact": ok_all,
        "nvme": {k: stats.get(k) for k in ("nvme_write_bytes", "nvme_read_bytes", "io_failure_count")},
        "gpu_launches": int(launches), "clocks": clocks,
    }
