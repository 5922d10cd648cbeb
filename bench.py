#!/usr/bin/env python3
"""Headline benchmark: evict/restore GB/s per GPU on B200 (aggregate over N GPUs).

Workload (single-B200 eviction sweep point, run on every GPU of the job): a
bf16 N(0,1) tensor (default 1 GiB, larger than the 126 MB L2 so every step
streams from HBM) is evicted GPU -> pinned arena with the fused content hash
(K1) and restored pinned -> GPU (K2), while an 8192x8192 bf16 matmul loop runs
concurrently on the same GPU. The arena lives on the GPU's NUMA node, slots
are 64 MiB, data stays pinned between evict and restore.

At N >= 2 (even) the line carries a ``weight_sync`` block, the second half
of the metric: the sealed-version weight-sync latency of a Qwen2.5-32B-shaped
model, trainer TP=N/2 on the first half of the GPUs -> rollout TP=N/2 on the
second half (each trainer GPU holds a TP=4 shard: 64 layers at 8 GPUs, 32 at
4, 16 at 2), 10 % of the tensors changed per version, bf16 and fp8 push
modes, persistence on (statespectre_b200/parallel/weight_sync_bench.py).

Timing: W warm-up steps, then K steps bracketed by barrier + synchronize;
device time from CUDA events on the copy stream, max over ranks. ``value`` is
the whole-job aggregate: N * K * 2 * nbytes / max_rank_time. ``e2e`` repeats
the cycle through the public API (destructive ``off.evict`` + ``h.restore()``
+ reading the content hash back) timed on the host.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--size-mb MB] [--matmul 0|1]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference      # the unmodified reference build, same workload
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Reference numbers (StateSpectre docs/PERFORMANCE.md:33, H20 PCIe Gen5, 1 GiB):
BASELINE_D2H_GBS = 53.6
BASELINE_H2D_GBS = 57.5
BASELINE_ROUNDTRIP_GBS = 2.0 / (1.0 / BASELINE_D2H_GBS + 1.0 / BASELINE_H2D_GBS)
METRIC = "evict/restore GB/s per GPU at 1/2/4/8 B200; 32B weight-sync latency (ms)"


def _reference_arm(args) -> int:
    """The unmodified StateSpectre build (baseline/_ref) through its own API;
    loaded by file path so nothing of this package is imported on that path."""
    import importlib.util

    path = os.path.join(ROOT, "baseline", "reference_bench.py")
    spec = importlib.util.spec_from_file_location("reference_bench", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    if args.workload not in ("evict_restore", "sweep"):
        print(json.dumps(mod.unavailable(f"no reference arm for workload {args.workload}")), flush=True)
        return 0
    return mod.main(args, METRIC, BASELINE_ROUNDTRIP_GBS)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--size-mb", type=int, default=1024)
    p.add_argument("--matmul", type=int, default=1)
    p.add_argument("--engine", default="kernel", choices=["kernel", "copy_engine"])
    p.add_argument("--uncoded", default="copy_engine", choices=["copy_engine", "bulk", "sm"],
                   help="kernel engine: how bytes that are not zbf16-coded move")
    p.add_argument("--coded-evict", default="copy_engine", choices=["copy_engine", "sm"],
                   help="how zbf16-coded evicts leave the GPU (K1 into host memory, or via staging + copy engine)")
    p.add_argument("--coded-restore", default="copy_engine", choices=["copy_engine", "sm"],
                   help="how zbf16-coded runs come back (strided copy-engine copies + HBM decode, or K2 from host)")
    p.add_argument("--dtype", default="bf16", choices=["bf16", "fp32"],
                   help="payload dtype (fp32: N(0, 0.02) values, like master weights; zf32-coded)")
    p.add_argument("--stage-ctas", type=int, default=0,
                   help="CTAs of the staged zbf16 coding/decoding passes (0 = auto)")
    p.add_argument("--stage-depth", type=int, default=0, help="staging buffers of the coded paths (0 = auto)")
    p.add_argument("--stage-piece-chunks", type=int, default=0, help="64 KiB chunks per staging buffer (0 = auto)")
    p.add_argument("--evict-ctas", type=int, default=0)
    p.add_argument("--restore-ctas", type=int, default=0)
    p.add_argument("--hash", type=int, default=1)
    p.add_argument("--host-hash-kb", type=int, default=-1,
                   help="uncoded evicts up to this size hash their pinned copy on the host (-1: the agent's default)")
    p.add_argument("--compress", type=int, default=1, help="zbf16 lossless coding of the bf16 payload over PCIe")
    p.add_argument("--e2e-steps", type=int, default=0, help="default: same as --steps")
    p.add_argument("--kernel-timing", type=int, default=0,
                   help="stamp kernels on the device (%%globaltimer) and report per-kernel time and GB/s")
    p.add_argument("--out", default="")
    # --workload weight_sync: in-box RL weight sync (trainer half -> rollout half of the GPUs)
    p.add_argument("--workload", default="evict_restore",
                   choices=["evict_restore", "weight_sync", "sweep", "kv_cache", "dp_dedup", "sections"])
    p.add_argument("--model", default="", help="weight_sync: qwen2.5-32b (default); dp_dedup: llama-3-8b (default)")
    p.add_argument("--layers", type=int, default=0, help="weight_sync: layer count override (0 = the model's)")
    p.add_argument("--push-mode", default="bf16", choices=["bf16", "fp8", "both"])
    p.add_argument("--weight-sync", type=int, default=1,
                   help="evict_restore at N >= 2: append the sealed-version weight-sync block "
                        "(Qwen2.5-32B-shaped, TP=N/2 -> TP=N/2, bf16 and fp8)")
    p.add_argument("--ws-versions", type=int, default=50, help="weight-sync block: timed versions per mode")
    p.add_argument("--ws-warmup", type=int, default=3, help="weight-sync block: untimed versions per mode")
    p.add_argument("--ref-ws-versions", type=int, default=3,
                   help="reference arm's weight-sync block: timed versions (each moves every tensor over TCP)")
    p.add_argument("--ref-ws-budget-s", type=float, default=300.0,
                   help="reference arm's weight-sync block: stop timing further versions after this many seconds "
                        "(at least one timed version)")
    p.add_argument("--rollout-replicas", type=int, default=1,
                   help="weight_sync: rollout engines fed by each trainer shard (GPUs split 1 + R ways)")
    p.add_argument("--transport", default="auto", choices=["auto", "p2p", "multicast"],
                   help="weight_sync: NVLS multicast team or one point-to-point push per replica")
    p.add_argument("--persist", type=int, default=1, help="weight_sync: seal every version in offloadd")
    p.add_argument("--verify", type=int, default=1, help="weight_sync: rollout re-hashes what it received")
    p.add_argument("--change-fraction", type=float, default=0.1)
    p.add_argument("--delta-std", type=float, default=1e-3)
    p.add_argument("--hint", type=int, default=0,
                   help="weight_sync: pass the changed-tensor list instead of hashing every tensor")
    p.add_argument("--max-size-mb", type=int, default=8192, help="sweep: largest tensor")
    p.add_argument("--arena-gb", type=int, default=0, help="sweep: pinned window per GPU (0: 3x the largest size)")
    p.add_argument("--kv-gb", type=float, default=40.0, help="kv_cache: KV cache bytes per GPU")
    p.add_argument("--evict-fraction", type=float, default=0.5, help="kv_cache: blocks moved per iteration")
    p.add_argument("--kv-batch", type=int, default=0,
                   help="kv_cache: blocks per evict_batch/restore_batch call (0: the whole iteration in one call)")
    p.add_argument("--pinned-gb", type=int, default=0, help="kv_cache: pinned window per GPU (0 = fits the set)")
    p.add_argument("--tier-threads", default="",
                   help="kv_cache: offloadd drain workers, readback workers and copy threads, e.g. 4,4,8")
    p.add_argument("--kv-group-mb", type=int, default=0, help="kv_cache: bytes per reservation group (0 = 256 MiB)")
    p.add_argument("--nvme-dir", default="", help="dp_dedup: NVMe spill directory")
    p.add_argument("--dedup-mode", default="p2p_verified",
                   choices=["p2p_verified", "device_hash_verified", "semantic_trusted", "hash_verified"],
                   help="dp_dedup: how replicas confirm the owner's copy")
    p.add_argument("--spill-timeout", type=float, default=600.0, help="dp_dedup: seconds to wait for the spill")
    return p.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        return _reference_arm(args)

    if args.workload != "evict_restore":
        if args.workload == "weight_sync":
            from statespectre_b200.parallel.weight_sync_bench import run
        elif args.workload == "sweep":
            from statespectre_b200.benchmarks.sweep import run
        elif args.workload == "kv_cache":
            from statespectre_b200.benchmarks.kv_cache import run
        elif args.workload == "sections":
            from statespectre_b200.benchmarks.sections import run
        else:
            from statespectre_b200.benchmarks.dp_dedup import run

        out = run(args, METRIC)
        if out is not None:
            line = json.dumps(out)
            print(line, flush=True)
            if args.out:
                with open(args.out, "w") as f:
                    f.write(line + "\n")
        return 0

    import torch
    import torch.distributed as dist

    from statespectre_b200 import launch_daemon, offload_context
    from statespectre_b200._native import native
    from statespectre_b200.utils.clocks import ClockSampler
    from statespectre_b200.utils.launch import host_mem_available_bytes
    from statespectre_b200.utils.topology import daemon_yaml, gpu_numa_nodes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        # the weight-sync block's trainer/rollout pairs exchange hashes with plain send/recv
        os.environ.setdefault("TORCH_NCCL_SHOW_EAGER_INIT_P2P_SERIALIZATION_WARNING", "false")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    nbytes = args.size_mb << 20
    # three tensors' room per GPU window, unless the host cannot pin that for
    # every window of the node (GPU hosts here have about 196 GB): then one
    # tensor plus 2 GB, which the evict/restore loop needs at any time
    n_windows = max(int(os.environ.get("LOCAL_WORLD_SIZE", str(world))), torch.cuda.device_count(), 1)
    avail = host_mem_available_bytes()
    room_gb = int(0.6 * avail / (1 << 30) / n_windows) if avail else 1 << 20
    window_gb = max(4, min((3 * nbytes >> 30) + 2, max((nbytes >> 30) + 2, room_gb)))
    run_dir = os.environ.get("OFLD_BENCH_DIR", "/tmp/ofld_bench")
    os.makedirs(run_dir, exist_ok=True)
    sock = os.path.join(run_dir, "offloadd.sock")
    daemon = None
    if local_rank == 0:
        if os.path.exists(sock):
            os.unlink(sock)
        cfg = os.path.join(run_dir, "offloadd.yaml")
        n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
        with open(cfg, "w") as f:
            f.write(daemon_yaml(sock, gpu_numa_nodes(max(n_local, torch.cuda.device_count())), window_gb))
        daemon = launch_daemon(sock, config=cfg, log_path=os.path.join(run_dir, "offloadd.log"))
    barrier()
    if world > 1 and local_rank != 0:
        deadline = time.time() + 120
        while not os.path.exists(sock) and time.time() < deadline:
            time.sleep(0.05)

    sess = offload_context(daemon_addr=sock, device=device, rank=rank, local_rank=local_rank, world_rank=rank,
                           eager_register=True, engine=args.engine, evict_ctas=args.evict_ctas,
                           restore_ctas=args.restore_ctas, hash_on_evict=bool(args.hash), stream_priority=-1,
                           compress=bool(args.compress), kernel_timing=bool(args.kernel_timing),
                           uncoded=args.uncoded, coded_restore=args.coded_restore, coded_evict=args.coded_evict,
                           stage_ctas=args.stage_ctas, stage_depth=args.stage_depth,
                           stage_piece_chunks=args.stage_piece_chunks)
    off = sess.off
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    if args.dtype == "fp32":
        x = torch.randn(nbytes // 4, dtype=torch.float32, device=device, generator=g) * 0.02
    else:
        x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=device, generator=g)
    ref_hash = off.hash_tensor(x)
    # what crosses PCIe: zbf16 / zf32 coding of the payload (host codec on a 64 MiB sample)
    coding = "none"
    if args.compress and args.engine == "kernel":
        sample = x.view(torch.uint8)[: min(nbytes, 64 << 20)].cpu().numpy()
        codec = "zf32" if args.dtype == "fp32" else "zbf16"
        coded = getattr(native(), f"{codec}_encode")(sample)
        if coded is not None:
            frac = getattr(native(), f"{codec}_coded_bytes")(coded) / len(sample)
            coding = f"{codec} lossless, {frac:.4f} of the bytes"
    copy_stream = torch.cuda.Stream(device=device, priority=-1)

    # ---- concurrent 8192^2 bf16 matmul loop on its own stream ----
    stop_mm = threading.Event()
    mm_count = [0]
    mm_thread = None
    if args.matmul:
        mm_stream = torch.cuda.Stream(device=device)
        a = torch.randn(8192, 8192, dtype=torch.bfloat16, device=device)
        b = torch.randn(8192, 8192, dtype=torch.bfloat16, device=device)
        c = torch.empty(8192, 8192, dtype=torch.bfloat16, device=device)

        def mm_loop():
            torch.cuda.set_device(device)
            with torch.cuda.stream(mm_stream):
                while not stop_mm.is_set():
                    for _ in range(8):
                        torch.matmul(a, b, out=c)
                    mm_stream.synchronize()
                    mm_count[0] += 8

        mm_thread = threading.Thread(target=mm_loop, daemon=True)
        mm_thread.start()

    tid = ((rank & 0x7FFFFF) << 40) | 0xB0000
    evict_ms, restore_ms = [], []

    def cycle(version: int, record: bool):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        e0.record(copy_stream)
        h = off.copy(x, stream=copy_stream, wait=True, tensor_id=tid, version=version)
        e1.record(copy_stream)
        h.restore_into(x, stream=copy_stream, wait=True)
        e2.record(copy_stream)
        h.discard()
        if record:
            e2.synchronize()
            evict_ms.append(e0.elapsed_time(e1))
            restore_ms.append(e1.elapsed_time(e2))
        return h

    for i in range(args.warmup):
        cycle(i + 1, False)
    torch.cuda.synchronize(device)
    assert off.hash_tensor(x) == ref_hash, "round trip corrupted the tensor"
    launches0 = native().kernel_launch_count()
    _, stamp0 = off.kernel_timings()
    sampler = ClockSampler([local_rank]).start().wait_first()
    barrier()
    torch.cuda.synchronize(device)
    sampler.mark_start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(copy_stream)
    for i in range(args.steps):
        cycle(1000 + i, False)
    t_end.record(copy_stream)
    torch.cuda.synchronize(device)
    sampler.mark_end()
    barrier()
    clocks = sampler.stop()
    launches = native().kernel_launch_count() - launches0
    kernels = off.kernel_profile(stamp0) if args.kernel_timing else None
    dev_ms = t_start.elapsed_time(t_end)
    dev_ms_max = max_over_ranks(dev_ms)
    value = world * args.steps * 2 * nbytes / (dev_ms_max / 1e3) / 1e9

    # per-direction rates (separately timed steps, for the breakdown)
    for i in range(3):
        cycle(5000 + i, True)
    # each rank's median, then the slowest rank's (host-memory write bandwidth shared by all
    # GPUs of a node shows up as the slowest rank's evict)
    ev = max_over_ranks(sorted(evict_ms)[len(evict_ms) // 2])
    rs = max_over_ranks(sorted(restore_ms)[len(restore_ms) // 2])

    # ---- end to end through the public API ----
    e2e_steps = args.e2e_steps or args.steps
    torch.cuda.synchronize(device)
    barrier()
    t0 = time.perf_counter()
    hashes_ok = True
    for i in range(e2e_steps):
        h = off.evict(x, wait=True, tensor_id=tid, version=20000 + i)   # D2H, VRAM released
        x = h.restore()                                                   # H2D from pinned host memory
        if args.hash:
            hashes_ok &= h.content_hash == ref_hash                       # 16 B result read back
        h.discard()
    torch.cuda.synchronize(device)
    e2e_s = time.perf_counter() - t0
    e2e_s_max = max_over_ranks(e2e_s)
    barrier()
    e2e_value = world * e2e_steps * 2 * nbytes / e2e_s_max / 1e9
    stop_mm.set()
    if mm_thread:
        mm_thread.join(timeout=30)
    mm_tflops = None
    assert hashes_ok, "content hash changed across the e2e round trips"
    if not args.hash:  # no digests on evict: the tensor itself is the check
        assert off.hash_tensor(x) == ref_hash, "e2e round trips corrupted the tensor"

    sess.close()
    barrier()
    if daemon is not None:
        daemon.stop()
    ws = None
    if world >= 2 and args.weight_sync and world % 2 == 0:
        # second half of the metric: sealed-version weight sync, TP=N/2 -> TP=N/2, each trainer GPU
        # holding a TP=4 shard of Qwen2.5-32B (all 64 layers at 8 GPUs, 32 at 4, 16 at 2)
        from statespectre_b200.parallel.weight_sync_bench import layers_for, run_block

        args.rollout_replicas = 1
        ws = run_block(args, world, rank, local_rank, device, ["bf16", "fp8"], args.ws_versions, args.ws_warmup,
                       layers=layers_for(world))
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s (aggregate over all GPUs, evict+restore bytes / device time)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / (world * BASELINE_ROUNDTRIP_GBS), 4),
            "dtype": args.dtype,
            "data": "synthetic: fp32 N(0, 0.02) random tensor, seeded per rank" if args.dtype == "fp32"
                    else "synthetic: bf16 N(0,1) random tensor, seeded per rank",
            "config": {
                "model": f"single-B200 eviction sweep point: {args.dtype} tensor evict (K1, fused ssh128 hash) + "
                         "restore (K2)",
                "tensor_bytes": nbytes, "global_batch": world, "seq_len": 0, "parallelism": f"dp{world}",
                "concurrent_matmul": "8192x8192 bf16 loop" if args.matmul else "none",
                "engine": args.engine, "hash": bool(args.hash), "slot_mb": 64,
                "uncoded_form": args.uncoded, "coded_evict": args.coded_evict, "coded_restore": args.coded_restore,
                "stage_ctas": args.stage_ctas or "auto", "stage_depth": args.stage_depth or "auto",
                "stage_piece_chunks": args.stage_piece_chunks or "auto",
                "transfer_coding": coding,
                "l2": "inputs (1 GiB) larger than the 126 MB L2; no flush needed",
                "baseline": f"StateSpectre H20 PCIe Gen5 1 GiB: D2H {BASELINE_D2H_GBS}, H2D {BASELINE_H2D_GBS} GB/s "
                            f"(round trip {BASELINE_ROUNDTRIP_GBS:.2f} GB/s per GPU)",
            },
            "evict_gbs_per_gpu": round(nbytes / (ev / 1e3) / 1e9, 3),
            "restore_gbs_per_gpu": round(nbytes / (rs / 1e3) / 1e9, 3),
            "per_gpu_basis": "slowest rank's median of 3 separately timed evicts / restores",
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s (aggregate, public API, host-timed)",
                    "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes + (16 if args.hash else 0)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "matmul_iters": mm_count[0],
        }
        if kernels is not None:
            line["kernels"] = kernels  # device-stamped, timed region, rank 0
        if ws is not None:
            line["weight_sync"] = ws
        print(json.dumps(line), flush=True)
        if args.out:
            with open(args.out, "w") as f:
                json.dump(line, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
