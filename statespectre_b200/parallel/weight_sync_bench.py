"""In-box RL weight-sync benchmark (trainer TP=N/(1+R) GPUs -> R rollout
engines of the same TP).

Workload: the trainer holds a Qwen2.5-32B-shaped bf16 model, random-init
N(0, 0.02), tensor-parallel over the first N/(1+R) GPUs; each of the R
rollout engines (``--rollout-replicas``, default 1) holds the same shards on
the next N/(1+R) GPUs (trainer tp rank r feeds tp rank r of every engine:
one NVLS multicast push for all of them, or one point-to-point push each,
``--transport``). Every version, a seeded 10 % of the tensors get +N(0, 1e-3); the
update arrives from pinned host memory (H2D) and is applied on the trainer.

One sealed-version step, timed on the host from the H2D of the update:
  1. push (K4): hash every chunk of the shard, move only chunks whose digest
     changed into the rollout's receive buffer over NVLink (fp8 mode:
     quantized to e4m3 with 1x128 scales on the way);
  2. the trainer sends the version's content hashes to the rollout, which
     re-hashes what it received (bf16 mode) and answers;
  3. meanwhile, with persistence on, every trainer rank records its shard of
     the version in offloadd (changed tensors copied to the host by K1 as new
     canonical objects, unchanged ones carried forward) and one rank seals and
     promotes it;
  4. the trainer reads the rollout's answer back (D2H). The step ends when
     the version is both verified by the rollout and sealed.

Reported per mode (max over ranks, median over versions): ``e2e_ms`` (the
sealed-version latency above), ``push_ms`` (CUDA events around the K4
launches) and ``seal_ms`` (host).

    torchrun --nproc-per-node 8 bench.py --workload weight_sync --gpus 8 --steps 50 --warmup 3
"""

from __future__ import annotations

import datetime
import os
import statistics
import time

import torch
import torch.distributed as dist

from ..models.shapes import MODELS, QWEN2_5_32B, num_params, param_shapes, pick_changed, random_init
from ..utils.clocks import ClockSampler
from ..utils.launch import host_mem_available_bytes, start_node_daemon
from .weight_sync import RolloutWeights, TrainerWeightSync, WeightLayout

GiB = 1 << 30


def layers_for(world: int, replicas: int = 1, full_layers: int = 64, full_tp: int = 4) -> int:
    """Layer count that gives each trainer GPU the shard it holds in the
    TP=4 -> TP=4 configuration (64 layers at 8 GPUs, 32 at 4, 16 at 2)."""
    tp = world // (1 + replicas)
    return max(1, full_layers * tp // full_tp)


def run_block(opts, world: int, rank: int, local_rank: int, device, modes, versions: int, warmup: int,
              layers: int = 0, run_dir: str = "") -> dict | None:
    """Weight-sync measurement on an initialized process group. Returns the
    per-mode results on rank 0 (None elsewhere)."""
    replicas = max(1, int(getattr(opts, "rollout_replicas", 1)))
    if world < 2 or world % (1 + replicas):
        raise SystemExit(f"weight_sync needs a multiple of {1 + replicas} GPUs (trainer + {replicas} rollout engines)")
    tp = world // (1 + replicas)
    trainer = rank < tp
    tp_rank = rank % tp
    engine = rank // tp - 1  # rollout engine index (-1 on trainer ranks)
    spec = MODELS.get(getattr(opts, "model", "") or "qwen2.5-32b", QWEN2_5_32B)
    shapes = param_shapes(spec, tp_rank, tp, layers=layers or None)
    shard_bytes = num_params(shapes) * 2
    change = float(getattr(opts, "change_fraction", 0.1))
    trainer_group = dist.new_group(list(range(tp)))

    # persistence needs pinned room for one full shard per trainer plus the
    # changed tensors of the retained versions (x6 margin for the contiguous
    # runs that multi-GB tensors need)
    n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    per_trainer_gb = int(shard_bytes * (1.0 + 6 * change) / GiB) + 4
    need = per_trainer_gb * GiB * min(tp, n_local)
    persist = bool(getattr(opts, "persist", 1))
    avail = host_mem_available_bytes()
    if persist and avail and need > 0.7 * avail:
        persist = False
    flag = torch.tensor([int(persist)], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    persist = bool(flag.item())
    windows = [per_trainer_gb if (i < tp and persist) else 0 for i in range(n_local)]
    if not any(windows):
        windows[0] = 1
    run_dir = run_dir or os.environ.get("OFLD_BENCH_DIR", "/tmp/ofld_wsync")
    # 2 MiB slots: a model has hundreds of small tensors (norms, biases)
    sock, daemon = start_node_daemon(local_rank, n_local, windows, run_dir, barrier=dist.barrier, slot_mb=2,
                                     extra_yaml="manifest:\n  retain_sealed_versions: 2\n")

    from .. import offload_context
    from .._native import native

    sess = offload_context(daemon_addr=sock, device=device, rank=rank, local_rank=local_rank, world_rank=rank,
                           job_name="wsync-bench", eager_register=persist and trainer)
    off = sess.off
    names = [n for n, _ in shapes]
    params = random_init(shapes, device, seed=1000 + tp_rank) if trainer else None
    if trainer:
        # pinned host pool of update deltas: as large as the largest tensor,
        # sliced cyclically (N(0, delta_std) drawn on the GPU, copied once)
        biggest = max(t.numel() for t in params.values())
        scratch = torch.empty(biggest, dtype=torch.bfloat16, device=device)
        scratch.normal_(0.0, float(getattr(opts, "delta_std", 1e-3)),
                        generator=torch.Generator(device=device).manual_seed(7 + tp_rank))
        pool = torch.empty(biggest, dtype=torch.bfloat16, pin_memory=True)
        pool.copy_(scratch)
    nitems = len(shapes)
    peers = [tp_rank + tp * (1 + j) for j in range(replicas)] if trainer else [tp_rank]
    hbuf = torch.zeros(2 * nitems, dtype=torch.int64, device=device)
    ack = torch.zeros(2, dtype=torch.int64, device=device)
    ack_host = torch.zeros(2, dtype=torch.int64, pin_memory=True)
    results = {}
    launches0 = native().kernel_launch_count()
    clocks = None
    version_base = 0
    for mode in modes:
        layout = WeightLayout([(n, s, torch.bfloat16) for n, s in shapes], mode)
        rw = tr = None
        if not trainer:
            rw = RolloutWeights(layout, device)
            rw.publish(off, f"rollout/{mode}/{engine}/{tp_rank}")
        dist.barrier()
        if trainer:
            tr = TrainerWeightSync(off, params, [f"rollout/{mode}/{j}/{tp_rank}" for j in range(replicas)],
                                   mode=mode, persist=persist, tp_rank=tp_rank,
                                   transport=getattr(opts, "transport", "auto"),
                                   seal_barrier=lambda: dist.barrier(group=trainer_group), sealer=tp_rank == 0)
        else:
            rw.connect(off)
        dist.barrier()
        transport = tr.transport if trainer else rw.transport

        def version_step(v: int, stats):
            t0 = time.perf_counter()
            h2d = 0
            chosen = []
            res = {}
            pushed = 0
            if trainer:
                if v > version_base + 1:
                    # H2D of this version's update from pinned memory, applied on the device
                    chosen = pick_changed(names, change, seed=v * 7919 + tp_rank)
                    off_e = 0
                    for i in chosen:
                        t = params[names[i]]
                        n = t.numel()
                        if off_e + n > pool.numel():
                            off_e = 0
                        scratch[:n].copy_(pool[off_e:off_e + n], non_blocking=True)
                        t.view(-1).add_(scratch[:n])
                        off_e += n
                        h2d += 2 * n
                torch.cuda.current_stream(device).synchronize()
            dist.barrier()
            if trainer:
                before = tr.pushers[0].result()["bytes_stored"]
                hint = [names[i] for i in chosen] if (getattr(opts, "hint", 0) and v > version_base + 1) else None
                res = tr.push_version(v, changed=hint)
                pushed = tr.pushers[0].result()["bytes_stored"] - before
                hbuf.copy_(tr.pushers[0].item_hash)
                for q in peers:
                    dist.send(hbuf, q)
                res.update(tr.seal_version())  # runs while the rollout checks what it received
                acks = 0
                for q in peers:
                    dist.recv(ack, q)
                    acks += int(ack[0].item())
                ack.fill_(acks)
                ack_host.copy_(ack)  # D2H of the rollouts' answers
            else:
                dist.recv(hbuf, peers[0])
                ok = 1
                if getattr(opts, "verify", 1) and mode == "bf16":
                    got = rw.content_hashes()
                    want = hbuf.view(-1, 2).tolist()
                    m = 2**64 - 1
                    for i, e in enumerate(layout.entries):
                        if got[e.name] != (want[i][0] & m, want[i][1] & m):
                            ok = 0
                ack.fill_(ok)
                dist.send(ack, peers[0])
            t2 = time.perf_counter()
            if stats is not None:
                vals = torch.tensor([res.get("push_ms", 0.0), res.get("seal_wall_ms", 0.0), (t2 - t0) * 1e3,
                                     float(pushed), 0.0 if trainer else float(ack[0].item() == 0), float(h2d),
                                     float(res.get("changed", 0))], dtype=torch.float64, device=device)
                gathered = [torch.zeros_like(vals) for _ in range(world)]
                dist.all_gather(gathered, vals)
                rows = torch.stack(gathered).cpu()
                stats["push_ms"].append(float(rows[:tp, 0].max()))
                stats["seal_ms"].append(float(rows[:tp, 1].max()))
                stats["e2e_ms"].append(float(rows[:, 2].max()))
                stats["bytes"].append(float(rows[:tp, 3].sum()))
                stats["verify_fail"] += int(rows[tp:, 4].sum())
                stats["h2d"].append(float(rows[:tp, 5].sum()))
                stats["changed"].append(float(rows[:tp, 6].sum()))

        for v in range(version_base + 1, version_base + warmup + 1):
            version_step(v, None)
        stats = {"push_ms": [], "seal_ms": [], "e2e_ms": [], "bytes": [], "h2d": [], "changed": [], "verify_fail": 0}
        sampler = ClockSampler([local_rank]).start().wait_first()
        dist.barrier()
        sampler.mark_start()
        for v in range(version_base + warmup + 1, version_base + warmup + versions + 1):
            version_step(v, stats)
        sampler.mark_end()
        mode_clocks = sampler.stop()
        clocks = clocks or mode_clocks
        last = version_base + warmup + versions
        if tr:
            tr.close()
        if rw:
            rw.close()
        dist.barrier()
        if trainer and persist and tp_rank == 0:
            for v in (last - 1, last):  # the retained versions of this mode
                off.drop_canonical_version("policy_rollout", v)
        dist.barrier()
        version_base = last + 1000
        if rank == 0:
            e2e = sorted(stats["e2e_ms"])
            push = sorted(stats["push_ms"])
            med_push = statistics.median(push)
            results[mode] = {
                "e2e_ms": round(statistics.median(e2e), 3),
                "e2e_ms_p90": round(e2e[min(len(e2e) - 1, int(0.9 * len(e2e)))], 3),
                "push_ms": round(med_push, 4),
                "push_ms_max": round(push[-1], 4),
                "seal_ms": round(statistics.median(stats["seal_ms"]), 3) if persist else None,
                "versions": versions,
                "transport": transport,
                "pushed_source_bytes_per_version": int(statistics.median(stats["bytes"])),
                "changed_tensors_per_version": int(statistics.median(stats["changed"])),
                "source_gbs_per_trainer": round(statistics.median(stats["bytes"]) / tp / (med_push / 1e3) / 1e9, 2),
                "verify": "rollout re-hash of every tensor" if (mode == "bf16" and getattr(opts, "verify", 1))
                          else "none (fp8 bytes differ from the bf16 source by design)",
                "verify_failures": stats["verify_fail"],
                "h2d_bytes_per_version": int(statistics.median(stats["h2d"])),
                "d2h_bytes_per_version": 16 * tp,
                "clocks": mode_clocks,
            }
    launches = torch.tensor([native().kernel_launch_count() - launches0], device=device)
    dist.all_reduce(launches)
    sess.close()
    dist.barrier()
    if daemon is not None:
        daemon.stop()
    dist.destroy_process_group(trainer_group)
    if rank != 0:
        return None
    full = param_shapes(spec, 0, 1, layers=layers or None)
    return {
        "model": f"{spec.name}-shaped" + (f" ({layers} of {spec.layers} layers)" if layers and layers != spec.layers
                                          else ""),
        "params": num_params(full), "model_bytes": num_params(full) * 2,
        "trainer": f"TP={tp} on GPUs 0-{tp - 1}",
        "rollout": f"{replicas} x TP={tp} on GPUs {tp}-{world - 1}",
        "parallelism": f"tp{tp}->tp{tp}" + (f" x{replicas}" if replicas > 1 else ""),
        "shard_bytes_per_trainer_gpu": shard_bytes,
        "change_fraction": change, "persist": persist, "slot_mb": 2,
        "change_detection": "caller hint" if getattr(opts, "hint", 0) else "device hash of every tensor",
        "modes": results,
        "gpu_launches": int(launches.item()),
        "clocks": clocks,
        "l2": "every push reads the whole shard (GBs) from HBM; no flush needed",
    }


def run(args, metric: str) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    # trainer/rollout pairs exchange hashes with plain send/recv on the default group
    os.environ.setdefault("TORCH_NCCL_SHOW_EAGER_INIT_P2P_SERIALIZATION_WARNING", "false")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    modes = [args.push_mode] if args.push_mode != "both" else ["bf16", "fp8"]
    block = run_block(args, world, rank, local_rank, device, modes, args.steps, args.warmup, layers=args.layers)
    dist.destroy_process_group()
    if block is None:
        return None
    first = block["modes"][modes[0]]
    return {
        "metric": metric, "workload": "weight_sync", "value": first["e2e_ms"],
        "unit": "ms (sealed-version latency: H2D update + push + seal || rollout verify + D2H answer; "
                "max over ranks, median over versions)",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": first["e2e_ms"],
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random-init N(0,0.02) weights of the named architecture; seeded 10% of tensors "
                "+N(0,1e-3) per version, update fed from pinned host memory",
        "config": {k: v for k, v in block.items() if k not in ("modes", "gpu_launches", "clocks")}
        | {"global_batch": 1, "seq_len": 0},
        "modes": block["modes"],
        "e2e": {"value": first["e2e_ms"], "unit": "ms (host wall per sealed version)",
                "h2d_bytes_per_step": first["h2d_bytes_per_version"],
                "d2h_bytes_per_step": first["d2h_bytes_per_version"]},
        "gpu_launches": block["gpu_launches"],
        "clocks": block["clocks"],
    }
