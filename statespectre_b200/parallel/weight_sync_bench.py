"""In-box RL weight-sync benchmark (trainer TP=N/(1+R) GPUs -> R rollout
engines of the same TP).

Workload: the trainer holds a Qwen2.5-32B-shaped bf16 model, random-init
N(0, 0.02), tensor-parallel over the first N/(1+R) GPUs; each of the R
rollout engines (``--rollout-replicas``, default 1) holds the same shards on
the next N/(1+R) GPUs (trainer tp rank r feeds tp rank r of every engine:
one NVLS multicast push for all of them, or one point-to-point push each,
``--transport``). Every version, a seeded 10 % of the tensors get +N(0, 1e-3); the
update arrives from pinned host memory (H2D) and is applied on the trainer.
The trainer then pushes the version (K4: hash every chunk, move only chunks
whose digest changed, quantize in fp8 mode) into the rollout's receive buffer
over NVLink, and, with persistence on, seals and promotes the version in
offloadd (changed tensors copied by K1, unchanged ones carried forward). The
rollout re-hashes what it received (bf16 mode) and answers; the trainer reads
the answer back (D2H).

Reported per timed version (max over trainer ranks): ``push_ms`` (CUDA events
around the K4 launches: the weight-sync latency), ``seal_ms`` (host) and
``e2e_ms`` (host wall time from the H2D of the update to the rollout's
verified answer). ``value`` is the median push latency.

    torchrun --nproc-per-node 8 bench.py --workload weight_sync --gpus 8 --steps 20 --warmup 3
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


def run(args, metric: str) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    replicas = max(1, int(getattr(args, "rollout_replicas", 1)))
    if world < 2 or world % (1 + replicas):
        raise SystemExit(f"weight_sync needs a multiple of {1 + replicas} GPUs (trainer + {replicas} rollout engines)")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    # trainer/rollout pairs exchange hashes with plain send/recv on the default group
    os.environ.setdefault("TORCH_NCCL_SHOW_EAGER_INIT_P2P_SERIALIZATION_WARNING", "false")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    tp = world // (1 + replicas)
    trainer = rank < tp
    tp_rank = rank % tp
    engine = rank // tp - 1  # rollout engine index (-1 on trainer ranks)
    spec = MODELS.get(args.model or "qwen2.5-32b", QWEN2_5_32B)
    shapes = param_shapes(spec, tp_rank, tp, layers=args.layers or None)
    shard_bytes = num_params(shapes) * 2
    mode = args.push_mode

    # persistence needs pinned room for one full shard per trainer plus the
    # changed tensors of the retained versions: until a seal drops the oldest
    # one, two older diffs and the version being written are live (x6 margin
    # for the contiguous runs that multi-GB tensors need)
    n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    per_trainer_gb = int(shard_bytes * (1.0 + 6 * args.change_fraction) / GiB) + 4
    need = per_trainer_gb * GiB * min(tp, n_local)
    persist = bool(args.persist)
    avail = host_mem_available_bytes()
    if persist and avail and need > 0.7 * avail:
        persist = False
    flag = torch.tensor([int(persist)], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    persist = bool(flag.item())
    windows = [per_trainer_gb if (i < tp and persist) else 0 for i in range(n_local)]
    if not any(windows):
        windows[0] = 1
    run_dir = os.environ.get("OFLD_BENCH_DIR", "/tmp/ofld_wsync")
    # 2 MiB slots: a model has hundreds of small tensors (norms, biases)
    sock, daemon = start_node_daemon(local_rank, n_local, windows, run_dir, barrier=dist.barrier, slot_mb=2,
                                     extra_yaml="manifest:\n  retain_sealed_versions: 2\n")

    from .. import offload_context
    from .._native import native

    sess = offload_context(daemon_addr=sock, device=device, rank=rank, local_rank=local_rank, world_rank=rank,
                           job_name="wsync-bench", eager_register=persist and trainer)
    off = sess.off
    layout = WeightLayout([(n, s, torch.bfloat16) for n, s in shapes], mode)
    rw = tr = None
    names = [n for n, _ in shapes]
    if not trainer:
        rw = RolloutWeights(layout, device)
        rw.publish(off, f"rollout/{engine}/{tp_rank}")
    dist.barrier()
    if trainer:
        params = random_init(shapes, device, seed=1000 + tp_rank)
        tr = TrainerWeightSync(off, params, [f"rollout/{j}/{tp_rank}" for j in range(replicas)], mode=mode,
                               persist=persist, tp_rank=tp_rank, transport=args.transport)
    else:
        rw.connect(off)
    dist.barrier()
    transport = tr.transport if trainer else rw.transport
    if trainer:
        # pinned host pool of update deltas: as large as the largest tensor,
        # sliced cyclically (N(0, delta_std) drawn on the GPU, copied once)
        biggest = max(t.numel() for t in params.values())
        scratch = torch.empty(biggest, dtype=torch.bfloat16, device=device)
        scratch.normal_(0.0, args.delta_std, generator=torch.Generator(device=device).manual_seed(7 + tp_rank))
        pool = torch.empty(biggest, dtype=torch.bfloat16, pin_memory=True)
        pool.copy_(scratch)
    nitems = len(shapes)
    peers = [tp_rank + tp * (1 + j) for j in range(replicas)] if trainer else [tp_rank]
    hbuf = torch.zeros(2 * nitems, dtype=torch.int64, device=device)
    ack = torch.zeros(2, dtype=torch.int64, device=device)
    ack_host = torch.zeros(2, dtype=torch.int64, pin_memory=True)

    def version_step(v: int, stats):
        t0 = time.perf_counter()
        pushed = h2d = 0
        chosen = []
        if trainer:
            if v > 1:
                # H2D of this version's update from pinned memory, applied on the device
                chosen = pick_changed(names, args.change_fraction, seed=v * 7919 + tp_rank)
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
        res = {}
        if trainer:
            before = tr.pushers[0].result()["bytes_stored"]
            hint = [names[i] for i in chosen] if (args.hint and v > 1) else None
            res = tr.publish_version(v, changed=hint)
            pushed = tr.pushers[0].result()["bytes_stored"] - before
            hbuf.copy_(tr.pushers[0].item_hash)
            for q in peers:
                dist.send(hbuf, q)
            acks = 0
            for q in peers:
                dist.recv(ack, q)
                acks += int(ack[0].item())
            ack.fill_(acks)
            ack_host.copy_(ack)  # D2H of the rollouts' answers
        else:
            dist.recv(hbuf, peers[0])
            ok = 1
            if args.verify and mode == "bf16":
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
            stats["e2e_ms"].append(float(rows[:tp, 2].max()))
            stats["bytes"].append(float(rows[:tp, 3].sum()))
            stats["verify_fail"] += int(rows[tp:, 4].sum())
            stats["h2d"].append(float(rows[:tp, 5].sum()))
            stats["changed"].append(float(rows[:tp, 6].sum()))

    for v in range(1, args.warmup + 1):
        version_step(v, None)
    stats = {"push_ms": [], "seal_ms": [], "e2e_ms": [], "bytes": [], "h2d": [], "changed": [], "verify_fail": 0}
    launches0 = native().kernel_launch_count()
    sampler = ClockSampler([local_rank]).start().wait_first()
    dist.barrier()
    sampler.mark_start()
    for v in range(args.warmup + 1, args.warmup + args.steps + 1):
        version_step(v, stats)
    sampler.mark_end()
    clocks = sampler.stop()
    launches = torch.tensor([native().kernel_launch_count() - launches0], device=device)
    dist.all_reduce(launches)
    out = None
    if rank == 0:
        push = sorted(stats["push_ms"])
        med = statistics.median(push)
        full = param_shapes(spec, 0, 1, layers=args.layers or None)
        out = {
            "metric": metric, "workload": "weight_sync", "value": round(med, 4),
            "unit": "ms (device, max over trainer ranks, median over versions)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init N(0,0.02) weights of the named architecture; seeded 10% of tensors "
                    "+N(0,1e-3) per version, update fed from pinned host memory",
            "config": {"model": f"{spec.name}-shaped" + (f" ({args.layers} layers)" if args.layers else ""),
                       "params": num_params(full), "model_bytes": num_params(full) * 2,
                       "trainer": f"TP={tp} on GPUs 0-{tp - 1}",
                       "rollout": f"{replicas} x TP={tp} on GPUs {tp}-{world - 1}",
                       "transport": transport, "push_mode": mode, "change_fraction": args.change_fraction,
                       "global_batch": 1, "seq_len": 0,
                       "parallelism": f"tp{tp}->tp{tp}" + (f" x{replicas}" if replicas > 1 else ""),
                       "persist": persist, "slot_mb": 2,
                       "change_detection": "caller hint" if args.hint else "device hash of every tensor",
                       "l2": "every push reads the whole shard (GBs) from HBM; no flush needed"},
            "push_ms_p90": round(push[min(len(push) - 1, int(0.9 * len(push)))], 4),
            "push_ms_max": round(push[-1], 4),
            "pushed_source_bytes_per_version": int(statistics.median(stats["bytes"])),
            "changed_tensors_per_version": int(statistics.median(stats["changed"])),
            "source_gbs_per_trainer": round(statistics.median(stats["bytes"]) / tp / (med / 1e3) / 1e9, 2),
            "seal_ms_median": round(statistics.median(stats["seal_ms"]), 3) if persist else None,
            "verify_failures": stats["verify_fail"],
            "e2e": {"value": round(statistics.median(stats["e2e_ms"]), 3),
                    "unit": "ms (host wall: H2D update + push + seal + rollout verify + D2H answer, max over ranks)",
                    "h2d_bytes_per_step": int(statistics.median(stats["h2d"])),
                    "d2h_bytes_per_step": 16 * tp},
            "delivered_bytes_per_version": int(statistics.median(stats["bytes"])) * replicas,
            "gpu_launches": int(launches.item()),
            "clocks": clocks,
        }
    if tr:
        tr.close()
    if rw:
        rw.close()
    sess.close()
    dist.barrier()
    dist.destroy_process_group()
    if daemon is not None:
        daemon.stop()
    return out
