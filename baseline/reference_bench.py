"""Reference arm of ``bench.py``: the unmodified StateSpectre build in
``baseline/_ref`` run through its own public Python API on the same box.

Workload and timing match the main arm exactly:
  * a bf16 N(0,1) tensor of ``--size-mb`` (1 GiB by default) per GPU, an
    8192x8192 bf16 matmul loop running concurrently on its own stream;
  * one step = ``off.copy(x, stream=s, wait=True)`` (D2H into the pinned
    arena, StateSpectre's ``cudaMemcpyAsync`` at src/agent/agent.cpp:825-829)
    then ``h.restore_into(x, stream=s, wait=True)`` (H2D,
    src/agent/agent.cpp:992-996) and ``h.discard()``;
  * W warm-up steps, K timed steps between barrier + synchronize, CUDA events
    on the copy stream, max over ranks; value = N * K * 2 * bytes / time;
  * e2e: ``off.evict(x, wait=True)`` (VRAM released), ``h.restore()`` and a
    16-byte device-to-host read of the restored tensor, host-timed.

The daemon is the reference's own ``offloadd`` (baseline/_ref/bin) with a
config in its YAML schema: one arena per NUMA node with a window per GPU,
64 MiB slots, no drain, no NVMe. Nothing from statespectre_b200 is imported:
the only helper loaded is the nvidia-smi clock sampler, by file path.
"""

from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")


def _isolate_sys_path() -> None:
    """Put the reference install first and drop the repository root, whose
    import-compatible ``state_spectre`` package would otherwise shadow it."""
    bad = {ROOT, "", "."}
    sys.path[:] = [p for p in sys.path if os.path.abspath(p or ".") != ROOT and p not in bad]
    sys.path.insert(0, REF)


def _clock_sampler_cls():
    spec = importlib.util.spec_from_file_location("_ref_clocks", os.path.join(ROOT, "statespectre_b200", "utils",
                                                                                "clocks.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.ClockSampler


def _gpu_numa_node(index: int) -> int:
    """NUMA node of CUDA device ``index`` from sysfs (PCI bus order), 0 when unknown."""
    base = "/sys/bus/pci/drivers/nvidia"
    try:
        bdfs = sorted(d for d in os.listdir(base) if d.count(":") == 2)
        with open(os.path.join(base, bdfs[index], "numa_node")) as f:
            n = int(f.read().strip())
        return max(n, 0)
    except (OSError, IndexError, ValueError):
        return 0


def reference_yaml(sock: str, ngpus: int, window_gb: int, overflow_gb: int = 1, slot_mb: int = 64) -> str:
    by_node = {}
    for g in range(ngpus):
        by_node.setdefault(_gpu_numa_node(g), []).append(g)
    lines = ["daemon:", f"  socket_path: {sock}", f"  control_shm_name: /ssref_ctrl_{os.getpid()}",
             "  heartbeat_timeout_ms: 30000", "arenas:", "  registration_policy: eager",
             f"  allocation_granularity_mb: {slot_mb}", "  per_numa:"]
    for node, gpus in sorted(by_node.items()):
        lines += [f"    - numa_node: {node}", f"      size_gb: {window_gb * len(gpus) + overflow_gb}",
                  f"      overflow_gb: {overflow_gb}", "      gpu_windows:"]
        for g in gpus:
            lines += [f"        - gpu: {g}", f"          size_gb: {window_gb}"]
    lines += ["drain_policy:", "  target_tier: pageable", "  drain_on_d2h_complete: false",
              "nvme:", "  enabled: false"]
    return "\n".join(lines) + "\n"


def unavailable(reason: str) -> dict:
    return {"impl": "reference", "unavailable": reason}


def ensure_built() -> str:
    """'' when the reference build is present (building it if needed), else why not."""
    sys.path.insert(0, HERE)
    try:
        import build_reference  # noqa: PLC0415
    finally:
        sys.path.remove(HERE)
    if build_reference.built():
        return ""
    try:
        build_reference.build()
    except Exception as e:  # noqa: BLE001
        return f"reference build failed: {e}"
    return "" if build_reference.built() else "reference build produced no extension"


def run(args, metric: str, baseline_roundtrip_gbs: float) -> dict | None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    why = ensure_built() if local_rank == 0 else ""
    _isolate_sys_path()
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        flag = torch.tensor([1 if why else 0], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if flag.item() and not why:
            why = "reference build failed on local rank 0"
    if why:
        if world > 1:
            dist.destroy_process_group()
        return unavailable(why) if rank == 0 else None

    import state_spectre  # the reference package, from baseline/_ref

    if not os.path.abspath(state_spectre.__file__).startswith(REF):
        return unavailable(f"state_spectre resolved to {state_spectre.__file__}, not the reference build")

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sweep_sizes = []
    if getattr(args, "workload", "evict_restore") == "sweep":
        s_ = 4096
        while s_ <= (args.max_size_mb << 20):
            sweep_sizes.append(s_)
            s_ <<= 1
    nbytes = args.size_mb << 20 if not sweep_sizes else sweep_sizes[-1]
    window_gb = max(4, (3 * nbytes >> 30) + 2, int(getattr(args, "arena_gb", 0) or 0))
    run_dir = os.environ.get("OFLD_REF_BENCH_DIR", "/tmp/ssref_bench")
    os.makedirs(run_dir, exist_ok=True)
    sock = os.path.join(run_dir, "offloadd.sock")
    daemon = None
    log = None
    if local_rank == 0:
        if os.path.exists(sock):
            os.unlink(sock)
        cfg = os.path.join(run_dir, "offloadd.yaml")
        n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
        with open(cfg, "w") as f:
            f.write(reference_yaml(sock, max(n_local, torch.cuda.device_count()), window_gb))
        log = open(os.path.join(run_dir, "offloadd.log"), "w")
        daemon = subprocess.Popen([os.path.join(REF, "bin", "offloadd"), "--config", cfg, "--socket", sock],
                                  stdout=log, stderr=log)
        deadline = time.time() + 300
        while not os.path.exists(sock) and time.time() < deadline and daemon.poll() is None:
            time.sleep(0.05)
        if not os.path.exists(sock):
            raise RuntimeError(f"reference offloadd did not come up (rc={daemon.poll()}, log {log.name})")
    barrier()
    if world > 1 and local_rank != 0:
        deadline = time.time() + 120
        while not os.path.exists(sock) and time.time() < deadline:
            time.sleep(0.05)

    sess = state_spectre.offload_context(daemon_addr=sock, device=device, rank=rank, local_rank=local_rank,
                                         world_rank=rank, eager_register=True)
    off = sess.__enter__()
    if sweep_sizes:
        return _sweep(args, metric, state_spectre, off, sess, sweep_sizes, world, rank, device, window_gb,
                      max_over_ranks, barrier, daemon, log)
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=device, generator=g)
    ref_copy = x.clone()
    torch.cuda.synchronize(device)  # the copy stream must not read x before it is written
    copy_stream = torch.cuda.Stream(device=device, priority=-1)

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

    evict_ms, restore_ms = [], []

    def cycle(record: bool):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        e0.record(copy_stream)
        h = off.copy(x, stream=copy_stream, wait=True)
        e1.record(copy_stream)
        h.restore_into(x, stream=copy_stream, wait=True)
        e2.record(copy_stream)
        h.discard()
        if record:
            e2.synchronize()
            evict_ms.append(e0.elapsed_time(e1))
            restore_ms.append(e1.elapsed_time(e2))

    for _ in range(args.warmup):
        cycle(False)
    torch.cuda.synchronize(device)
    assert torch.equal(x, ref_copy), "reference round trip corrupted the tensor"
    sampler = _clock_sampler_cls()([local_rank]).start().wait_first()
    barrier()
    torch.cuda.synchronize(device)
    sampler.mark_start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(copy_stream)
    for _ in range(args.steps):
        cycle(False)
    t_end.record(copy_stream)
    torch.cuda.synchronize(device)
    sampler.mark_end()
    barrier()
    clocks = sampler.stop()
    dev_ms_max = max_over_ranks(t_start.elapsed_time(t_end))
    value = world * args.steps * 2 * nbytes / (dev_ms_max / 1e3) / 1e9
    for _ in range(3):
        cycle(True)
    # each rank's median, then the slowest rank's (the same basis as this repository's arm)
    ev = max_over_ranks(sorted(evict_ms)[len(evict_ms) // 2])
    rs = max_over_ranks(sorted(restore_ms)[len(restore_ms) // 2])

    e2e_steps = args.e2e_steps or args.steps
    torch.cuda.synchronize(device)
    barrier()
    t0 = time.perf_counter()
    ok = True
    probe = ref_copy.view(torch.int64)[:2].cpu()
    for _ in range(e2e_steps):
        h = off.evict(x, wait=True)                  # D2H, VRAM released
        x = h.restore()                              # H2D from the pinned arena
        ok &= torch.equal(x.view(torch.int64)[:2].cpu(), probe)   # 16 B read back
        h.discard()
    torch.cuda.synchronize(device)
    e2e_s_max = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = world * e2e_steps * 2 * nbytes / e2e_s_max / 1e9
    stop_mm.set()
    if mm_thread:
        mm_thread.join(timeout=30)
    assert ok and torch.equal(x, ref_copy), "reference e2e round trip corrupted the tensor"
    sess.close()
    barrier()
    if daemon is not None:
        daemon.terminate()
        try:
            daemon.wait(timeout=30)
        except subprocess.TimeoutExpired:
            daemon.kill()
        log.close()
    ws = None
    if world >= 2 and getattr(args, "weight_sync", 1) and world % 2 == 0:
        ws = run_weight_sync(args, world, rank, local_rank, device, state_spectre,
                             versions=getattr(args, "ref_ws_versions", 3), warmup=1)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    out = {
        "impl": "reference",
        "metric": metric,
        "value": round(value, 3),
        "unit": "GB/s (aggregate over all GPUs, evict+restore bytes / device time)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms_max / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": round(value / (world * baseline_roundtrip_gbs), 4),
        "dtype": "bf16",
        "data": "synthetic: bf16 N(0,1) random tensor, seeded per rank",
        "config": {
            "model": "single-B200 eviction sweep point: bf16 tensor evict + restore through StateSpectre's "
                     "offload_context (cudaMemcpyAsync D2H/H2D into its registered pinned arena)",
            "tensor_bytes": nbytes, "global_batch": world, "seq_len": 0, "parallelism": f"dp{world}",
            "concurrent_matmul": "8192x8192 bf16 loop" if args.matmul else "none",
            "engine": "copy_engine (reference build, baseline/_ref)", "slot_mb": 64,
            "l2": "inputs (1 GiB) larger than the 126 MB L2; no flush needed",
        },
        "evict_gbs_per_gpu": round(nbytes / (ev / 1e3) / 1e9, 3),
        "restore_gbs_per_gpu": round(nbytes / (rs / 1e3) / 1e9, 3),
        "per_gpu_basis": "slowest rank's median of 3 separately timed evicts / restores",
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s (aggregate, public API, host-timed)",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes + 16},
        "gpu_launches": 0,
        "clocks": clocks,
        "matmul_iters": mm_count[0],
        "reference_build": os.path.relpath(REF, ROOT),
    }
    if ws is not None:
        out["weight_sync"] = ws
    return out


def _sweep(args, metric, state_spectre, off, sess, sizes, world, rank, device, window_gb, max_over_ranks,
           barrier, daemon, log):
    """The size sweep through the reference: bf16 N(0,1) tensors 4 KB .. max,
    ``copy(wait=True)`` + ``restore_into(wait=True)`` per repeat, each
    direction timed with CUDA events on the copy stream, max over ranks,
    median over repeats, under the same GEMM loop."""
    import statistics

    import torch
    import torch.distributed as dist

    stream = torch.cuda.Stream(device=device, priority=-1)
    stop_mm = threading.Event()
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

        mm_thread = threading.Thread(target=mm_loop, daemon=True)
        mm_thread.start()
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    rows = []
    sampler = _clock_sampler_cls()([int(device.index)]).start().wait_first()
    sampler.mark_start()
    for nbytes in sizes:
        x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=device, generator=g)
        ref = x.clone()
        torch.cuda.synchronize(device)  # the copy stream must not read x before it is written
        ev, rs = [], []
        for i in range(args.warmup + args.steps):
            barrier()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            h = off.copy(x, stream=stream, wait=True)
            e1.record(stream)
            h.restore_into(x, stream=stream, wait=True)
            e2.record(stream)
            h.discard()
            e2.synchronize()
            if i >= args.warmup:
                ev.append(max_over_ranks(e0.elapsed_time(e1)))
                rs.append(max_over_ranks(e1.elapsed_time(e2)))
        ok = bool(torch.equal(x, ref))
        e_ms, r_ms = statistics.median(ev), statistics.median(rs)
        rows.append({"bytes": nbytes, "evict_gbs": round(nbytes / (e_ms / 1e3) / 1e9, 3),
                     "restore_gbs": round(nbytes / (r_ms / 1e3) / 1e9, 3), "evict_ms": round(e_ms, 4),
                     "restore_ms": round(r_ms, 4), "byte_exact": ok})
        del x, ref
    sampler.mark_end()
    clocks = sampler.stop()
    stop_mm.set()
    if mm_thread:
        mm_thread.join(timeout=30)
    sess.close()
    barrier()
    if daemon is not None:
        daemon.terminate()
        try:
            daemon.wait(timeout=30)
        except subprocess.TimeoutExpired:
            daemon.kill()
        log.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    head = next((r for r in rows if r["bytes"] == 1 << 30), rows[-1])
    rt = 2 * head["bytes"] / ((head["evict_ms"] + head["restore_ms"]) / 1e3) / 1e9
    return {"impl": "reference", "metric": metric, "workload": "sweep", "value": round(rt * world, 3),
            "unit": "GB/s (aggregate round trip at the 1 GiB point; per-size rows below)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(head["evict_ms"] + head["restore_ms"], 4), "higher_is_better": True,
            "scaling": "weak", "dtype": "bf16", "data": "synthetic: bf16 N(0,1) per size, seeded per rank",
            "config": {"model": "evict/restore size sweep through the reference (cudaMemcpyAsync)",
                       "arena_gb_per_gpu": window_gb, "slot_mb": 64,
                       "concurrent_matmul": "8192x8192 bf16 loop" if args.matmul else "none"},
            "sweep": rows, "all_byte_exact": all(r["byte_exact"] for r in rows), "clocks": clocks}


# ---------------------------------------------------------------------------
# Weight sync through the reference: the same Qwen2.5-32B-shaped TP shards and
# per-version update as the main arm, moved the way StateSpectre moves a
# sealed version (python_api/state_spectre/__init__.py:575-633,
# _rollout.py:64-189, tests/python/trainer_seal.py): every trainer rank
# canonical_evicts each tensor of its shard under the new model version
# (D2H into the pinned arena), one rank promotes the version, and every
# rollout rank reads the manifest of its TP shard and pulls the changed
# objects over TCP from the daemon (RolloutWeightClient), then copies them
# into its GPU tensors. The previous version is dropped once pulled.
# ---------------------------------------------------------------------------

QWEN2_5_32B = dict(layers=64, hidden=5120, ffn=27648, heads=40, kv_heads=8, head_dim=128, vocab=152064)


def qwen_shard_shapes(tp_rank: int, tp: int, layers: int):
    """(name, shape) of one TP shard in Hugging Face parameter order."""
    c = QWEN2_5_32B
    h, q, kv = c["hidden"], c["heads"] * c["head_dim"] // tp, c["kv_heads"] * c["head_dim"] // tp
    f, v = c["ffn"] // tp, c["vocab"] // tp
    out = [("model.embed_tokens.weight", (v, h))]
    for i in range(layers):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (h,)), (p + "self_attn.q_proj.weight", (q, h)),
                (p + "self_attn.q_proj.bias", (q,)), (p + "self_attn.k_proj.weight", (kv, h)),
                (p + "self_attn.k_proj.bias", (kv,)), (p + "self_attn.v_proj.weight", (kv, h)),
                (p + "self_attn.v_proj.bias", (kv,)), (p + "self_attn.o_proj.weight", (h, q)),
                (p + "post_attention_layernorm.weight", (h,)), (p + "mlp.gate_proj.weight", (f, h)),
                (p + "mlp.up_proj.weight", (f, h)), (p + "mlp.down_proj.weight", (h, f))]
    out += [("model.norm.weight", (h,)), ("lm_head.weight", (v, h))]
    return out


def _changed(names, fraction: float, seed: int):
    import torch

    gen = torch.Generator()
    gen.manual_seed(seed)
    k = max(1, int(round(fraction * len(names))))
    return sorted(torch.randperm(len(names), generator=gen)[:k].tolist())


def run_weight_sync(args, world: int, rank: int, local_rank: int, device, state_spectre, versions: int,
                    warmup: int) -> dict | None:
    import statistics

    import torch
    import torch.distributed as dist

    tp = world // 2
    trainer = rank < tp
    tp_rank = rank % tp
    layers = max(1, 64 * tp // 4)
    shapes = qwen_shard_shapes(tp_rank, tp, layers)
    names = [n for n, _ in shapes]
    shard_bytes = sum(2 * _numel(s) for _, s in shapes)
    trainer_group = dist.new_group(list(range(tp)))
    port = 47311
    run_dir = os.environ.get("OFLD_REF_BENCH_DIR", "/tmp/ssref_bench") + "_wsync"
    os.makedirs(run_dir, exist_ok=True)
    sock = os.path.join(run_dir, "offloadd.sock")
    daemon = log = None
    n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    if local_rank == 0:
        if os.path.exists(sock):
            os.unlink(sock)
        # trainer GPUs hold one version: the previous one is dropped before the
        # next is recorded (its rollout pull finished in the previous step), so
        # 8 GPUs fit the GPU hosts' ~196 GB of memory (two versions would pin 150 GB)
        win = int(shard_bytes / (1 << 30)) + 6
        by_node = {}
        for g in range(max(n_local, torch.cuda.device_count())):
            by_node.setdefault(_gpu_numa_node(g), []).append(g)
        lines = ["daemon:", f"  socket_path: {sock}", f"  control_shm_name: /ssref_ws_{os.getpid()}",
                 "  heartbeat_timeout_ms: 60000", "arenas:", "  registration_policy: eager",
                 "  allocation_granularity_mb: 2", "  per_numa:"]
        for node, gpus in sorted(by_node.items()):
            sizes = {g: (win if g < tp else 1) for g in gpus}
            lines += [f"    - numa_node: {node}", f"      size_gb: {sum(sizes.values()) + 2}", "      overflow_gb: 2",
                      "      gpu_windows:"]
            for g in gpus:
                lines += [f"        - gpu: {g}", f"          size_gb: {sizes[g]}"]
        lines += ["drain_policy:", "  target_tier: pageable", "  drain_on_d2h_complete: false", "nvme:",
                  "  enabled: false"]
        cfg = os.path.join(run_dir, "offloadd.yaml")
        with open(cfg, "w") as f:
            f.write("\n".join(lines) + "\n")
        log = open(os.path.join(run_dir, "offloadd.log"), "w")
        daemon = subprocess.Popen([os.path.join(REF, "bin", "offloadd"), "--config", cfg, "--socket", sock,
                                   "--tcp-port", str(port)], stdout=log, stderr=log)
        deadline = time.time() + 300
        while not os.path.exists(sock) and time.time() < deadline and daemon.poll() is None:
            time.sleep(0.05)
        if not os.path.exists(sock):
            raise RuntimeError(f"reference offloadd did not come up (log {log.name})")
    dist.barrier()
    ident = torch.zeros(2, dtype=torch.int64, device=device)
    sess = off = client = None
    if trainer:
        sess = state_spectre.offload_context(daemon_addr=sock, device=device, rank=rank, local_rank=local_rank,
                                             world_rank=rank, eager_register=True, job_name="wsync-ref")
        off = sess.__enter__()
        g = torch.Generator(device=device)
        g.manual_seed(1000 + tp_rank)
        params = {}
        for n, s in shapes:
            t = torch.empty(s, dtype=torch.bfloat16, device=device)
            t.normal_(1.0 if n.endswith("norm.weight") else 0.0, 0.02, generator=g)
            params[n] = t
        biggest = max(t.numel() for t in params.values())
        scratch = torch.empty(biggest, dtype=torch.bfloat16, device=device)
        scratch.normal_(0.0, float(args.delta_std), generator=torch.Generator(device=device).manual_seed(7 + tp_rank))
        pool = torch.empty(biggest, dtype=torch.bfloat16, pin_memory=True)
        pool.copy_(scratch)
        if tp_rank == 0:
            ident[0], ident[1] = int(off.job_id) & 0x7FFFFFFFFFFFFFFF, int(off.launch_epoch)
            ident_hi = int(off.job_id) >> 63
        dist.barrier(group=trainer_group)
    dist.broadcast(ident, 0)
    hi = torch.tensor([ident_hi if rank == 0 else 0], dtype=torch.int64, device=device)
    dist.broadcast(hi, 0)
    job_id = int(ident[0].item()) | (int(hi.item()) << 63)
    epoch = int(ident[1].item())
    if not trainer:
        from state_spectre._rollout import RolloutWeightClient

        client = RolloutWeightClient(f"tcp://127.0.0.1:{port}", job_id, epoch, recv_host="127.0.0.1")
        bufs = {n: torch.empty(s, dtype=torch.bfloat16, device=device) for n, s in shapes}
    peer = tp_rank + tp if trainer else tp_rank
    go = torch.zeros(1, dtype=torch.int64, device=device)

    def step(v: int, stats):
        t0 = time.perf_counter()
        h2d = 0
        if trainer:
            if v > 1:  # this version's update from pinned memory, applied on the device
                off_e = 0
                for i in _changed(names, args.change_fraction, seed=v * 7919 + tp_rank):
                    t = params[names[i]]
                    n = t.numel()
                    if off_e + n > pool.numel():
                        off_e = 0
                    scratch[:n].copy_(pool[off_e:off_e + n], non_blocking=True)
                    t.view(-1).add_(scratch[:n])
                    off_e += n
                    h2d += 2 * n
            torch.cuda.synchronize(device)
            if v > 1:  # the rollout finished pulling v - 1 in the previous step
                if tp_rank == 0:
                    off.drop_canonical_version("policy_rollout", v - 1)
                dist.barrier(group=trainer_group)  # every trainer's window is free again
            for n in names:  # the reference records every tensor of the version
                key = off.canonical_key(model_role="policy_rollout", model_version=v, param_name=n,
                                        tensor=params[n], pp_rank=0, tp_rank=tp_rank, expert_id=-1)
                off.canonical_evict(params[n], key, destructive=False, wait=True)
            dist.barrier(group=trainer_group)
            if tp_rank == 0:
                off.promote_rollout_version(v)
            dist.barrier(group=trainer_group)
            go.fill_(v)
            dist.send(go, peer)
            dist.recv(go, peer)  # the rollout's answer
            if int(go.item()) != 1:  # .item(): an NCCL recv only orders the stream, the host waits here
                raise RuntimeError(f"reference rollout pulled nothing for version {v}")
            dist.barrier(group=trainer_group)
        else:
            dist.recv(go, peer)
            if int(go.item()) != v:  # wait on the host for the trainer's promote of version v
                raise RuntimeError(f"rollout expected version {v}, trainer announced {int(go.item())}")
            man = client.get_manifest(v, {"tp": tp_rank})
            changed = {e["object_id"] for e in client.diff_local(man)}
            pulled = 0
            for e in man["tensors"]:
                if e["object_id"] not in changed:
                    continue
                payload = client.pull_tensor(e, v)
                dst = bufs[e["key"]["param_fqn_debug"]]
                dst.view(-1).view(torch.uint8).copy_(torch.frombuffer(payload, dtype=torch.uint8))
                pulled += len(payload)
            torch.cuda.synchronize(device)
            go.fill_(1 if pulled else 0)
            dist.send(go, peer)
        t1 = time.perf_counter()
        if stats is not None:
            vals = torch.tensor([(t1 - t0) * 1e3, float(h2d)], dtype=torch.float64, device=device)
            dist.all_reduce(vals[:1], op=dist.ReduceOp.MAX)
            stats["e2e_ms"].append(float(vals[0].item()))

    t_begin = time.time()
    for v in range(1, warmup + 1):
        step(v, None)
    stats = {"e2e_ms": []}
    sampler = _clock_sampler_cls()([local_rank]).start().wait_first()
    dist.barrier()
    sampler.mark_start()
    budget = float(getattr(args, "ref_ws_budget_s", 300.0))
    v = warmup + 1
    while v <= warmup + versions:
        step(v, stats)
        v += 1
        # every version moves the whole shard over TCP: stop early (same decision on every rank)
        over = torch.tensor([1.0 if time.time() - t_begin > budget else 0.0], device=device)
        dist.all_reduce(over, op=dist.ReduceOp.MAX)
        if over.item():
            break
    versions = len(stats["e2e_ms"])
    sampler.mark_end()
    clocks = sampler.stop()
    if sess is not None:
        sess.close()
    dist.barrier()
    if daemon is not None:
        daemon.terminate()
        try:
            daemon.wait(timeout=60)
        except subprocess.TimeoutExpired:
            daemon.kill()
        log.close()
    dist.destroy_process_group(trainer_group)
    if rank != 0:
        return None
    e2e = sorted(stats["e2e_ms"])
    return {
        "model": "Qwen2.5-32B-shaped" + (f" ({layers} of 64 layers)" if layers != 64 else ""),
        "trainer": f"TP={tp} on GPUs 0-{tp - 1}", "rollout": f"TP={tp} on GPUs {tp}-{world - 1}",
        "parallelism": f"tp{tp}->tp{tp}", "shard_bytes_per_trainer_gpu": shard_bytes,
        "change_fraction": args.change_fraction, "persist": True,
        "path": "canonical_evict of every tensor (wait=True) + promote_rollout_version; rollout "
                "RolloutWeightClient get_manifest(tp filter) + pull_tensor over TCP + H2D",
        "modes": {"bf16": {"e2e_ms": round(statistics.median(e2e), 3), "e2e_ms_max": round(e2e[-1], 3),
                           "versions": versions, "clocks": clocks},
                  "fp8": "not available: the reference has no fp8 weight path"},
    }


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def main(args, metric: str, baseline_roundtrip_gbs: float) -> int:
    out = run(args, metric, baseline_roundtrip_gbs)
    if out is not None:
        print(json.dumps(out), flush=True)
        if getattr(args, "out", ""):
            with open(args.out, "w") as f:
                f.write(json.dumps(out) + "\n")
    return 0
