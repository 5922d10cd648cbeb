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

    nbytes = args.size_mb << 20
    window_gb = max(4, (3 * nbytes >> 30) + 2)
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
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    x = torch.randn(nbytes // 2, dtype=torch.bfloat16, device=device, generator=g)
    ref_copy = x.clone()
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
    ev = sorted(evict_ms)[len(evict_ms) // 2]
    rs = sorted(restore_ms)[len(restore_ms) // 2]

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
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {
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
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s (aggregate, public API, host-timed)",
                "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes + 16},
        "gpu_launches": 0,
        "clocks": clocks,
        "matmul_iters": mm_count[0],
        "reference_build": os.path.relpath(REF, ROOT),
    }


def main(args, metric: str, baseline_roundtrip_gbs: float) -> int:
    out = run(args, metric, baseline_roundtrip_gbs)
    if out is not None:
        print(json.dumps(out), flush=True)
        if getattr(args, "out", ""):
            with open(args.out, "w") as f:
                f.write(json.dumps(out) + "\n")
    return 0
