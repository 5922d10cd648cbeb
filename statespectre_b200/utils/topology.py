"""Node topology: GPU -> NUMA node affinity and daemon config generation."""

from __future__ import annotations

import os
from typing import Dict, List


def gpu_numa_nodes(num_gpus: int) -> List[int]:
    """NUMA node of each visible GPU (0 when unknown)."""
    out = []
    try:
        import torch
    except ImportError:  # pragma: no cover
        return [0] * num_gpus
    for i in range(num_gpus):
        node = 0
        try:
            bus = torch.cuda.get_device_properties(i).pci_bus_id.lower()
            if bus.count(":") == 1:
                bus = "0000:" + bus
            parts = bus.split(":")
            parts[0] = parts[0][-4:].rjust(4, "0")
            path = f"/sys/bus/pci/devices/{':'.join(parts)}/numa_node"
            with open(path) as f:
                node = max(int(f.read().strip()), 0)
        except Exception:  # noqa: BLE001
            node = 0
        out.append(node)
    return out


def daemon_yaml(socket_path: str, gpu_nodes: List[int], window_gb_per_gpu, slot_mb: int = 64,
                overflow_gb: int = 1, drain_on_complete: bool = False, extra: str = "",
                drain_target: str = "pageable", nvme_dir: str = "", tier_threads: str = "") -> str:
    """A daemon config with one arena per NUMA node holding a window per GPU.

    ``window_gb_per_gpu`` is one size for every GPU or a list (one per GPU;
    GPUs with 0 get no window and allocate from the overflow pool).
    ``tier_threads`` "drain,readback,copy" sets drain_policy's drain and
    readback worker counts and its copy-pool size (empty: the defaults)."""
    sizes = list(window_gb_per_gpu) if isinstance(window_gb_per_gpu, (list, tuple)) else \
        [window_gb_per_gpu] * len(gpu_nodes)
    sizes += [0] * (len(gpu_nodes) - len(sizes))
    by_node: Dict[int, List[int]] = {}
    for g, n in enumerate(gpu_nodes):
        if sizes[g] > 0:
            by_node.setdefault(n, []).append(g)
    lines = ["daemon:", f"  socket_path: {socket_path}", "  heartbeat_timeout_ms: 30000",
             "arenas:", f"  allocation_granularity_mb: {slot_mb}", "  per_numa:"]
    for node, gpus in sorted(by_node.items()):
        size = sum(sizes[g] for g in gpus) + overflow_gb
        lines += [f"    - numa_node: {node}", f"      size_gb: {size}", f"      overflow_gb: {overflow_gb}",
                  "      gpu_windows:"]
        for g in gpus:
            lines += [f"        - gpu: {g}", f"          size_gb: {sizes[g]}"]
    lines += ["drain_policy:", f"  target_tier: {drain_target}",
              f"  drain_on_d2h_complete: {str(drain_on_complete).lower()}"]
    if tier_threads:
        dw, rw, ct = (int(x) for x in tier_threads.split(","))
        lines += [f"  drain_workers: {dw}", f"  readback_workers: {rw}", f"  copy_threads: {ct}"]
    lines += ["nvme:"]
    if nvme_dir:
        lines += ["  enabled: true", f"  path: {nvme_dir}", "  io_engine: io_uring", "  direct_io: true"]
    else:
        lines += ["  enabled: false"]
    return "\n".join(lines) + "\n" + extra


def host_numa_nodes() -> List[int]:
    base = "/sys/devices/system/node"
    try:
        return sorted(int(d[4:]) for d in os.listdir(base) if d.startswith("node") and d[4:].isdigit())
    except OSError:
        return [0]
