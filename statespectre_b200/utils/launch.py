"""Node-local daemon start-up shared by the benchmarks and harnesses.

Local rank 0 writes an offloadd config for the node (one pinned arena window
per GPU, grouped by NUMA node) and launches the daemon; the other local ranks
wait for its socket. Every rank then opens its own session.
"""

from __future__ import annotations

import os
import time
from typing import Optional, Tuple

from .topology import daemon_yaml, gpu_numa_nodes


def start_node_daemon(local_rank: int, n_local: int, window_gb, run_dir: str, barrier=None,
                      n_devices: Optional[int] = None, extra_yaml: str = "", slot_mb: int = 64,
                      **yaml_kw) -> Tuple[str, object]:
    """Returns (socket path, daemon handle or None on non-zero local ranks).

    ``window_gb`` is one size for every GPU or a list with one size per GPU."""
    from ..daemon import launch_daemon

    os.makedirs(run_dir, exist_ok=True)
    sock = os.path.join(run_dir, "offloadd.sock")
    daemon = None
    if local_rank == 0:
        if os.path.exists(sock):
            os.unlink(sock)
        cfg = os.path.join(run_dir, "offloadd.yaml")
        with open(cfg, "w") as f:
            f.write(daemon_yaml(sock, gpu_numa_nodes(max(n_local, n_devices or n_local)), window_gb,
                                slot_mb=slot_mb, extra=extra_yaml, **yaml_kw))
        daemon = launch_daemon(sock, config=cfg, log_path=os.path.join(run_dir, "offloadd.log"))
    if barrier is not None:
        barrier()
    if local_rank != 0:
        deadline = time.time() + 120
        while not os.path.exists(sock) and time.time() < deadline:
            time.sleep(0.05)
    return sock, daemon


def host_mem_available_bytes() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0
