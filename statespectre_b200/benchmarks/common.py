"""Shared plumbing of the benchmark workloads: rank environment, process
group, node daemon, device timing, max over ranks."""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..utils.launch import start_node_daemon


@dataclass
class Env:
    world: int
    rank: int
    local_rank: int
    n_local: int
    device: torch.device

    def barrier(self):
        if self.world > 1:
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return float(v)
        t = torch.tensor([float(v)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if self.world == 1:
            return float(v)
        t = torch.tensor([float(v)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.world > 1:
            dist.barrier()
            dist.destroy_process_group()


def setup() -> Env:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n_local = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    return Env(world, rank, local_rank, n_local, device)


def node_daemon(env: Env, window_gb, run_dir: str, slot_mb: int = 64, extra_yaml: str = "", **yaml_kw):
    return start_node_daemon(env.local_rank, env.n_local, window_gb, run_dir, barrier=env.barrier,
                             slot_mb=slot_mb, extra_yaml=extra_yaml, **yaml_kw)


class DeviceTimer:
    """CUDA events on one stream; elapsed() synchronizes the end event."""

    def __init__(self, stream):
        self.stream = stream
        self.e0 = torch.cuda.Event(enable_timing=True)
        self.e1 = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.e0.record(self.stream)
        return self

    def __exit__(self, *exc):
        self.e1.record(self.stream)

    def ms(self) -> float:
        self.e1.synchronize()
        return self.e0.elapsed_time(self.e1)
