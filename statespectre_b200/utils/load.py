"""Background GPU load for benchmarks: a bf16 GEMM loop on its own stream
(the "concurrent training step" of the offload workloads)."""

from __future__ import annotations

import threading

import torch


class GemmLoad:
    def __init__(self, device, n: int = 8192, dtype=torch.bfloat16):
        self.device = torch.device(device)
        self.n = n
        self.iters = 0
        self._stop = threading.Event()
        self._thread = None
        self._stream = torch.cuda.Stream(device=self.device)
        g = torch.Generator(device=self.device).manual_seed(17)
        self.a = torch.randn(n, n, dtype=dtype, device=self.device, generator=g)
        self.b = torch.randn(n, n, dtype=dtype, device=self.device, generator=g)
        self.c = torch.empty(n, n, dtype=dtype, device=self.device)

    def start(self) -> "GemmLoad":
        def loop():
            torch.cuda.set_device(self.device)
            with torch.cuda.stream(self._stream):
                while not self._stop.is_set():
                    for _ in range(8):
                        torch.matmul(self.a, self.b, out=self.c)
                    self._stream.synchronize()
                    self.iters += 8

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def stop(self) -> int:
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=60)
        return self.iters

    def describe(self) -> str:
        return f"{self.n}x{self.n} bf16 GEMM loop"
