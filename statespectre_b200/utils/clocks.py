"""Sample GPU clocks and throttle reasons while a timed region runs.

Runs ``nvidia-smi --query-gpu=... -lms 200`` in the background (read-only
queries; no GPU setting is changed) and summarises the samples as
``{"sm_mhz": median, "sm_max_mhz": ..., "reasons": [...], "samples": n}``.
"""

from __future__ import annotations

import shutil
import statistics
import subprocess
import threading
import time
from typing import List, Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_indices: Optional[List[int]] = None, period_ms: int = 100):
        self.gpus = gpu_indices
        self.period_ms = period_ms
        self.rows: List[list] = []  # [monotonic time, *csv fields]
        self._proc = None
        self._thread = None
        self._window = None

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        args = [exe, f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
        if self.gpus:
            args.append("--id=" + ",".join(str(g) for g in self.gpus))
        self._proc = subprocess.Popen(args, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)

        def reader():
            for line in self._proc.stdout:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    self.rows.append([time.monotonic()] + parts)

        self._thread = threading.Thread(target=reader, daemon=True)
        self._thread.start()
        return self

    def wait_first(self, timeout_s: float = 5.0) -> "ClockSampler":
        """Block until nvidia-smi delivered its first sample (it starts slowly)."""
        end = time.monotonic() + timeout_s
        while self._proc is not None and not self.rows and time.monotonic() < end:
            time.sleep(0.02)
        return self

    def mark_start(self) -> None:
        self._window = [time.monotonic(), None]

    def mark_end(self) -> None:
        if self._window:
            self._window[1] = time.monotonic()

    def stop(self) -> dict:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            if self._thread:
                self._thread.join(timeout=2)
        return self.summary()

    def summary(self) -> dict:
        rows = self.rows
        if self._window and self._window[1] is not None and rows:
            # samples inside the marked window, plus the nearest one on each side
            t0, t1 = self._window
            inside = [i for i, r in enumerate(rows) if t0 <= r[0] <= t1]
            before = [i for i, r in enumerate(rows) if r[0] < t0][-1:]
            after = [i for i, r in enumerate(rows) if r[0] > t1][:1]
            rows = [rows[i] for i in before + inside + after]
        rows = [r[1:] for r in rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm, mx, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(REASON_COLS, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}
