"""Launching and talking to ``offloadd``.

``launch_daemon`` starts the daemon as a separate process (the production
shape: one daemon per node, every rank connects over its socket);
``in_process_daemon`` runs it on a thread of the calling process (tests and
single-process benchmarks). ``DaemonClient`` speaks the control protocol from
pure Python.
"""

from __future__ import annotations

import os
import signal
import subprocess
import tempfile
import time
from typing import Optional

from . import _wire
from ._native import bin_path, native


class DaemonProcess:
    """A running ``offloadd`` child process."""

    def __init__(self, args, socket_path: str, log_path: Optional[str], env=None):
        self.socket_path = socket_path
        self.log_path = log_path
        self._log = open(log_path, "ab") if log_path else subprocess.DEVNULL
        self.proc = subprocess.Popen(args, stdout=self._log, stderr=self._log, env=env)

    def wait_ready(self, timeout: float = 60.0) -> "DaemonProcess":
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            if self.proc.poll() is not None:
                raise RuntimeError(f"offloadd exited with code {self.proc.returncode} (log: {self.log_path})")
            if os.path.exists(self.socket_path):
                try:
                    with _wire.Connection(self.socket_path, timeout=5) as c:
                        c.call(_wire.Op.GET_STATS, rank_id=0xFFFFFFFF)
                    return self
                except OSError:
                    pass
            time.sleep(0.02)
        raise TimeoutError(f"offloadd did not come up on {self.socket_path}")

    def stats(self) -> dict:
        with _wire.Connection(self.socket_path) as c:
            r = c.call(_wire.Op.GET_STATS, rank_id=0xFFFFFFFF)
        return {e["key"]: e["value"] for e in r["stats"]}

    def stop(self, timeout: float = 15.0) -> int:
        if self.proc.poll() is None:
            try:
                with _wire.Connection(self.socket_path, timeout=2) as c:
                    c.call(_wire.Op.SHUTDOWN, token=0)
            except (OSError, _wire.WireError):
                self.proc.send_signal(signal.SIGTERM)
            try:
                self.proc.wait(timeout=timeout)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
        if self._log not in (None, subprocess.DEVNULL):
            self._log.close()
        return self.proc.returncode

    def kill(self) -> None:
        """Hard kill (crash tests)."""
        if self.proc.poll() is None:
            self.proc.kill()
            self.proc.wait()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.stop()


def launch_daemon(socket_path: Optional[str] = None, *, config: Optional[str] = None, arena_mb: int = 256,
                  slot_mb: Optional[int] = None, numa: int = 0, gpu: int = 0, tcp_port: int = 0,
                  trace: Optional[str] = None, nvme_dir: Optional[str] = None,
                  drain_on_complete: Optional[bool] = None, log_path: Optional[str] = None,
                  extra_args=(), wait: bool = True, env=None, binary: str = "offloadd") -> DaemonProcess:
    """Start ``offloadd`` (or a sanitizer build of it, ``binary="offloadd_asan"``
    / ``"offloadd_tsan"``); returns once it answers on its socket."""
    if socket_path is None:
        socket_path = os.path.join(tempfile.mkdtemp(prefix="offloadd-"), "offloadd.sock")
    args = [bin_path(binary), "--socket", socket_path]
    if config:
        args += ["--config", config]
    else:
        args += ["--smoke-arena-mb", str(arena_mb), "--numa", str(numa), "--gpu", str(gpu)]
    if slot_mb:
        args += ["--slot-mb", str(slot_mb)]
    if tcp_port:
        args += ["--tcp-port", str(tcp_port)]
    if trace:
        args += ["--trace", trace]
    if nvme_dir:
        args += ["--nvme-dir", nvme_dir]
    if drain_on_complete is not None:
        args += ["--drain-on-complete", "1" if drain_on_complete else "0"]
    args += list(extra_args)
    d = DaemonProcess(args, socket_path, log_path, env=env)
    return d.wait_ready() if wait else d


def in_process_daemon(**kw):
    """Run the daemon on a thread of this process (``_C.DaemonThread``).

    Keywords: socket, arena_mb, slot_mb, numa, gpu, yaml, drain_on_complete,
    heartbeat_timeout_ms, tcp_port, nvme_dir, direct_io, drain_target,
    pageable_limit_mb, io_engine, retain_sealed_versions, thresholds,
    quota_max_pinned_bytes, creating_policy, copy_threads.
    """
    if "socket" not in kw:
        kw["socket"] = os.path.join(tempfile.mkdtemp(prefix="offloadd-"), "offloadd.sock")
    d = native().DaemonThread(**kw)
    import atexit
    import weakref

    ref = weakref.ref(d)
    atexit.register(lambda: ref() is not None and ref().stop())
    return d


class DaemonClient(_wire.Connection):
    """Pure-Python control connection (``unix://path``, a path, or ``tcp://host:port``)."""

    def stats(self) -> dict:
        r = self.call(_wire.Op.GET_STATS, rank_id=0xFFFFFFFF)
        return {e["key"]: e["value"] for e in r["stats"]}

    def shutdown(self) -> dict:
        return self.call(_wire.Op.SHUTDOWN, token=0)
