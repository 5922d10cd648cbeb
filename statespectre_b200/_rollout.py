"""RolloutWeightClient: pull sealed model versions from a trainer's daemon.

Flow (StateSpectre's, reference: python_api/state_spectre/_rollout.py:40-197):
discover the latest promoted version, fetch its manifest, diff against the
local cache, pull only what changed. What this client does differently:

  * diff keys on the tensor's identity (param id + partition coordinates) and
    its content hash, so an unchanged tensor is skipped across versions even
    though each version has new object ids (StateSpectre's cache keyed on
    object_id re-pulled every tensor every version, reference: _rollout.py:89-98);
  * control RPCs reuse connections, and ``sync_latest(workers=N)`` keeps N
    pulls in flight, each with its own receive socket;
  * ``transport="file"`` pulls through a path on a shared filesystem;
  * ``daemon_addr`` may be ``tcp://host:port`` or a local socket path.
"""

from __future__ import annotations

import os
import socket
import tempfile
import threading
from concurrent.futures import ThreadPoolExecutor
from typing import Callable, Dict, Optional

from . import _wire
from ._wire import Op


def _identity(key: dict) -> tuple:
    return (key["param_id"], key["pp_rank"], key["tp_rank"], key["ep_rank"], key["etp_rank"], key["expert_id"],
            key["shard_offset"], key["shard_nbytes"])


class RolloutWeightClient:
    """Pull sealed weights; see module docstring."""

    def __init__(self, daemon_addr: str, job_id: int, launch_epoch: int, model_role="policy_rollout",
                 tenant_id: int = 0, job_name: str = "", recv_host: Optional[str] = None, timeout: float = 60.0):
        from .api import ModelRole

        if daemon_addr.startswith("tcp://"):
            host = daemon_addr[6:].rpartition(":")[0]
            self._local = host in ("127.0.0.1", "localhost", "::1")
        else:
            self._local = True
        self.daemon_addr = daemon_addr
        self.tenant_id = int(tenant_id)
        self.job_id = int(job_id)
        self.launch_epoch = int(launch_epoch)
        self.job_name = job_name
        self.model_role = ModelRole.parse(model_role)
        if recv_host is None:
            recv_host = "127.0.0.1" if self._local else socket.gethostbyname(socket.gethostname())
        self._recv_host = recv_host
        self._timeout = timeout
        self._tls = threading.local()
        self._cache: Dict[int, tuple] = {}      # object_id -> content hash (reference-compatible view)
        self._by_identity: Dict[tuple, tuple] = {}  # identity -> content hash
        self.bytes_pulled = 0

    # ---- control plane ----
    def _conn(self) -> _wire.Connection:
        c = getattr(self._tls, "conn", None)
        if c is None:
            c = _wire.Connection(self.daemon_addr, timeout=self._timeout)
            self._tls.conn = c
        return c

    def _job(self) -> dict:
        return {"tenant_id": self.tenant_id, "job_id": self.job_id, "launch_epoch": self.launch_epoch,
                "job_name": self.job_name}

    def get_latest_sealed_version(self) -> Optional[int]:
        r = self._conn().call(Op.GET_LATEST_SEALED_VERSION, job=self._job(), model_role=self.model_role)
        return r["model_version"] if r["ok"] and r["found"] else None

    def get_manifest(self, model_version: int, flt: Optional[dict] = None) -> dict:
        r = self._conn().call(Op.GET_MANIFEST, job=self._job(), model_role=self.model_role,
                              model_version=int(model_version), filter=flt or {})
        if not r["ok"]:
            raise IOError(f"get_manifest failed: {r['message']}")
        return r

    def diff_local(self, manifest: dict) -> list:
        """Manifest entries whose content is not in the local cache."""
        changed = []
        for e in manifest["tensors"]:
            h = (e["content_hash_lo"], e["content_hash_hi"])
            known = self._by_identity.get(_identity(e["key"]))
            if h == (0, 0) or known != h:
                if self._cache.get(e["object_id"]) != h or h == (0, 0):
                    changed.append(e)
        return changed

    def _remember(self, entry: dict) -> None:
        h = (entry["content_hash_lo"], entry["content_hash_hi"])
        self._cache[entry["object_id"]] = h
        self._by_identity[_identity(entry["key"])] = h

    # ---- data plane ----
    def pull_tensor(self, entry: dict, model_version: int, transport: str = "tcp",
                    libfabric_descriptor: Optional[str] = None, into: Optional[memoryview] = None) -> bytes:
        """Pull one manifest entry; returns its bytes (or fills ``into``)."""
        oid = int(entry["object_id"])
        expect = int(entry["nbytes"])
        base = {"job": self._job(), "model_role": self.model_role, "model_version": int(model_version),
                "object_id": oid}
        if transport == "tcp":
            lsock = getattr(self._tls, "listener", None)
            if lsock is None:
                lsock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
                lsock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
                lsock.bind(("127.0.0.1" if self._local else "0.0.0.0", 0))
                lsock.listen(4)
                lsock.settimeout(self._timeout)
                self._tls.listener = lsock
            target = f"{self._recv_host}:{lsock.getsockname()[1]}"
            result: dict = {}

            def rpc():
                try:
                    result["resp"] = self._conn_for_pull().call(Op.PULL_TENSOR, base, transport=_wire.TK_TCP,
                                                                 target_descriptor=target)
                except Exception as ex:  # noqa: BLE001
                    result["err"] = ex

            th = threading.Thread(target=rpc, daemon=True)
            th.start()
            try:
                conn, _ = lsock.accept()
            except socket.timeout:
                th.join(self._timeout)
                raise IOError(f"pull_tensor: daemon never connected back ({result})")
            with conn:
                meta = _wire.parse_export_header(_wire.recv_exact(conn, _wire.EXPORT_HEADER_SIZE))
                n = meta["nbytes"]
                buf = into if into is not None else memoryview(bytearray(n))
                got = 0
                while got < n:
                    k = conn.recv_into(buf[got:], n - got)
                    if k == 0:
                        raise ConnectionError("export stream closed early")
                    got += k
            th.join(self._timeout)
            if "err" in result:
                raise result["err"]
            if not result.get("resp", {}).get("ok"):
                raise IOError(f"pull_tensor failed: {result.get('resp', {}).get('message')}")
            if meta["object_id"] != oid or meta["nbytes"] != expect:
                raise IOError("pulled object/nbytes mismatch vs manifest")
            payload = buf if into is not None else bytes(buf)
        elif transport == "file":
            fd, path = tempfile.mkstemp(prefix=f"pull-{oid}-", dir=os.environ.get("OFLD_PULL_DIR"))
            os.close(fd)
            try:
                r = self._conn_for_pull().call(Op.PULL_TENSOR, base, transport=_wire.TK_FILE, target_descriptor=path)
                if not r["ok"]:
                    raise IOError(f"pull_tensor(file) failed: {r['message']}")
                with open(path, "rb") as f:
                    meta = _wire.parse_export_header(f.read(_wire.EXPORT_HEADER_SIZE))
                    if meta["object_id"] != oid or meta["nbytes"] != expect:
                        raise IOError("pulled object/nbytes mismatch vs manifest")
                    if into is not None:
                        f.readinto(into)
                        payload = into
                    else:
                        payload = f.read(expect)
            finally:
                os.unlink(path)
        elif transport in ("libfabric", "libfabric_send"):
            if not libfabric_descriptor:
                raise ValueError("libfabric transport needs libfabric_descriptor ('<nic>|<address_hex>')")
            r = self._conn_for_pull().call(Op.PULL_TENSOR, base, transport=_wire.TK_LIBFABRIC_SEND,
                                           target_descriptor=libfabric_descriptor)
            if not r["ok"]:
                raise IOError(f"pull_tensor(libfabric) failed: {r['message']}")
            payload = b""
        else:
            raise ValueError(f"unknown transport {transport!r}")
        self._remember(entry)
        self.bytes_pulled += expect
        return payload

    def _conn_for_pull(self) -> _wire.Connection:
        c = getattr(self._tls, "pull_conn", None)
        if c is None:
            c = _wire.Connection(self.daemon_addr, timeout=self._timeout)
            self._tls.pull_conn = c
        return c

    def sync_latest(self, transport: str = "tcp", workers: int = 1,
                    sink: Optional[Callable[[dict, bytes], None]] = None) -> dict:
        """Pull every changed tensor of the latest promoted version.

        ``sink(entry, data)`` receives each pulled tensor (for example to copy it
        into a GPU buffer); without a sink the bytes are returned in ``data``.
        Returns {"version", "pulled", "skipped", "bytes", "data"}.
        """
        version = self.get_latest_sealed_version()
        if version is None:
            return {"version": None, "pulled": [], "skipped": [], "bytes": 0, "data": {}}
        manifest = self.get_manifest(version)
        changed = self.diff_local(manifest)
        changed_ids = {e["object_id"] for e in changed}
        skipped = [e["object_id"] for e in manifest["tensors"] if e["object_id"] not in changed_ids]
        data: Dict[int, bytes] = {}
        lock = threading.Lock()

        def one(e):
            b = self.pull_tensor(e, version, transport=transport)
            if sink is not None:
                sink(e, b)
            else:
                with lock:
                    data[e["object_id"]] = b
            return e["object_id"], e["nbytes"]

        if workers <= 1:
            done = [one(e) for e in changed]
        else:
            with ThreadPoolExecutor(max_workers=workers) as ex:
                done = list(ex.map(one, changed))
        return {"version": version, "pulled": [o for o, _ in done], "skipped": skipped,
                "bytes": sum(n for _, n in done), "data": data}

    def close(self) -> None:
        for attr in ("conn", "pull_conn"):
            c = getattr(self._tls, attr, None)
            if c is not None:
                c.close()
                setattr(self._tls, attr, None)
        lsock = getattr(self._tls, "listener", None)
        if lsock is not None:
            lsock.close()
            self._tls.listener = None
