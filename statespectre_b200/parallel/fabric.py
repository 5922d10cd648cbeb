"""Intra-node GPU fabric: device buffers shared between rank processes.

A rank exports the allocation behind a tensor as a CUDA IPC handle and
publishes it under a string key through offloadd's peer-buffer broker
(``PublishPeerBuffer`` / ``LookupPeerBuffer``); another rank on the same node
looks the key up and maps the buffer into its own address space. The mapped
pointer is only ever handed to this package's kernels (K3 verify loads, K4
weight-sync stores); it is deliberately not wrapped as a torch tensor, so no
library kernel is ever given another GPU's memory as an operand.

StateSpectre has no GPU-to-GPU path: replicas and rollout engines only meet
through host memory and TCP (reference: src/daemon/canonical_rollout.cpp:240-411).
"""

from __future__ import annotations

import torch

from .. import _wire
from .._native import native

KIND_RAW = 0
KIND_WEIGHTS = 1  # a rollout weight buffer laid out by parallel.weight_sync.WeightLayout
KIND_REPLICA = 2  # a DP replica's parameter for P2P hash verification


def export_tensor(t: torch.Tensor) -> dict:
    """IPC export of the allocation containing ``t`` (handle, offset, device)."""
    if t.device.type != "cuda":
        raise ValueError("export_tensor: a CUDA tensor is required")
    e = dict(native().ipc_export(t.data_ptr()))
    e["nbytes"] = t.numel() * t.element_size()
    return e


class PeerBuffer:
    """Another process's device buffer mapped into this one (raw pointer).

    ``ptr`` is valid on this process's current device once peer access is
    possible (CUDA IPC enables it lazily); ``close()`` drops the mapping
    reference (mappings are shared per allocation and refcounted)."""

    def __init__(self, key: str, ptr: int, nbytes: int, device: int, owner_rank: int, kind: int,
                 mapped: bool = True):
        self.key, self.ptr, self.nbytes = key, int(ptr), int(nbytes)
        self.device, self.owner_rank, self.kind = int(device), int(owner_rank), int(kind)
        self._mapped = mapped
        self._open = True

    def close(self) -> None:
        if self._open:
            if self._mapped:
                native().ipc_close(self.ptr)
            self._open = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __repr__(self) -> str:
        return (f"PeerBuffer(key={self.key!r}, owner_rank={self.owner_rank}, device={self.device}, "
                f"nbytes={self.nbytes}, open={self._open})")


# Handles exported by this process -> allocation base. CUDA IPC handles cannot
# be opened by the process that exported them, so such lookups resolve here.
_LOCAL_EXPORTS: dict = {}


def describe(key: str, t: torch.Tensor, owner_rank: int, kind: int = KIND_RAW) -> dict:
    e = export_tensor(t)
    _LOCAL_EXPORTS[bytes(e["handle"])] = int(e["base"])
    return {"key": key, "owner_rank": int(owner_rank), "device": int(e["device"]), "kind": int(kind),
            "nbytes": int(e["nbytes"]), "offset": int(e["offset"]), "handle": e["handle"]}


def publish(off, key: str, t: torch.Tensor, kind: int = KIND_RAW) -> dict:
    """Publish ``t`` under ``key`` through the daemon of session ``off``."""
    desc = describe(key, t, off.rank, kind)
    ok, msg = off._agent.publish_peer_buffer(_wire.encode("PeerBufferDesc", desc), -1)
    if not ok:
        raise RuntimeError(f"publish_peer_buffer({key!r}) failed: {msg}")
    return desc


def open_desc(desc: dict) -> PeerBuffer:
    """Map a published buffer description (from ``lookup`` or an out-of-band exchange)."""
    base = _LOCAL_EXPORTS.get(bytes(desc["handle"]))
    if base is not None:  # exported by this process: use the pointer directly
        return PeerBuffer(desc["key"], base + int(desc["offset"]), desc["nbytes"], desc["device"],
                          desc["owner_rank"], desc["kind"], mapped=False)
    ptr = native().ipc_open(desc["handle"], int(desc["offset"]))
    return PeerBuffer(desc["key"], ptr, desc["nbytes"], desc["device"], desc["owner_rank"], desc["kind"])


def lookup(off, key: str, wait_ms: int = 30000) -> PeerBuffer:
    """Wait up to ``wait_ms`` for ``key`` to be published, then map it."""
    found, body, _fd = off._agent.lookup_peer_buffer(key, int(wait_ms))
    if not found:
        raise TimeoutError(f"peer buffer {key!r} not published within {wait_ms} ms")
    return open_desc(_wire.decode("PeerBufferDesc", body))


def can_access_peer(device: int, peer: int) -> bool:
    return bool(native().can_access_peer(int(device), int(peer)))
