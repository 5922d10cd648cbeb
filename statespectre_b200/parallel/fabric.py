"""Intra-node GPU fabric: device buffers shared between rank processes.

A rank exports the allocation behind a tensor as a CUDA IPC handle, or a
buffer from the CUDA virtual memory API (:class:`DeviceBuffer`) as a POSIX
fd, and publishes it under a string key through offloadd's peer-buffer broker
(``PublishPeerBuffer`` / ``LookupPeerBuffer``, fds passed with SCM_RIGHTS);
another rank on the same node looks the key up and maps the buffer into its
own address space. VMM buffers can also join an NVLS multicast team
(:class:`MulticastTeam`), so one store by a trainer GPU reaches several
rollout GPUs through the NVSwitch. Mapped peer pointers and team pointers are
only ever handed to this package's kernels (K3 verify loads, K4 weight-sync
stores); they are deliberately not wrapped as torch tensors, so no library
kernel is ever given another GPU's memory as an operand.

StateSpectre has no GPU-to-GPU path: replicas and rollout engines only meet
through host memory and TCP (reference: src/daemon/canonical_rollout.cpp:240-411).
"""

from __future__ import annotations

import os
import struct
from typing import Dict, Optional, Sequence

import torch

from .. import _wire
from .._native import native

KIND_RAW = 0
KIND_WEIGHTS = 1  # a rollout weight buffer laid out by parallel.weight_sync.WeightLayout
KIND_REPLICA = 2  # a DP replica's parameter for P2P hash verification
KIND_TEAM = 3     # a multicast team object (fd) and its member count / size
KIND_SIGNAL = 4   # a rendezvous marker of the team protocol (no buffer)

# `handle` of a VMM-shared buffer: magic + allocation size (the fd travels
# beside the description); CUDA IPC handles are 64 bytes.
_VMM_MAGIC = b"VMM1"


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
    possible (CUDA IPC enables it lazily; a VMM import is mapped with access
    for this device); ``close()`` drops the mapping (IPC mappings are shared
    per allocation and refcounted)."""

    def __init__(self, key: str, ptr: int, nbytes: int, device: int, owner_rank: int, kind: int,
                 mapped: bool = True, vmm=None, desc: Optional[dict] = None):
        self.key, self.ptr, self.nbytes = key, int(ptr), int(nbytes)
        self.device, self.owner_rank, self.kind = int(device), int(owner_rank), int(kind)
        self.desc = desc
        self._mapped = mapped
        self._vmm = vmm
        self._open = True

    @property
    def is_vmm(self) -> bool:
        return self.desc is not None and is_vmm_desc(self.desc)

    def close(self) -> None:
        if self._open:
            if self._vmm is not None:
                native().vmm_free(self._vmm)
                self._vmm = None
            elif self._mapped:
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


def is_vmm_desc(desc: dict) -> bool:
    return bytes(desc["handle"])[:4] == _VMM_MAGIC


def open_desc(desc: dict, fd: int = -1) -> PeerBuffer:
    """Map a published buffer description (from ``lookup`` or an out-of-band
    exchange). VMM-shared buffers need the fd that came with it (not closed)."""
    if is_vmm_desc(desc):
        local = _LOCAL_VMM.get(desc["key"])
        if local is not None:  # published by this process
            return PeerBuffer(desc["key"], local.ptr, desc["nbytes"], desc["device"], desc["owner_rank"],
                              desc["kind"], mapped=False, desc=desc)
        if fd < 0:
            raise ValueError(f"{desc['key']!r}: a VMM buffer needs its fd")
        (size,) = struct.unpack_from("<Q", bytes(desc["handle"]), 4)
        v = native().vmm_import(fd, size, int(desc["device"]), torch.cuda.current_device())
        return PeerBuffer(desc["key"], v.ptr, desc["nbytes"], desc["device"], desc["owner_rank"], desc["kind"],
                          vmm=v, desc=desc)
    base = _LOCAL_EXPORTS.get(bytes(desc["handle"]))
    if base is not None:  # exported by this process: use the pointer directly
        return PeerBuffer(desc["key"], base + int(desc["offset"]), desc["nbytes"], desc["device"],
                          desc["owner_rank"], desc["kind"], mapped=False, desc=desc)
    ptr = native().ipc_open(desc["handle"], int(desc["offset"]))
    return PeerBuffer(desc["key"], ptr, desc["nbytes"], desc["device"], desc["owner_rank"], desc["kind"], desc=desc)


def lookup_desc(off, key: str, wait_ms: int = 30000):
    """(description, fd or -1) of a published key, waiting up to ``wait_ms``.
    The caller owns the fd."""
    found, body, fd = off._agent.lookup_peer_buffer(key, int(wait_ms))
    if not found:
        raise TimeoutError(f"peer buffer {key!r} not published within {wait_ms} ms")
    return _wire.decode("PeerBufferDesc", body), int(fd)


def lookup(off, key: str, wait_ms: int = 30000) -> PeerBuffer:
    """Wait up to ``wait_ms`` for ``key`` to be published, then map it."""
    desc, fd = lookup_desc(off, key, wait_ms)
    try:
        return open_desc(desc, fd)
    finally:
        if fd >= 0:
            os.close(fd)


def signal(off, key: str, note: bytes = b"") -> None:
    """Publish a rendezvous marker (no buffer); ``note`` rides in the handle."""
    desc = {"key": key, "owner_rank": int(off.rank), "device": 0, "kind": KIND_SIGNAL, "nbytes": 0,
            "offset": 0, "handle": bytes(note)}
    ok, msg = off._agent.publish_peer_buffer(_wire.encode("PeerBufferDesc", desc), -1)
    if not ok:
        raise RuntimeError(f"publish({key!r}) failed: {msg}")


def wait_signal(off, key: str, wait_ms: int = 30000) -> bytes:
    desc, fd = lookup_desc(off, key, wait_ms)
    if fd >= 0:
        os.close(fd)
    return bytes(desc["handle"])


# ---------------------------------------------------------------------------
# VMM buffers and multicast teams
# ---------------------------------------------------------------------------

class _ArrayView:
    """``__cuda_array_interface__`` over a raw device range; a tensor made
    from it holds a reference to the owner of the memory."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": (int(nbytes),), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 2}


class DeviceBuffer:
    """Device memory from the CUDA virtual memory API (``cuMemCreate``),
    shareable with other processes as an fd and bindable to a multicast
    team. ``tensor`` is a uint8 view of the first ``nbytes`` (it keeps the
    buffer alive; ``close()`` frees the memory explicitly)."""

    def __init__(self, nbytes: int, device=None, align_to: int = 0):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.nbytes = int(nbytes)
        self._v = native().vmm_alloc(dev.index, self.nbytes, int(align_to))
        self.tensor = torch.as_tensor(_ArrayView(self._v.ptr, self.nbytes, self), device=dev)

    @property
    def ptr(self) -> int:
        return int(self._v.ptr)

    @property
    def size(self) -> int:
        """Allocated bytes (``nbytes`` rounded up to the granularity)."""
        return int(self._v.size)

    @property
    def vmm(self):
        return self._v

    def export_fd(self) -> int:
        return int(native().vmm_export(self._v))

    def close(self) -> None:
        if self._v is not None:
            self.tensor = None
            native().vmm_free(self._v)
            self._v = None


# VMM buffers published by this process, by key (lookups of them resolve here)
_LOCAL_VMM: Dict[str, DeviceBuffer] = {}


def vmm_available(device: int) -> bool:
    try:
        native().vmm_granularity(int(device), False, 1)
        return True
    except RuntimeError:
        return False


def multicast_supported(device: int) -> bool:
    return bool(native().multicast_supported(int(device)))


def team_granularity(device: int, ndevices: int = 8) -> int:
    """Size multiple that lets a buffer on ``device`` join a multicast team."""
    return int(native().vmm_granularity(int(device), True, int(ndevices)))


def publish_vmm(off, key: str, buf: DeviceBuffer, kind: int = KIND_RAW) -> dict:
    """Publish a VMM buffer under ``key`` (its fd travels to the daemon)."""
    desc = {"key": key, "owner_rank": int(off.rank), "device": int(buf.device.index), "kind": int(kind),
            "nbytes": int(buf.nbytes), "offset": 0, "handle": _VMM_MAGIC + struct.pack("<Q", buf.size)}
    fd = buf.export_fd()
    try:
        ok, msg = off._agent.publish_peer_buffer(_wire.encode("PeerBufferDesc", desc), fd)
    finally:
        os.close(fd)
    if not ok:
        raise RuntimeError(f"publish_peer_buffer({key!r}) failed: {msg}")
    _LOCAL_VMM[key] = buf
    return desc


class MulticastTeam:
    """An NVLS multicast team over a trainer GPU and the rollout buffers it
    feeds: one ``multimem.st`` by the trainer writes every member's buffer.

    Every team device (two or more) binds one buffer of ``size`` bytes: the
    members bind their rollout buffers; the trainer's GPU binds a member's
    buffer when one lives on it, else a scratch buffer. Members in other
    processes join through the daemon's broker (``RolloutWeights.connect``):

      trainer: create, publish ``mcteam/<name>`` (fd), add its device, invite
               each member (``wsync/invite/<member key>``)
      member:  import, add its device, signal ``.../added/<key>``
      trainer: bind, signal ``.../bind``
      member:  bind, signal ``.../bound/<key>``
      trainer: map the team for its device (the pointer the kernel stores to)

    and tear down the other way round: ``close()`` signals ``.../closed``,
    members unbind only after it (a member must not leave while the trainer
    may still store)."""

    def __init__(self, off, name: str, members: Sequence[dict], device: int, size: int, wait_ms: int = 60000):
        """``members``: one dict per rollout buffer with its ``key``,
        ``device`` and ``nbytes_alloc`` (see ``member_of``)."""
        C = native()
        self.off, self.name, self.device = off, name, int(device)
        self.members = list(members)
        devices = {self.device} | {int(m["device"]) for m in self.members}
        if len(devices) != len(self.members) + (0 if any(int(m["device"]) == self.device
                                                         for m in self.members) else 1):
            raise ValueError("multicast team: two members on one GPU")
        self.ndevices = len(devices)
        if self.ndevices < 2:  # the driver rejects one-device teams
            raise ValueError("a multicast team needs two or more GPUs")
        self.team = C.team_create(self.ndevices, int(size))
        self.size = int(self.team.size)
        self.scratch: Optional[DeviceBuffer] = None
        self.ptr = 0
        self._closed = False
        local = [m for m in self.members if m["key"] in _LOCAL_VMM]
        remote = [m for m in self.members if m["key"] not in _LOCAL_VMM]
        for m in self.members:
            if int(m["nbytes_alloc"]) < self.size:
                raise ValueError(f"{m['key']!r}: buffer of {m['nbytes_alloc']} bytes cannot bind "
                                 f"{self.size} bytes")
        fd = C.team_export(self.team)
        try:
            desc = {"key": f"mcteam/{name}", "owner_rank": int(off.rank), "device": self.device,
                    "kind": KIND_TEAM, "nbytes": self.size, "offset": self.ndevices, "handle": b""}
            ok, msg = off._agent.publish_peer_buffer(_wire.encode("PeerBufferDesc", desc), fd)
        finally:
            os.close(fd)
        if not ok:
            raise RuntimeError(f"publish(mcteam/{name}) failed: {msg}")
        for d in devices:
            if d == self.device or any(int(m["device"]) == d for m in local):
                C.team_add_device(self.team, d)
        for m in remote:
            signal(off, f"wsync/invite/{m['key']}", b"mc:" + name.encode())
        for m in remote:
            wait_signal(off, f"mcteam/{name}/added/{m['key']}", wait_ms)
        mine = [m for m in local if int(m["device"]) == self.device]
        if not mine:
            self.scratch = DeviceBuffer(self.size, torch.device("cuda", self.device),
                                        team_granularity(self.device, self.ndevices))
            C.team_bind(self.team, self.scratch.vmm)
        for m in local:
            C.team_bind(self.team, _LOCAL_VMM[m["key"]].vmm)
        signal(off, f"mcteam/{name}/bind")
        for m in remote:
            wait_signal(off, f"mcteam/{name}/bound/{m['key']}", wait_ms)
        self.ptr = int(C.team_map(self.team, self.device))

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        C = native()
        torch.cuda.synchronize(self.device)
        try:
            signal(self.off, f"mcteam/{self.name}/closed")
        except Exception:  # the session may already be gone; members time out
            pass
        for d in sorted({self.device} | {int(m["device"]) for m in self.members if m["key"] in _LOCAL_VMM}):
            C.team_unbind(self.team, d)
        C.team_release(self.team)
        if self.scratch is not None:
            self.scratch.close()
            self.scratch = None


def member_of(desc: dict) -> dict:
    """Team member record of a published VMM buffer description."""
    (size,) = struct.unpack_from("<Q", bytes(desc["handle"]), 4)
    return {"key": desc["key"], "device": int(desc["device"]), "nbytes_alloc": int(size)}


class TeamMembership:
    """A rollout buffer's side of a multicast team (made by ``join``)."""

    def __init__(self, off, name: str, team, device: int):
        self.off, self.name, self.team, self.device = off, name, team, int(device)
        self._closed = False

    def close(self, wait_ms: int = 60000) -> None:
        """Leave the team once its trainer has closed it (bounded wait)."""
        if self._closed:
            return
        self._closed = True
        try:
            wait_signal(self.off, f"mcteam/{self.name}/closed", wait_ms)
        except (TimeoutError, RuntimeError):
            pass
        C = native()
        C.team_unbind(self.team, self.device)
        C.team_release(self.team)


def join(off, key: str, buf: DeviceBuffer, wait_ms: int = 60000) -> Optional[TeamMembership]:
    """Member side of the team protocol for the buffer published as ``key``:
    waits for the trainer's invitation; returns None when the trainer pushes
    point to point instead."""
    note = wait_signal(off, f"wsync/invite/{key}", wait_ms)
    if not note.startswith(b"mc:"):
        return None
    name = note[3:].decode()
    desc, fd = lookup_desc(off, f"mcteam/{name}", wait_ms)
    try:
        team = native().team_import(fd, int(desc["offset"]), int(desc["nbytes"]))
    finally:
        if fd >= 0:
            os.close(fd)
    C = native()
    dev = int(buf.device.index)
    C.team_add_device(team, dev)
    signal(off, f"mcteam/{name}/added/{key}")
    wait_signal(off, f"mcteam/{name}/bind", wait_ms)
    C.team_bind(team, buf.vmm)
    signal(off, f"mcteam/{name}/bound/{key}")
    return TeamMembership(off, name, team, dev)


def can_access_peer(device: int, peer: int) -> bool:
    return bool(native().can_access_peer(int(device), int(peer)))
