"""In-box RL weight sync: trainer GPUs push sealed versions into rollout GPUs.

StateSpectre syncs a rollout engine by sealing a version in offloadd (every
object copied device -> pinned host first), after which the rollout pulls each
changed object over TCP and copies it host -> device (reference:
python_api/state_spectre/_rollout.py:101-175, src/daemon/canonical_rollout.cpp:240-411).
On one B200 node the rollout GPUs are NVLink peers of the trainer GPUs, so the
bytes take one hop instead:

* the rollout allocates ONE receive buffer for all its parameters, laid out by
  :class:`WeightLayout` (bf16 as trained, or fp8 e4m3 + fp32 1x128 block
  scales for 2-D weights), and publishes it under a key through the daemon's
  peer-buffer broker (:mod:`.fabric`);
* the trainer maps it and runs the K4 push kernel: every parameter is read
  from HBM once, hashed per 64 KiB chunk (ssh128), and only chunks whose digest
  differs from what the rollout already holds cross NVLink, quantized on the
  fly in fp8 mode; the same pass yields every parameter's 128-bit content hash;
* the version is then made durable in offloadd without re-copying unchanged
  parameters: changed ones go through one ``canonical_evict_batch`` (K1, D2H
  + hash, zbf16-coded over PCIe; every round trip and copy issued before the
  first copy is awaited), unchanged ones are carried forward (objects that share the previous
  version's storage), then the version is sealed and promoted. Manifests are
  the same as StateSpectre's, so cross-node rollouts pull as before.
"""

from __future__ import annotations

import math
import os
import struct
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .._native import native
from . import fabric

ALIGN = 256
CHUNK = 64 * 1024
_ITEM = struct.Struct("<QQQQQIIQQ")  # PushItem: src, dst, dst_scales, nbytes, chunk_begin, mode, flags, digest_base, -
PUSH_RAW, PUSH_FP8, PUSH_HASH = 0, 1, 2
PUSH_DELTA, PUSH_MULTICAST = 1, 2
TRANSPORTS = ("auto", "p2p", "multicast")


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class LayoutEntry:
    name: str
    shape: Tuple[int, ...]
    dtype: torch.dtype
    nbytes: int          # source (trainer) bytes
    quant: bool          # stored as fp8 e4m3 + scales on the rollout
    dst_offset: int
    dst_nbytes: int
    scale_offset: int = 0
    nscales: int = 0


class WeightLayout:
    """Deterministic placement of a parameter list in one rollout buffer.

    Trainer and rollout build it from the same (name, shape, dtype) list, so
    no offsets travel; ``fingerprint`` lets both sides check they agree."""

    def __init__(self, specs: Sequence[Tuple[str, Sequence[int], torch.dtype]], mode: str = "bf16"):
        if mode not in ("bf16", "fp8"):
            raise ValueError("mode must be 'bf16' or 'fp8'")
        self.mode = mode
        self.entries: List[LayoutEntry] = []
        off = 0
        for name, shape, dtype in specs:
            shape = tuple(int(s) for s in shape)
            nel = math.prod(shape)
            esz = torch.empty((), dtype=dtype).element_size()
            nbytes = nel * esz
            if nbytes % 16:
                raise ValueError(f"{name}: {nbytes} bytes is not a multiple of 16")
            quant = mode == "fp8" and dtype == torch.bfloat16 and len(shape) >= 2 and nel % 128 == 0
            e = LayoutEntry(name, shape, dtype, nbytes, quant, off, nel if quant else nbytes)
            off = _align(off + e.dst_nbytes)
            if quant:
                e.scale_offset, e.nscales = off, nel // 128
                off = _align(off + 4 * e.nscales)
            self.entries.append(e)
        self.total_bytes = max(off, ALIGN)
        self.by_name = {e.name: e for e in self.entries}
        h = 1469598103934665603
        for e in self.entries:
            for b in f"{e.name}|{e.shape}|{e.dtype}|{int(e.quant)};".encode():
                h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        self.fingerprint = h

    @classmethod
    def from_params(cls, params: Dict[str, torch.Tensor], mode: str = "bf16") -> "WeightLayout":
        return cls([(n, tuple(t.shape), t.dtype) for n, t in params.items()], mode)

    @property
    def total_chunks(self) -> int:
        return sum((e.nbytes + CHUNK - 1) // CHUNK for e in self.entries)


class RolloutWeights:
    """Rollout-side receive buffer holding every parameter of a layout.

    The buffer comes from the CUDA virtual memory API when the driver offers
    it (shareable as an fd, sized to join a multicast team), else from
    torch's allocator (shared through CUDA IPC, point-to-point only)."""

    def __init__(self, layout: WeightLayout, device=None, vmm: Optional[bool] = None):
        self.layout = layout
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.key: Optional[str] = None
        self.dbuf: Optional[fabric.DeviceBuffer] = None
        self.membership = None
        self.transport: Optional[str] = None
        if vmm is None:
            vmm = fabric.vmm_available(self.device.index)
        if vmm:
            align = fabric.team_granularity(self.device.index) if fabric.multicast_supported(self.device.index) else 0
            self.dbuf = fabric.DeviceBuffer(layout.total_bytes, self.device, align)
            self.buf = self.dbuf.tensor
            self.buf.zero_()
        else:
            self.buf = torch.zeros(layout.total_bytes, dtype=torch.uint8, device=self.device)

    def publish(self, off, key: str) -> dict:
        """Make the buffer reachable by trainer ranks as ``key``."""
        self.key = key
        if self.dbuf is not None:
            return fabric.publish_vmm(off, key, self.dbuf, kind=fabric.KIND_WEIGHTS)
        return fabric.publish(off, key, self.buf, kind=fabric.KIND_WEIGHTS)

    def connect(self, off, wait_ms: int = 60000) -> str:
        """Wait for the trainer that feeds this buffer (in another process)
        and join its multicast team when it builds one. Returns the
        transport, "multicast" or "p2p"."""
        if self.key is None:
            raise RuntimeError("publish() the buffer first")
        if self.dbuf is None:
            fabric.wait_signal(off, f"wsync/invite/{self.key}", wait_ms)
            self.transport = "p2p"
        else:
            self.membership = fabric.join(off, self.key, self.dbuf, wait_ms)
            self.transport = "multicast" if self.membership is not None else "p2p"
        return self.transport

    def close(self, wait_ms: int = 60000) -> None:
        """Leave the multicast team (after its trainer closed it) and free
        the buffer; views returned by ``get`` must not be used afterwards."""
        if self.membership is not None:
            self.membership.close(wait_ms)
            self.membership = None
        if self.dbuf is not None:
            if self.key is not None:
                fabric._LOCAL_VMM.pop(self.key, None)
            self.buf = None
            self.dbuf.close()
            self.dbuf = None

    def get(self, name: str):
        """bf16 view of a parameter, or (fp8 e4m3 view, fp32 scales) when quantized."""
        e = self.layout.by_name[name]
        raw = self.buf[e.dst_offset:e.dst_offset + e.dst_nbytes]
        if not e.quant:
            return raw.view(e.dtype).view(e.shape)
        q = raw.view(torch.float8_e4m3fn).view(e.shape)
        sc = self.buf[e.scale_offset:e.scale_offset + 4 * e.nscales].view(torch.float32)
        return q, sc

    def dequantized(self, name: str) -> torch.Tensor:
        """A parameter as bf16 (fp8 entries rescaled block by block)."""
        v = self.get(name)
        if not isinstance(v, tuple):
            return v
        q, sc = v
        return (q.float().view(-1, 128) * sc.view(-1, 1)).view(q.shape).to(torch.bfloat16)

    def content_hashes(self, names: Optional[Sequence[str]] = None, stream=None) -> Dict[str, Tuple[int, int]]:
        """ssh128 of the received bytes of bf16 entries (equal to the trainer's
        manifest content hash when the push was byte-exact). One hash-only K4
        launch over every selected entry plus the item-hash fold."""
        ents = [e for e in self.layout.entries if not e.quant and (names is None or e.name in names)]
        if not ents:
            return {}
        key = tuple(e.name for e in ents)
        if getattr(self, "_hash_key", None) != key:
            buf = bytearray()
            chunk = 0
            for e in ents:
                buf += _ITEM.pack(self.buf.data_ptr() + e.dst_offset, 0, 0, e.nbytes, chunk, PUSH_HASH, 0, chunk, 0)
                chunk += (e.nbytes + CHUNK - 1) // CHUNK
            self._hash_items = torch.frombuffer(buf, dtype=torch.uint8).to(self.device)
            self._hash_dig = torch.empty(chunk, dtype=torch.int64, device=self.device)
            self._hash_out = torch.empty(2 * len(ents), dtype=torch.int64, device=self.device)
            self._hash_err = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._hash_chunks = chunk
            self._hash_key = key
        s = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            native().k_push(self._hash_items.data_ptr(), len(ents), self._hash_chunks, self._hash_dig.data_ptr(),
                            self._hash_out.data_ptr(), 0, self._hash_err.data_ptr(), s.cuda_stream, 0, 0)
        s.synchronize()
        if int(self._hash_err.item()):
            raise RuntimeError(f"hash pass failed with device status {int(self._hash_err.item())}")
        h = self._hash_out.view(-1, 2).tolist()
        m = 2**64 - 1
        return {e.name: (h[i][0] & m, h[i][1] & m) for i, e in enumerate(ents)}


class WeightPusher:
    """Trainer-side K4 launcher for one destination buffer.

    ``digests`` records, per 64 KiB chunk, the digest of what the destination
    holds, so each push (``delta=True``) only moves chunks that changed since
    the previous push to the same destination. A 64-bit chunk digest decides
    the skip; ``invalidate()`` forces the next push to send everything."""

    def __init__(self, params: Dict[str, torch.Tensor], layout: WeightLayout, dst_ptr: int, device=None,
                 delta: bool = True, ctas: int = 0, multicast: bool = False):
        self.params = params
        self.layout = layout
        self.dst_ptr = int(dst_ptr)
        self.delta = delta
        self.ctas = ctas
        self.multicast = multicast  # dst_ptr is a multicast team mapping
        first = next(iter(params.values()))
        self.device = torch.device(device) if device is not None else first.device
        n = len(layout.entries)
        if [e.name for e in layout.entries] != list(params):
            raise ValueError("params and layout disagree on names / order")
        if self.dst_ptr % 16:
            raise ValueError("destination buffer must be 16-byte aligned")
        self.total_chunks = layout.total_chunks
        self.digests = torch.zeros(max(1, self.total_chunks), dtype=torch.int64, device=self.device)
        self.item_hash = torch.zeros(2 * n, dtype=torch.int64, device=self.device)
        self.stats = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ptrs: List[int] = []
        self.items = None
        self._build_items()

    def _table(self, entries) -> Tuple[torch.Tensor, int, List[int]]:
        """Work table for `entries` (layout order): compact work-chunk
        indices, digest-table indices of the full layout."""
        buf = bytearray()
        work = 0
        ptrs = []
        for e in entries:
            t = self.params[e.name]
            if not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"{e.name}: push sources must be contiguous tensors on {self.device}")
            if t.numel() * t.element_size() != e.nbytes:
                raise ValueError(f"{e.name}: size differs from the layout")
            p = t.data_ptr()
            if p % 16:
                raise ValueError(f"{e.name}: source must be 16-byte aligned")
            ptrs.append(p)
            mode = PUSH_FP8 if e.quant else PUSH_RAW
            scales = self.dst_ptr + e.scale_offset if e.quant else 0
            flags = (PUSH_DELTA if self.delta else 0) | (PUSH_MULTICAST if self.multicast else 0)
            buf += _ITEM.pack(p, self.dst_ptr + e.dst_offset, scales, e.nbytes, work, mode, flags,
                              self._digest_base[e.name], 0)
            work += (e.nbytes + CHUNK - 1) // CHUNK
        host = torch.frombuffer(buf, dtype=torch.uint8) if buf else torch.zeros(64, dtype=torch.uint8)
        return host.to(self.device), work, ptrs

    def _build_items(self) -> None:
        self._digest_base = {}
        chunk = 0
        for e in self.layout.entries:
            self._digest_base[e.name] = chunk
            chunk += (e.nbytes + CHUNK - 1) // CHUNK
        self.items, _, self._ptrs = self._table(self.layout.entries)
        self._subsets: Dict[tuple, tuple] = {}
        self._row = {e.name: i for i, e in enumerate(self.layout.entries)}

    def refresh(self) -> None:
        """Rebuild the work list if any parameter was reallocated."""
        if [self.params[e.name].data_ptr() for e in self.layout.entries] != self._ptrs:
            self._build_items()

    def invalidate(self) -> None:
        self.digests.zero_()

    def push(self, stream=None, names: Optional[Sequence[str]] = None) -> None:
        """Enqueue the push on ``stream`` (default: current stream).

        ``names`` restricts the launch to those parameters (the caller knows
        the others did not change); their hashes land in the rows of
        ``item_hash`` that the full layout gives them."""
        s = stream or torch.cuda.current_stream(self.device)
        C = native()
        flags = PUSH_DELTA if self.delta else 0
        if names is None:
            C.k_push(self.items.data_ptr(), len(self.layout.entries), self.total_chunks, self.digests.data_ptr(),
                     self.item_hash.data_ptr(), self.stats.data_ptr(), self.err.data_ptr(), s.cuda_stream,
                     self.ctas, flags)
            return
        want = set(names)
        ents = [e for e in self.layout.entries if e.name in want]
        if not ents:
            return
        key = tuple(e.name for e in ents)
        sub = self._subsets.get(key)
        if sub is None or sub[3] != [self.params[n].data_ptr() for n in key]:
            items, work, ptrs = self._table(ents)
            rows = torch.tensor([self._row[n] for n in key], dtype=torch.int64, device=self.device)
            out = torch.zeros(2 * len(ents), dtype=torch.int64, device=self.device)
            if len(self._subsets) > 64:
                self._subsets.clear()
            sub = self._subsets[key] = (items, work, out, ptrs, rows)
        items, work, out, _, rows = sub
        C.k_push(items.data_ptr(), len(ents), work, self.digests.data_ptr(), out.data_ptr(), self.stats.data_ptr(),
                 self.err.data_ptr(), s.cuda_stream, self.ctas, flags)
        with torch.cuda.stream(s):
            self.item_hash.view(-1, 2).index_copy_(0, rows, out.view(-1, 2))

    def result(self) -> dict:
        """Totals since construction (synchronizes the device)."""
        st = self.stats.tolist()
        return {"chunks_stored": st[0], "bytes_stored": st[1], "error": int(self.err.item())}

    def hashes(self) -> Dict[str, Tuple[int, int]]:
        h = self.item_hash.view(-1, 2).tolist()
        m = 2**64 - 1
        return {e.name: (h[i][0] & m, h[i][1] & m) for i, e in enumerate(self.layout.entries)}


class TrainerWeightSync:
    """Trainer side of in-box weight sync for one TP/PP shard.

    ``publish_version(v)`` pushes the changed chunks of ``params`` into every
    rollout buffer in ``rollout_keys`` (the replicas of this shard), then,
    with ``persist=True``, records version ``v`` in offloadd: changed
    parameters are copied (K1) as new canonical objects, unchanged ones are
    carried forward from ``v - 1``, and the version is sealed and promoted.

    ``transport``: "multicast" builds an NVLS multicast team over this GPU
    and every rollout buffer, so one K4 launch with ``multimem.st`` stores
    feeds all replicas through the NVSwitch; "p2p" maps each buffer and runs
    one K4 launch per replica with plain stores over NVLink; "auto" takes
    multicast for two or more replicas when every buffer is VMM-shared on its
    own GPU and the GPUs support it, else p2p. Rollout ranks in other
    processes call ``RolloutWeights.connect`` to take part.

    Several trainer ranks sharing one version (TP / PP shards of one model)
    pass ``seal_barrier`` (a callable every one of them calls after recording
    its shard) and ``sealer=True`` on exactly one of them.
    """

    def __init__(self, off, params: Dict[str, torch.Tensor], rollout_keys: Sequence[str], mode: str = "bf16",
                 model_role="policy_rollout", persist: bool = True, tp_rank: int = 0, pp_rank: int = 0,
                 lookup_wait_ms: int = 60000, ctas: int = 0, transport: Optional[str] = None,
                 seal_barrier=None, sealer: bool = True):
        from ..api import ModelRole
        if transport is None:  # the daemon config's nvlink.weight_sync, else auto
            transport = getattr(off, "nvlink_options", {}).get("weight_sync", "auto")
        if transport not in TRANSPORTS:
            raise ValueError(f"transport must be one of {TRANSPORTS}")
        self.off = off
        self.params = dict(params)
        self.layout = WeightLayout.from_params(self.params, mode)
        self.role = ModelRole.parse(model_role)
        self.persist = persist
        self.tp_rank, self.pp_rank = tp_rank, pp_rank
        first = next(iter(self.params.values()))
        self.device = first.device
        self.team: Optional[fabric.MulticastTeam] = None
        self.peers = []
        found = [fabric.lookup_desc(off, k, lookup_wait_ms) for k in rollout_keys]
        try:
            for desc, _ in found:
                if desc["nbytes"] < self.layout.total_bytes:
                    raise ValueError(f"rollout buffer {desc['key']!r} holds {desc['nbytes']} bytes, layout needs "
                                     f"{self.layout.total_bytes}")
            self.transport = self._choose(transport, [d for d, _ in found])
            if self.transport == "multicast":
                members = [fabric.member_of(d) for d, _ in found]
                self.team = fabric.MulticastTeam(off, f"{rollout_keys[0]}#{off.rank}", members, self.device.index,
                                                 self.layout.total_bytes, lookup_wait_ms)
                self.pushers = [WeightPusher(self.params, self.layout, self.team.ptr, self.device, ctas=ctas,
                                             multicast=True)]
            else:
                self.peers = [fabric.open_desc(d, fd) for d, fd in found]
                for d, _ in found:
                    if d["key"] not in fabric._LOCAL_VMM:
                        fabric.signal(off, f"wsync/invite/{d['key']}", b"p2p")
                self.pushers = [WeightPusher(self.params, self.layout, p.ptr, self.device, ctas=ctas)
                                for p in self.peers]
        finally:
            for _, fd in found:
                if fd >= 0:
                    os.close(fd)
        self.stream = torch.cuda.Stream(self.device)
        self.last_hash: Dict[str, Tuple[int, int]] = {}
        self.last_version: Optional[int] = None
        self._pids: Dict[str, int] = {}
        self._pending = None  # (version, changed names, hashes) between push_version and seal_version
        self.seal_barrier = seal_barrier
        self.sealer = sealer

    def _choose(self, transport: str, descs) -> str:
        if transport == "p2p":
            return "p2p"
        dev = self.device.index
        devices = [int(d["device"]) for d in descs]
        ok = (all(fabric.is_vmm_desc(d) for d in descs) and len(set(devices)) == len(devices)
              and len(set(devices) | {dev}) >= 2
              and all(fabric.multicast_supported(x) for x in set(devices) | {dev}))
        if transport == "multicast":
            if not ok:
                raise RuntimeError("multicast transport needs VMM-shared rollout buffers on distinct GPUs "
                                   "(two or more GPUs in all) with switch multicast support")
            return "multicast"
        return "multicast" if ok and len(descs) >= 2 else "p2p"

    def _key(self, name: str, version: int):
        k = self.off.canonical_key(model_role=self.role, model_version=version, param_name=name,
                                   tensor=self.params[name], tp_rank=self.tp_rank, pp_rank=self.pp_rank)
        self._pids[name] = k.param_id
        return k

    def push(self, names: Optional[Sequence[str]] = None) -> Tuple[torch.cuda.Event, torch.cuda.Event]:
        """Enqueue the pushes after the work already on the current stream."""
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for p in self.pushers:
            p.refresh()
            p.push(self.stream, names)
        e1.record(self.stream)
        return e0, e1

    def publish_version(self, version: int, changed: Optional[Sequence[str]] = None) -> dict:
        """Push and (with ``persist``) seal version ``version``: ``push_version``
        followed by ``seal_version``.

        Without ``changed`` every parameter is hashed on the device and the
        changed set is found by comparing content hashes with the previous
        version (the manifest diff). With ``changed`` (names the caller
        updated) only those parameters are hashed and pushed; the others keep
        their previous hashes. The first version always covers everything."""
        out = self.push_version(version, changed)
        out.update(self.seal_version())
        return out

    def push_version(self, version: int, changed: Optional[Sequence[str]] = None) -> dict:
        """The NVLink half of ``publish_version``: push the changed chunks into
        every rollout buffer and find the changed parameters. When it returns
        the rollout holds version ``version``; ``seal_version`` records it in
        offloadd and may run while the rollout checks what it received."""
        if self._pending is not None:
            raise RuntimeError(f"version {self._pending[0]} was pushed but not sealed")
        t0 = time.perf_counter()
        hint = None if (changed is None or self.last_version is None) else list(changed)
        e0, e1 = self.push(hint)
        e1.synchronize()
        push_ms = e0.elapsed_time(e1)
        res = self.pushers[0].result() if self.pushers else {"error": 0}
        if res["error"]:
            raise RuntimeError(f"weight push failed with device status {res['error']}")
        hashes = self.pushers[0].hashes() if self.pushers else {}
        names = [n for n in self.params if self.last_hash.get(n) != hashes.get(n)]
        self._pending = (version, names, hashes)
        return {"version": version, "changed": len(names), "push_ms": push_ms,
                "push_wall_ms": (time.perf_counter() - t0) * 1e3}

    def seal_version(self) -> dict:
        """Record the pushed version in offloadd (``persist``): changed
        parameters are copied to the host as new canonical objects, this
        shard's unchanged ones are carried forward from the previous version,
        and the version is sealed and promoted. With several trainer ranks per
        version (``seal_barrier``), every rank records its shard first and the
        ``sealer`` rank then seals."""
        if self._pending is None:
            raise RuntimeError("seal_version without a pushed version")
        version, changed, hashes = self._pending
        t0 = time.perf_counter()
        out = {}
        if self.persist:
            carry = self.last_version is not None
            # one batch: every round trip and copy issued before the first is awaited
            self.off.canonical_evict_batch([(self.params[n], self._key(n, version))
                                            for n in (changed if carry else self.params)],
                                           destructive=False, stream=self.stream)
            if carry:
                unchanged = [self._pids[n] if n in self._pids else self._key(n, version).param_id
                             for n in self.params if n not in changed]
                if unchanged:
                    self.off.carry_forward_version(self.role, self.last_version, version, unchanged,
                                                   tp_rank=self.tp_rank, pp_rank=self.pp_rank)
            self.stream.synchronize()
            self.off._agent.synchronize()
            if self.seal_barrier is not None:
                self.seal_barrier()
            if self.sealer:
                self.off.promote_rollout_version(version) if self.role == 2 else \
                    self.off.seal_model_version(self.role, version)
            out["seal_wall_ms"] = (time.perf_counter() - t0) * 1e3
        self.last_hash = hashes
        self.last_version = version
        self._pending = None
        return out

    def close(self) -> None:
        """Release the mappings (and the multicast team: its members may
        leave after this)."""
        torch.cuda.synchronize(self.device)
        if self.team is not None:
            self.team.close()
            self.team = None
        for p in self.peers:
            p.close()
        self.peers = []
