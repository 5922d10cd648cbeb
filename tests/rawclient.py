"""A rank that speaks the wire protocol directly and never touches the arenas.

It drives the slot state machine (reserve, mark submitted/complete, prefetch,
release) without copying bytes, so daemon behaviour is testable on any host.
"""

import mmap
import os
import socket
import struct

from statespectre_b200 import _wire
from statespectre_b200._wire import Op

# Control-region offsets of the v1 ABI: ofld_slot_table_header_t keeps
# control_ring_offset at byte 72 and the ring geometry (max_ranks, stride,
# capacity) in its reserved bytes from 80; a ring header holds capacity,
# owner_rank and rank_epoch at 0/4/8, head at 64, tail at 128, and its 40-byte
# completion entries (lease, tensor, version, slot, event, timestamp) from 192.
_SLOTS_OFFSET_AT = 64
_RING_OFFSET_AT = 72
_GEOMETRY_AT = 80
_ENTRY = struct.Struct("<QQQIIQ")
# ofld_slot_entry_t: 256 bytes; arena_id at 16, arena_offset 24, nbytes 40,
# tensor_id 48, lease_id 64.
_SLOT_SIZE = 256


class RawRank:
    def __init__(self, sock_path: str, rank_id: int, pid: int | None = None, gpu: int = 0, numa: int = 0,
                 map_control: bool = False):
        self.conn = _wire.Connection(sock_path)
        self.rank_id = rank_id
        self.gpu = gpu
        self.numa = numa
        req = dict(rank_id=rank_id, local_rank=rank_id, world_rank=rank_id, gpu_id=gpu, numa_node=numa,
                   pid=pid if pid is not None else os.getpid() * 1000 + rank_id)
        self.control = None
        self.arenas = {}
        if map_control:
            r = self._register_with_fds(req)
        else:
            r = self.conn.call(Op.REGISTER_RANK, **req)
        assert r["ok"], r["message"]
        self.epoch = r["rank_epoch"]
        self.ring_index = r["ring_index"]
        self.num_slots = r["num_slots"]

    def _register_with_fds(self, req: dict) -> dict:
        """RegisterRank, keeping the descriptors that ride on the reply's frame
        header, and map the control region read-write as an agent does."""
        sock = self.conn.sock
        sock.sendall(_wire.make_frame(Op.REGISTER_RANK, _wire.encode("RegisterRankRequest", req)))
        head, fds, _, _ = socket.recv_fds(sock, _wire.FRAME_HEADER.size, 64)
        if len(head) < _wire.FRAME_HEADER.size:
            head += _wire.recv_exact(sock, _wire.FRAME_HEADER.size - len(head))
        _op, _flags, n = _wire.parse_frame_header(head)
        r = _wire.decode("RegisterRankResponse", _wire.recv_exact(sock, n))
        try:
            if r["ok"]:
                self.control = mmap.mmap(fds[r["control_fd_index"]], r["control_size"])
                for a in r["arenas"]:
                    self.arenas[a["arena_id"]] = mmap.mmap(fds[a["fd_index"]], a["size"])
        finally:
            for fd in fds:
                os.close(fd)
        return r

    # ---- direct writes into this rank's completion ring (needs map_control) ----
    def _ring(self) -> int:
        base = struct.unpack_from("<Q", self.control, _RING_OFFSET_AT)[0]
        _max_ranks, stride, _cap = struct.unpack_from("<III", self.control, _GEOMETRY_AT)
        return base + self.ring_index * stride

    def ring_capacity(self) -> int:
        return struct.unpack_from("<III", self.control, _GEOMETRY_AT)[2]

    def write_ring_header(self, owner_rank: int, rank_epoch: int, capacity: int) -> None:
        struct.pack_into("<IIQ", self.control, self._ring(), capacity, owner_rank, rank_epoch)

    def ring_head_tail(self) -> tuple:
        r = self._ring()
        return struct.unpack_from("<Q", self.control, r + 64)[0], struct.unpack_from("<Q", self.control, r + 128)[0]

    def ring_push(self, lease, tid, ver, slot, event=1) -> None:
        r = self._ring()
        _head, tail = self.ring_head_tail()
        at = r + 192 + (tail & (self.ring_capacity() - 1)) * _ENTRY.size
        _ENTRY.pack_into(self.control, at, lease, tid, ver, slot, event, 1)
        struct.pack_into("<Q", self.control, r + 128, tail + 1)

    def scribble_slot(self, slot: int, arena_id: int, arena_offset: int, nbytes: int) -> None:
        """Overwrite where a slot entry says its bytes are, as a faulty rank could."""
        at = struct.unpack_from("<Q", self.control, _SLOTS_OFFSET_AT)[0] + slot * _SLOT_SIZE
        struct.pack_into("<QQ", self.control, at + 16, arena_id, arena_offset)
        struct.pack_into("<Q", self.control, at + 40, nbytes)

    def slot_fields(self, slot: int) -> tuple:
        """(state, arena_id, arena_offset, nbytes, tensor_id) of a slot entry."""
        at = struct.unpack_from("<Q", self.control, _SLOTS_OFFSET_AT)[0] + slot * _SLOT_SIZE
        state = struct.unpack_from("<I", self.control, at)[0]
        arena_id, off = struct.unpack_from("<QQ", self.control, at + 16)
        return state, arena_id, off, struct.unpack_from("<Q", self.control, at + 40)[0], \
            struct.unpack_from("<Q", self.control, at + 48)[0]

    def write_arena(self, arena_id: int, offset: int, data: bytes) -> None:
        """Store bytes in a reserved run, as an agent's copy would (needs map_control)."""
        self.arenas[arena_id][offset:offset + len(data)] = data

    def set_ring_tail(self, tail: int) -> None:
        struct.pack_into("<Q", self.control, self._ring() + 128, tail)

    def call(self, op, **kw):
        return self.conn.call(op, **kw)

    def heartbeat(self, epoch=None):
        return self.call(Op.HEARTBEAT, rank_id=self.rank_id, rank_epoch=self.epoch if epoch is None else epoch,
                         timestamp_ns=1)

    def reserve(self, tid, ver, nbytes, flags=0, epoch=None):
        return self.call(Op.REQUEST_OFFLOAD, rank_id=self.rank_id, rank_epoch=self.epoch if epoch is None else epoch,
                         tensor_id=tid, version=ver, nbytes=nbytes, gpu_id=self.gpu, numa_node=self.numa,
                         alignment=256, flags=flags)

    def mark(self, op, lease, tid, ver, slot, epoch=None):
        return self.call(op, rank_id=self.rank_id, rank_epoch=self.epoch if epoch is None else epoch, lease_id=lease,
                         tensor_id=tid, version=ver, slot_id=slot, seq=1, timestamp_ns=1)

    def offload(self, tid, ver, nbytes):
        """Full D2H cycle without data: reserve, submitted, complete."""
        g = self.reserve(tid, ver, nbytes)
        assert g["ok"], g["message"]
        assert self.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], tid, ver, g["slot_id"])["ok"]
        c = self.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], tid, ver, g["slot_id"])
        assert c["ok"], c["message"]
        return g

    def prefetch(self, tid, ver=0, flags=0):
        return self.call(Op.REQUEST_PREFETCH, rank_id=self.rank_id, rank_epoch=self.epoch, tensor_id=tid,
                         version=ver, gpu_id=self.gpu, numa_node=self.numa, flags=flags)

    def h2d_complete(self, lease, tid, ver, slot, keep_pinned=False):
        return self.call(Op.MARK_H2D_COMPLETE, rank_id=self.rank_id, rank_epoch=self.epoch, lease_id=lease,
                         tensor_id=tid, version=ver, slot_id=slot, keep_pinned=keep_pinned, seq=1, timestamp_ns=1)

    def release(self, lease, slot=0):
        return self.call(Op.RELEASE_LEASE, rank_id=self.rank_id, rank_epoch=self.epoch, lease_id=lease,
                         slot_id=slot, reason="test")

    def location(self, tid, ver=0):
        return self.call(Op.QUERY_LOCATION, tensor_id=tid, version=ver)

    def stats(self):
        r = self.call(Op.GET_STATS, rank_id=0xFFFFFFFF)
        return {e["key"]: e["value"] for e in r["stats"]}

    def close(self):
        for m in self.arenas.values():
            m.close()
        if self.control is not None:
            self.control.close()
        self.conn.close()
