"""A rank that speaks the wire protocol directly and never touches the arenas.

It drives the slot state machine (reserve, mark submitted/complete, prefetch,
release) without copying bytes, so daemon behaviour is testable on any host.
"""

import os

from statespectre_b200 import _wire
from statespectre_b200._wire import Op


class RawRank:
    def __init__(self, sock_path: str, rank_id: int, pid: int | None = None, gpu: int = 0, numa: int = 0):
        self.conn = _wire.Connection(sock_path)
        self.rank_id = rank_id
        self.gpu = gpu
        self.numa = numa
        r = self.conn.call(Op.REGISTER_RANK, rank_id=rank_id, local_rank=rank_id, world_rank=rank_id, gpu_id=gpu,
                           numa_node=numa, pid=pid if pid is not None else os.getpid() * 1000 + rank_id)
        assert r["ok"], r["message"]
        self.epoch = r["rank_epoch"]
        self.ring_index = r["ring_index"]
        self.num_slots = r["num_slots"]

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
        self.conn.close()
