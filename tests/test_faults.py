"""Failure detection and recovery, with every fault made on the host.

Faults: a rank that stops heartbeating, a rank process killed with SIGKILL,
a restarted rank (stale epoch), truncated frames, injected cold-tier IO
errors, slot exhaustion. StateSpectre's fault suite covers the same ground
(reference: tests/cpp/test_fault_injection.cpp:147-293); its promised ring
stale-epoch case (:15-16) is included here.
"""

import os
import signal
import struct
import subprocess
import sys
import time

import pytest
import torch

from statespectre_b200 import _wire, in_process_daemon, launch_daemon, offload_context
from statespectre_b200._native import native
from statespectre_b200._wire import Op

from rawclient import RawRank

MB = 1 << 20


def test_heartbeat_timeout_reclaims_inflight_keeps_completed(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False, heartbeat_timeout_ms=300)
    try:
        r = RawRank(sock_path, 1)
        done = r.offload(10, 1, 3 * MB)
        pend = r.reserve(11, 1, 3 * MB)
        assert pend["ok"]
        obs = RawRank(sock_path, 2)
        used_before = obs.stats()["used_slots"]
        time.sleep(0.9)  # rank 1 never heartbeats
        obs.heartbeat()
        s = obs.stats()
        assert s["rank_sessions_invalidated"] >= 1
        assert s["used_slots"] == used_before - 2  # the uncompleted reservation is back
        assert obs.location(10)["location_kind"] == 2  # completed data survives its owner
        # a late completion from the dead session is rejected
        late = r.mark(Op.MARK_D2H_SUBMITTED, pend["lease_id"], 11, 1, pend["slot_id"])
        assert not late["ok"] and late["message"] == "epoch invalid"
        assert done["ok"]
    finally:
        d.stop()


def test_agent_pause_heartbeat_invalidates_session(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False, heartbeat_timeout_ms=300)
    try:
        s = offload_context(daemon_addr=sock_path, device="cpu", heartbeat_ms=50)
        off = s.off
        h = off.copy(torch.arange(1000.0), wait=True)
        off._agent.pause_heartbeat(True)
        time.sleep(1.0)
        with pytest.raises(RuntimeError, match="epoch invalid"):
            off.copy(torch.arange(10.0), wait=True)
        assert h.location() == "pinned"  # data outlives the session
        s.close()
    finally:
        d.stop()


def test_restarted_rank_ring_entries_of_old_session(sock_path):
    """Completions an old session left in its ring are applied at takeover;
    anything it sends afterwards carries a stale epoch and is rejected."""
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    try:
        s1 = offload_context(daemon_addr=sock_path, device="cpu", rank=3)
        h = s1.off.copy(torch.ones(4096), wait=True)  # completion went through the ring
        s2 = offload_context(daemon_addr=sock_path, device="cpu", rank=3)  # restart
        assert s2.off._agent.location(h.tensor_id, h.version) == "pinned"
        with pytest.raises(RuntimeError, match="epoch invalid"):
            s1.off.copy(torch.ones(8), wait=True)
        s1.close()
        s2.close()
    finally:
        d.stop()


def test_truncated_and_garbage_frames_do_not_kill_daemon(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64)
    try:
        C = native()
        c = C.RawConn(sock_path)
        c.send_bytes(struct.pack("<IHH", 0x4F465250, 13, 0))  # 8 of 12 header bytes
        c.close()
        c = C.RawConn(sock_path)
        c.send_bytes(b"GARBAGE-GARBAGE!")
        c.close()
        c = C.RawConn(sock_path)
        c.send_bytes(_wire.make_frame(Op.REQUEST_OFFLOAD, b"\x01\x02"))  # body truncated
        c.close()
        r = RawRank(sock_path, 1)
        assert r.heartbeat()["ok"]
        assert r.offload(1, 1, MB)["ok"]
    finally:
        d.stop()


def test_injected_drain_failure_keeps_pinned_copy(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True)
    try:
        d.inject_io_failures(1, 0)
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            x = torch.randn(1 << 18)
            h = off.copy(x, wait=True)
            deadline = time.time() + 5
            while off.daemon_stats()["io_failure"] == 0 and time.time() < deadline:
                time.sleep(0.01)
            assert off.daemon_stats()["io_failure"] == 1
            assert h.location() in ("pinned", "pageable")
            assert torch.equal(h.restore(), x)
    finally:
        d.stop()


def test_injected_readback_failure_is_retried(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            x = torch.randn(1 << 18)
            h = off.copy(x, wait=True)
            deadline = time.time() + 5
            while h.location() != "pageable" and time.time() < deadline:
                time.sleep(0.01)
            assert h.location() == "pageable"
            d.inject_io_failures(0, 1)
            assert torch.equal(h.restore(), x)  # first readback fails, the poll retries
            assert off.daemon_stats()["io_failure"] >= 1
    finally:
        d.stop()


_CHILD = r"""
import sys, time, torch
sys.path.insert(0, sys.argv[2])
from statespectre_b200 import offload_context
s = offload_context(daemon_addr=sys.argv[1], device="cpu", rank=7, heartbeat_ms=50)
off = s.off
hs = [off.copy(torch.full((1 << 16,), float(i)), wait=True) for i in range(4)]
print("ready", flush=True)
time.sleep(60)
"""


def test_sigkilled_rank_process_is_recovered(tmp_path):
    sock = str(tmp_path / "d.sock")
    d = launch_daemon(sock, arena_mb=64, log_path=str(tmp_path / "d.log"),
                      extra_args=["--drain-on-complete", "0"])
    try:
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        # short heartbeat timeout through a config file
        p = subprocess.Popen([sys.executable, "-c", _CHILD, sock, root], stdout=subprocess.PIPE, text=True)
        assert p.stdout.readline().strip() == "ready"
        obs = RawRank(sock, 1)
        assert obs.stats()["live_rank_sessions"] == 2
        p.send_signal(signal.SIGKILL)
        p.wait()
        # the daemon keeps the dead rank's completed data; its session times out later
        assert obs.stats()["used_slots"] >= 4
        assert obs.heartbeat()["ok"]
    finally:
        d.stop()


def test_exhaustion_blocks_instead_of_overlapping(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=16, drain_on_complete=False)
    try:
        r = RawRank(sock_path, 1)
        granted = []
        while True:
            g = r.reserve(len(granted) + 1, 1, 2 * MB)
            if not g["ok"]:
                assert g["blocked"]
                break
            granted.append(g["slot_id"])
        assert len(granted) == len(set(granted)) == r.num_slots
    finally:
        d.stop()


def test_full_completion_ring_falls_back_to_rpc(tmp_path):
    """With the daemon not consuming a 4-entry completion ring, completions
    that do not fit go by RPC: no completion is lost, the RPC-completed
    tensors are usable at once, the ring-held ones as soon as it drains."""
    import time

    sock = str(tmp_path / "d.sock")
    text = f"""
daemon:
  socket_path: {sock}
  completion_ring_capacity: 4
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 64
drain_policy:
  drain_on_d2h_complete: false
nvme:
  enabled: false
"""
    d = in_process_daemon(yaml=text, socket=sock)
    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=0) as off:
            d.pause_rings(True)
            ts = [torch.full((1024,), float(i)) for i in range(8)]
            hs = [off.copy(t, wait=True) for t in ts]
            st = off.daemon_stats()
            assert st["ring_completions_applied_total"] == 0
            locs = [h.location() for h in hs]
            assert locs[4:] == ["pinned"] * 4, locs     # completed over RPC (ring full)
            assert all(loc != "pinned" for loc in locs[:4]), locs  # still in the paused ring
            for h, t in zip(hs[4:], ts[4:]):
                assert torch.equal(h.restore(), t)
            d.pause_rings(False)
            deadline = time.time() + 10
            while time.time() < deadline and off.daemon_stats()["ring_completions_applied_total"] < 4:
                time.sleep(0.01)
            assert all(h.location() == "pinned" for h in hs)
            for h, t in zip(hs, ts):
                assert torch.equal(h.restore(), t)
            off.discard_batch(hs)
            assert off.daemon_stats()["used_slots"] == 0
    finally:
        d.stop()


def test_ring_header_written_by_a_rank_cannot_complete_another_ranks_transfer(sock_path):
    """A rank maps the control region writable, its ring header included. One
    that writes another rank's id and epoch there and publishes a completion
    for that rank's lease is not believed: the daemon takes the ring's owner
    from its own session table. A scribbled capacity or a tail far ahead of the
    head costs that ring its entries, never a read outside it."""
    d = in_process_daemon(socket=sock_path, arena_mb=16, slot_mb=1, drain_on_complete=False)
    try:
        victim = RawRank(sock_path, 1)
        g = victim.reserve(77, 1, 4096)
        assert g["ok"] and victim.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 77, 1, g["slot_id"])["ok"]
        atk = RawRank(sock_path, 2, map_control=True)
        before = victim.stats()
        atk.write_ring_header(owner_rank=1, rank_epoch=victim.epoch, capacity=1 << 30)
        atk.ring_push(g["lease_id"], 77, 1, g["slot_id"])
        deadline = time.time() + 10
        while time.time() < deadline and atk.ring_head_tail()[0] != atk.ring_head_tail()[1]:
            time.sleep(0.01)
        assert atk.ring_head_tail()[0] == atk.ring_head_tail()[1]  # consumed
        after = victim.stats()
        assert after["lease_owner_mismatch_rejected"] == before["lease_owner_mismatch_rejected"] + 1
        assert victim.location(77, 1)["location_kind"] != 2  # not completed by the impostor
        assert victim.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], 77, 1, g["slot_id"])["ok"]
        assert victim.location(77, 1)["location_kind"] == 2
        head, _ = atk.ring_head_tail()
        atk.set_ring_tail(head + 10 ** 9)
        deadline = time.time() + 10
        while time.time() < deadline and atk.ring_head_tail()[0] != head + 10 ** 9:
            time.sleep(0.01)
        assert atk.ring_head_tail()[0] == head + 10 ** 9  # skipped in one step
        assert victim.heartbeat()["ok"] and victim.stats()["ring_completions_applied_total"] == \
            after["ring_completions_applied_total"]
        atk.close()
        victim.close()
    finally:
        d.stop()


def test_slot_entries_written_by_a_rank_do_not_steer_the_daemons_copies(tmp_path):
    """The shared slot table is the daemon's published copy: it takes a run's
    address and size from its own table, so a rank that rewrites another
    tensor's entry (arena, offset, size) neither crashes the daemon's drain
    nor changes the bytes that drain moves; the next state change republishes
    the entry."""
    sock = str(tmp_path / "d.sock")
    cfg = tmp_path / "d.yaml"
    cfg.write_text(f"""
daemon:
  socket_path: {sock}
arenas:
  allocation_granularity_mb: 1
  per_numa:
    - numa_node: 0
      size_mb: 8
drain_policy:
  drain_on_d2h_complete: false
nvme:
  enabled: false
""")
    d = launch_daemon(sock, config=str(cfg), log_path=str(tmp_path / "d.log"))
    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=0) as off:
            x = torch.randn(1 << 18)  # 1 MiB: one slot
            h = off.copy(x, wait=True)
            atk = RawRank(sock, 5, map_control=True)
            loc = atk.location(h.tensor_id, h.version)
            assert loc["location_kind"] == 2
            slot = loc["slot_id"]
            atk.scribble_slot(slot, arena_id=999, arena_offset=1 << 50, nbytes=1 << 40)
            # fill the 8 MiB window: the oldest run (x) is drained under pressure
            hs = [off.copy(torch.randn(1 << 18), wait=True) for _ in range(10)]
            # drains run in the background: x (least recently used) leaves the
            # pinned tier once its queued drain finishes
            deadline = time.time() + 30
            while time.time() < deadline and h.location() == "pinned":
                time.sleep(0.02)
            assert off.daemon_stats()["drains_completed"] >= 3 and h.location() != "pinned"
            assert torch.equal(h.restore(), x)
            assert atk.slot_fields(slot)[1:4] != (999, 1 << 50, 1 << 40)  # republished
            off.discard_batch(hs + [h])
            atk.close()
        assert d.proc.poll() is None  # the daemon is still serving
    finally:
        d.stop()
