"""Cold tiers: pinned -> pageable / NVMe drains, readback, spill and pressure."""

import os
import time

import pytest
import torch

from statespectre_b200 import in_process_daemon, offload_context

MB = 1 << 20


def wait_for(pred, timeout=10.0):
    end = time.time() + timeout
    while time.time() < end:
        if pred():
            return True
        time.sleep(0.01)
    return False


def roundtrip_tier(sock, expect_tier, n=1 << 20):
    with offload_context(daemon_addr=sock, device="cpu") as off:
        xs = [torch.randn(n) for _ in range(3)]
        hs = [off.copy(x, wait=True) for x in xs]
        for h in hs:
            assert wait_for(lambda: h.location() == expect_tier), h.location()
        for h, x in zip(hs, xs):
            assert torch.equal(h.restore(), x)
            # the pinned run of the readback is released again (cold copy is durable)
            assert h.location() == expect_tier
        stats = off.daemon_stats()
        for h in hs:
            h.discard()
        after = off.daemon_stats()
        return stats, after


def test_drain_to_pageable_and_readback(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True)
    try:
        s, after = roundtrip_tier(sock_path, "pageable")
        assert s["drains_completed"] == 3 and s["readbacks_completed"] == 3
        assert s["pinned_to_pageable_bytes"] == 3 * 4 * MB
        assert after["pageable_resident_bytes"] == 0  # discard freed the cold copies
    finally:
        d.stop()


@pytest.mark.parametrize("engine", ["pwrite", "io_uring"])
def test_drain_to_nvme_and_readback(sock_path, tmp_path, engine):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True, nvme_dir=str(tmp_path / "nvme"),
                          drain_target="nvme", io_engine=engine)
    try:
        s, after = roundtrip_tier(sock_path, "nvme", n=(1 << 20) + 333)
        assert s["nvme_write_bytes"] == 3 * ((4 << 20) + 4 * 333)
        assert s["nvme_read_bytes"] >= s["nvme_write_bytes"]
        files = os.listdir(tmp_path / "nvme")
        assert any(f.startswith("off_stripe_") for f in files)
        assert after["nvme_resident_bytes"] == 0
    finally:
        d.stop()


def test_pageable_then_nvme_spills_past_budget(sock_path, tmp_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True, nvme_dir=str(tmp_path / "nv"),
                          drain_target="pageable_then_nvme", pageable_limit_mb=6)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            xs = [torch.randn(1 << 20) for _ in range(3)]  # 4 MiB each; budget fits one
            hs = []
            for x in xs:
                h = off.copy(x, wait=True)
                assert wait_for(lambda: h.location() in ("pageable", "nvme"))
                hs.append(h)
            tiers = [h.location() for h in hs]
            assert tiers[0] == "pageable" and "nvme" in tiers[1:]
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
    finally:
        d.stop()


def test_forced_drain_makes_room_when_full(sock_path):
    # 16 MiB arena, 2 MiB slots: 8 x 4 MiB tensors do not fit without drains
    d = in_process_daemon(socket=sock_path, arena_mb=16, drain_on_complete=False, thresholds=(0.99, 0.995, 0.999))
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            xs = [torch.randn(1 << 20) for _ in range(8)]
            hs = [off.copy(x, wait=True) for x in xs]
            s = off.daemon_stats()
            assert s["drains_completed"] >= 4
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
    finally:
        d.stop()


def test_pressure_threshold_queues_background_drains(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=32, drain_on_complete=False, thresholds=(0.5, 0.7, 0.9))
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            hs = [off.copy(torch.randn(1 << 20), wait=True) for _ in range(6)]  # 24 of 32 MiB
            assert wait_for(lambda: off.daemon_stats()["drains_completed"] >= 1)
            s = off.daemon_stats()
            assert s["pressure_drains_normal_total"] + s["pressure_drains_priority_total"] + \
                s["pressure_drains_aggressive_total"] >= 1
            assert s["pinned_pressure_ppm"] <= 700_000
            for h in hs:
                h.restore()
    finally:
        d.stop()


def test_pageable_pool_reuses_drained_buffers(sock_path):
    """Buffers of drained tensors go back to a bounded pool and the next drains
    of the same sizes reuse them (already faulted-in memory)."""
    import time

    import torch

    from statespectre_b200 import in_process_daemon, offload_context

    d = in_process_daemon(socket=sock_path, arena_mb=256, slot_mb=4, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            xs = [torch.randn(n) for n in (3 << 20, 5 << 20, 1000)]
            for cycle in range(2):
                hs = [off.copy(x, wait=True) for x in xs]
                deadline = time.time() + 30
                while time.time() < deadline and not all(h.location() == "pageable" for h in hs):
                    time.sleep(0.005)
                assert all(h.location() == "pageable" for h in hs)
                for h, x in zip(hs, xs):
                    assert torch.equal(h.restore(), x)
                off.discard_batch(hs)
                st = off.daemon_stats()
                assert st["pageable_resident_bytes"] == 0
                # 12 MiB + 20 MiB + one 2 MiB class are pooled, and stay pooled across cycles
                assert st["pageable_pool_bytes"] == (12 + 20 + 2) << 20, (cycle, st["pageable_pool_bytes"])
    finally:
        d.stop()


@pytest.mark.parametrize("drain_on_complete", [True, False])
@pytest.mark.parametrize("wait", [True, False])
def test_evict_batch_larger_than_pinned_window_waits_out_backpressure(sock_path, drain_on_complete, wait):
    # 8 MiB window, 1 MiB slots, one batch of 24 x 1 MiB: the items past the
    # window are answered blocked until the batch's own earlier copies are
    # published and drained (in the background, or forced by the reservation).
    d = in_process_daemon(socket=sock_path, arena_mb=8, slot_mb=1, drain_on_complete=drain_on_complete,
                          thresholds=(0.99, 0.995, 0.999))
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            xs = [torch.randn(1 << 18) for _ in range(24)]
            hs = off.evict_batch(xs, wait=wait)
            s = off.daemon_stats()
            assert s["blocked_reservation_count"] > 0 and s["drains_completed"] >= 16
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
            off.discard_batch(hs)
    finally:
        d.stop()


def test_pressure_drains_stop_at_the_normal_threshold_during_a_batch(sock_path):
    # 11 slots of 4 MiB, 8 blocks per batch: 73 % full after the batch, so
    # pressure drains take it back to the 60 % normal threshold (2 runs), not
    # every run that completes while earlier drains are still queued.
    d = in_process_daemon(socket=sock_path, arena_mb=44, slot_mb=4, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            blocks = [torch.randn(1 << 20) for _ in range(16)]
            for it in range(6):
                sel = blocks[it % 2 * 8: it % 2 * 8 + 8]
                hs = off.evict_batch(sel, wait=True)
                outs = [torch.empty_like(b) for b in sel]
                off.restore_batch(hs, outs)
                assert all(torch.equal(o, b) for o, b in zip(outs, sel))
                off.discard_batch(hs)
            s = off.daemon_stats()
            assert 1 <= s["drains_completed"] <= 3 * 6, s["drains_completed"]
            assert s["readbacks_completed"] <= 3 * 6
    finally:
        d.stop()


def test_restore_waits_for_pinned_capacity_instead_of_failing(sock_path):
    """A readback that finds every pinned run busy (D2H copies in flight, which
    no drain can take) backs off and completes once capacity returns, rather
    than failing the restore."""
    import threading

    from rawclient import RawRank
    from statespectre_b200._wire import Op

    d = in_process_daemon(socket=sock_path, arena_mb=16, slot_mb=1, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            x = torch.randn(1 << 18)  # 1 MiB: one slot
            h = off.copy(x, wait=True)
            assert wait_for(lambda: h.location() == "pageable"), h.location()
            r = RawRank(sock_path, 9)
            held = []
            for i in range(64):  # hold every free slot with a D2H that has not completed
                g = r.reserve(1000 + i, 1, 1 << 20)
                if not g["ok"]:
                    break
                assert r.mark(Op.MARK_D2H_SUBMITTED, g["lease_id"], 1000 + i, 1, g["slot_id"])["ok"]
                held.append((1000 + i, g))
            assert held, "no slot could be reserved"
            out = {}

            def restore():
                try:
                    out["y"] = h.restore()
                except Exception as e:  # noqa: BLE001
                    out["err"] = e

            t = threading.Thread(target=restore, daemon=True)
            t.start()
            t.join(1.0)
            assert t.is_alive() and not out, out  # waiting, not failed
            assert off.daemon_stats()["blocked_reservation_count"] >= 1
            for tid, g in held:  # the copies finish; their runs drain and free
                assert r.mark(Op.MARK_D2H_COMPLETE, g["lease_id"], tid, 1, g["slot_id"])["ok"]
            t.join(60)
            assert not t.is_alive() and "err" not in out, out
            assert torch.equal(out["y"], x)
            r.close()
    finally:
        d.stop()


def test_batched_restores_under_pressure_from_several_ranks_make_progress():
    """Ranks moving batches of blocks through a pinned window half the size
    of what they hold: restore_batch hands on the completions of the blocks it
    already restored before it waits for readback capacity, so a batch never
    waits on runs it holds itself (or another rank's batch on those)."""
    from statespectre_b200.benchmarks.control import run_kv

    r = run_kv(1.5, ranks=2, nblocks=16)
    assert r["errors"] == [] and r["byte_exact"]
    assert r["items_per_s"] > 0 and r["drains"] > 0 and r["readbacks"] > 0


@pytest.mark.parametrize("copy_threads", [0, 8])
def test_tier_copies_split_over_the_copy_pool_are_exact(sock_path, copy_threads):
    """Drains and readbacks of sizes that split into uneven 1 MiB pieces (and
    a size below two pieces) come back byte-exact with and without pool
    threads."""
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True, copy_threads=copy_threads)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            g = torch.Generator().manual_seed(copy_threads)
            xs = [torch.randint(0, 255, (n,), dtype=torch.uint8, generator=g)
                  for n in (3 * MB + 4097, 1 * MB + 17, 9 * MB + 123, 2 * MB)]
            hs = [off.copy(x, wait=True) for x in xs]
            for h in hs:
                assert wait_for(lambda: h.location() == "pageable"), h.location()
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
                h.discard()
    finally:
        d.stop()


def test_drains_stay_pinned_when_the_host_is_out_of_memory(sock_path):
    """Without a pageable budget the pageable tier takes only what the host
    has to spare: with (fake) available memory under the reserve, drains fail
    and the tensors stay pinned and restorable; once memory is back, drains
    go through."""
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=True)
    try:
        d.fake_host_memory(1 << 30)  # 1 GiB available: below the 4 GiB reserve
        with offload_context(daemon_addr=sock_path, device="cpu") as off:
            xs = [torch.randn(1 << 20) for _ in range(3)]
            hs = [off.copy(x, wait=True) for x in xs]
            assert wait_for(lambda: off.daemon_stats()["pageable_room_rejected_total"] >= 3)
            assert all(h.location() == "pinned" for h in hs)
            assert off.daemon_stats()["pageable_resident_bytes"] == 0
            for h, x in zip(hs, xs):
                assert torch.equal(h.restore(), x)
            d.fake_host_memory(1 << 50)
            more = [torch.randn(1 << 20) for _ in range(2)]
            hm = [off.copy(x, wait=True) for x in more]
            for h in hm:
                assert wait_for(lambda: h.location() == "pageable"), h.location()
            for h, x in zip(hm, more):
                assert torch.equal(h.restore(), x)
    finally:
        d.stop()


def test_daemon_refuses_arenas_larger_than_host_memory(sock_path):
    """Arenas are faulted in at start: a config asking for more than the host
    has is refused with the numbers instead of the daemon being killed
    half-way through the first touch."""
    with pytest.raises(Exception, match="arenas need .* MiB but the host has .* MiB available"):
        in_process_daemon(socket=sock_path, arena_mb=1 << 26)  # 64 TiB
