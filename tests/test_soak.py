"""Randomized soak of the daemon and host-mode agents (no GPU).

Four ranks, each on its own session, run a seeded random mix of evict, copy,
restore, restore_into, prefetch, batch evict/restore, location queries and
discards against a daemon whose pinned window is far smaller than the data in
flight, so reservations block, drains to pageable memory run continuously and
restores read back. Every restore is checked byte for byte; at the end the
daemon's invariant counters must be clean and every slot and pageable buffer
returned.
"""

import os
import random
import threading
import time

import pytest
import torch

from statespectre_b200 import _build, launch_daemon, offload_context

SECONDS = 8.0
RANKS = 4


def _rank(sock: str, rank: int, errors: list, counts: dict) -> None:
    rng = random.Random(1000 + rank)
    g = torch.Generator().manual_seed(rank)
    live = []  # (handle, reference tensor)
    n = 0
    try:
        with offload_context(daemon_addr=sock, device="cpu", rank=rank) as off:
            deadline = time.time() + SECONDS
            while time.time() < deadline:
                op = rng.random()
                if op < 0.30 or not live:
                    t = torch.randn(rng.choice([17, 1000, 65536, 262144, 700001]), generator=g)
                    ref = t.clone()
                    h = off.evict(t, wait=True) if rng.random() < 0.5 else off.copy(t, wait=True)
                    live.append((h, ref))
                elif op < 0.45:
                    ts = [torch.randn(rng.choice([256, 4096, 65536]), generator=g) for _ in range(rng.randint(2, 6))]
                    hs = off.evict_batch([t.clone() for t in ts])
                    outs = [torch.empty_like(t) for t in ts]
                    off.restore_batch(hs, outs)
                    for o, t in zip(outs, ts):
                        if not torch.equal(o, t):
                            errors.append(f"rank {rank}: batch round trip differs")
                    for h, t in zip(hs, ts):
                        live.append((h, t))
                elif op < 0.65:
                    h, ref = live[rng.randrange(len(live))]
                    if rng.random() < 0.5:
                        got = h.restore()
                    else:
                        got = torch.empty_like(ref)
                        h.restore_into(got)
                    if not torch.equal(got, ref):
                        errors.append(f"rank {rank}: restore differs ({h.location()})")
                elif op < 0.72:
                    h, ref = live[rng.randrange(len(live))]
                    p = h.prefetch()
                    p.wait()
                    if not torch.equal(h.restore(), ref):
                        errors.append(f"rank {rank}: restore after prefetch differs")
                elif op < 0.80:
                    h, _ = live[rng.randrange(len(live))]
                    if h.location() not in ("pinned", "pageable", "nvme"):
                        errors.append(f"rank {rank}: bad location {h.location()}")
                else:
                    h, _ = live.pop(rng.randrange(len(live)))
                    h.discard()
                n += 1
            for h, ref in live:
                if not torch.equal(h.restore(), ref):
                    errors.append(f"rank {rank}: final restore differs")
                h.discard()
            live.clear()
            off.synchronize()
    except Exception as e:  # noqa: BLE001
        errors.append(f"rank {rank}: {e!r}")
    counts[rank] = n


@pytest.mark.parametrize("binary", ["offloadd", "offloadd_tsan"])
def test_soak_random_mix_under_pressure(tmp_path, binary):
    if binary != "offloadd":
        _build.build(sanitizers=True)
    sock = str(tmp_path / "soak.sock")
    log = str(tmp_path / "d.log")
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=0")
    d = launch_daemon(sock, arena_mb=24, slot_mb=1, drain_on_complete=False, log_path=log, binary=binary, env=env)
    try:
        errors, counts = [], {}
        ths = [threading.Thread(target=_rank, args=(sock, r, errors, counts)) for r in range(RANKS)]
        for t in ths:
            t.start()
        for t in ths:
            t.join(SECONDS + 120)
        assert not any(t.is_alive() for t in ths), "a rank hung"
        assert not errors, errors[:10]
        assert sum(counts.values()) > 200, counts
        st = d.stats()
        for k in ("slot_overlap_prevented", "invalid_transition_rejected", "checksum_mismatch", "io_failure",
                  "lease_owner_mismatch_rejected", "rank_epoch_mismatch_rejected"):
            assert st[k] == 0, (k, st[k])
        deadline = time.time() + 10
        while time.time() < deadline and (st["used_slots"] or st["pageable_resident_bytes"]):
            time.sleep(0.05)
            st = d.stats()
        assert st["used_slots"] == 0 and st["pageable_resident_bytes"] == 0, st
        assert st["drains_completed"] > 0 and st["readbacks_completed"] > 0, st
    finally:
        rc = d.stop()
    text = open(log, errors="replace").read()
    assert "WARNING: ThreadSanitizer" not in text, text[-6000:]
    assert rc == 0
