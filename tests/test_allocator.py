"""Slot-run placement in a GPU window (host-mode sessions, no GPU).

Large runs are placed from the top of the window and small ones first-fit
from the bottom, so releasing many small objects leaves one contiguous hole
that a later multi-slot object can use.
"""

import torch

from statespectre_b200 import in_process_daemon, offload_context

SLOT = 2 << 20


def _blob(slots: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 255, (slots * SLOT,), dtype=torch.uint8, generator=g)


def test_small_releases_leave_room_for_a_large_run(sock_path):
    # 256 MiB arena in 2 MiB slots = 128 slots
    d = in_process_daemon(socket=sock_path, arena_mb=256, slot_mb=2, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0) as off:
            small, large = [], []
            for i in range(6):  # interleaved: 6 x 1 slot and 6 x 16 slots = 102 slots
                small.append(off.copy(_blob(1, i), wait=True))
                large.append(off.copy(_blob(16, 100 + i), wait=True))
            for h in small:
                h.discard()
            big = _blob(30, 7)  # needs 30 contiguous slots; only 32 are free in total
            h = off.copy(big, wait=True)
            assert torch.equal(h.restore(), big)
            for i, hl in enumerate(large):  # the large runs kept their bytes
                assert torch.equal(hl.restore(), _blob(16, 100 + i))
    finally:
        d.stop()
