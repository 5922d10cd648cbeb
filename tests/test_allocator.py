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


def test_versioned_persistence_under_pinned_pressure(sock_path):
    """Many sealed versions with carry-forward in a window only 1.6x the model:
    reservations that find no contiguous run wait for the pressure drains
    (pinned -> pageable) instead of failing."""
    from statespectre_b200 import ModelRole
    from statespectre_b200.models.shapes import pick_changed

    sizes = [24 << 20, 24 << 20] + [4 << 20] * 20 + [64 << 10] * 20  # bytes, model-like mix
    total = sum(sizes)
    d = in_process_daemon(socket=sock_path, arena_mb=int(total * 1.6) >> 20, slot_mb=2, drain_on_complete=False,
                          retain_sealed_versions=2)
    try:
        with offload_context(daemon_addr=sock_path, device="cpu", rank=0, job_name="pressure") as off:
            roll = ModelRole.POLICY_ROLLOUT
            names = [f"w{i}" for i in range(len(sizes))]
            params = {n: torch.zeros(sz // 2, dtype=torch.bfloat16) for n, sz in zip(names, sizes)}
            pids = {}
            for v in range(1, 13):
                changed = names if v == 1 else [names[i] for i in pick_changed(names, 0.1, v)]
                for n in changed:
                    params[n].add_(1)
                    k = off.canonical_key(model_role=roll, model_version=v, param_name=n, tensor=params[n])
                    pids[n] = k.param_id
                    off.canonical_evict(params[n], k, destructive=False, wait=False)
                off._agent.synchronize()
                if v > 1:
                    off.carry_forward_version(roll, v - 1, v, [pids[n] for n in names if n not in changed])
                off.promote_rollout_version(v)
            man = off.get_manifest(roll, 12)
            assert len(man["tensors"]) == len(names)
    finally:
        d.stop()
