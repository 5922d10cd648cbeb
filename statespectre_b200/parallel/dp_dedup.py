"""Data-parallel deduplicated canonical eviction.

Every DP replica holds the same parameter bytes; only one of them should pay
the GPU -> host copy. StateSpectre lets the first rank to arrive create and
the rest attach on trust, or makes every replica copy a candidate and
compares host-side hashes (reference: src/daemon/canonical.cpp:298-341).

Here, for each parameter one owner rank creates the object (K1 copies the
bytes and computes the ssh128 hash in the same pass); after a barrier the
other replicas run in ``device_hash_verified`` mode: each hashes its own GPU
copy at HBM rate and the daemon compares it with the owner's hash, so no
verification byte crosses PCIe. Ownership is round-robin over parameters by
default, which spreads the copies over all the replicas' PCIe links instead of
funnelling the whole model through one.

``verify_p2p`` (parallel.fabric) additionally compares replica bytes exactly
against the owner's GPU copy over NVLink while the owner still holds it.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

from ..api import CanonicalHandle, DedupPolicy, Off


def _world(group) -> tuple:
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def dedup_evict_params(off: Off, params: Dict[str, torch.Tensor], *, model_role, model_version: int,
                       policy: Optional[DedupPolicy] = None, group=None, owner: str = "round_robin",
                       destructive: bool = True, tp_rank: int = 0, pp_rank: int = 0) -> Dict[str, CanonicalHandle]:
    """Canonically evict ``params`` (identical on every rank of ``group``).

    Returns name -> CanonicalHandle. Owners see NEED_D2H_CREATE; replicas see
    VERIFIED_BY_DEVICE_HASH (device_hash_verified), ATTACHED_EXISTING
    (semantic_trusted) or DUPLICATE_CANDIDATE (hash_verified).
    """
    import torch.distributed as dist

    policy = policy or DedupPolicy("device_hash_verified")
    rank, world = _world(group)
    names = sorted(params)

    def owner_of(i: int) -> int:
        return 0 if owner == "rank0" else i % world

    out: Dict[str, CanonicalHandle] = {}
    keys = {n: off.canonical_key(model_role=model_role, model_version=model_version, param_name=n,
                                 tensor=params[n], tp_rank=tp_rank, pp_rank=pp_rank) for n in names}
    for i, n in enumerate(names):  # phase 1: owners create
        if owner_of(i) == rank:
            out[n] = off.canonical_evict(params[n], keys[n], dedup_policy=policy, destructive=destructive)
    if world > 1:
        dist.barrier(group)
    for i, n in enumerate(names):  # phase 2: replicas verify or attach
        if owner_of(i) != rank:
            out[n] = off.canonical_evict(params[n], keys[n], dedup_policy=policy, destructive=destructive,
                                         wait_for_creator=True)
    if world > 1:
        dist.barrier(group)
    return out
