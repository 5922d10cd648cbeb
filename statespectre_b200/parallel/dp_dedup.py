"""Data-parallel deduplicated canonical eviction.

Every DP replica holds the same parameter bytes; only one of them should pay
the GPU -> host copy. StateSpectre lets the first rank to arrive create and
the rest attach on trust, or makes every replica copy a candidate and
compares host-side hashes (reference: src/daemon/canonical.cpp:298-341,
324-341 and 488-495 for the candidate path).

Here, for each parameter one owner rank creates the object (K1 copies the
bytes to pinned memory, zbf16-coded for bf16 parameters, and computes the
ssh128 hash of the raw bytes in the same pass; each rank's parameters go in
one ``canonical_evict_batch``).
Ownership is round-robin over parameters by default, which spreads the copies
over all the replicas' PCIe links instead of funnelling the whole model
through one. The other replicas then verify without copying, by one of:

  * ``device_hash_verified`` (dedup mode 4): each replica hashes its own GPU
    copy at HBM rate and the daemon compares it with the owner's hash; no
    verification byte crosses PCIe or NVLink.
  * ``p2p_verified`` (dedup mode 5): each replica compares its bytes exactly
    with the owner's GPU copy over NVLink (K3 ``verify_peer``: plain peer
    loads of the owner's allocation, mapped by CUDA IPC, against the local
    bytes, hashing the local copy in the same pass), then attaches. The owners
    keep their GPU copies until every replica has compared; a destructive
    eviction releases them after that.

With ``semantic_trusted`` replicas attach without any check.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch

from ..api import CanonicalHandle, DedupPolicy, Off, _invalidate_callback


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
    VERIFIED_BY_DEVICE_HASH (device_hash_verified), VERIFIED_BY_P2P
    (p2p_verified), ATTACHED_EXISTING (semantic_trusted) or
    DUPLICATE_CANDIDATE (hash_verified). In ``p2p_verified`` mode a replica
    whose bytes differ from the owner's raises ``RuntimeError`` on every rank
    (after all ranks finished the collective steps).
    """
    import torch.distributed as dist

    policy = policy or DedupPolicy("device_hash_verified")
    rank, world = _world(group)
    names = sorted(params)
    p2p = policy.mode == "p2p_verified" and world > 1

    def owner_of(i: int) -> int:
        return 0 if owner == "rank0" else i % world

    out: Dict[str, CanonicalHandle] = {}
    keys = {n: off.canonical_key(model_role=model_role, model_version=model_version, param_name=n,
                                 tensor=params[n], tp_rank=tp_rank, pp_rank=pp_rank) for n in names}
    # phase 1: owners create (and keep their GPU copy for peers in p2p mode);
    # one batch, so the round trips of later parameters overlap earlier copies
    mine = [n for i, n in enumerate(names) if owner_of(i) == rank]
    for n, h in zip(mine, off.canonical_evict_batch([(params[n], keys[n]) for n in mine], dedup_policy=policy,
                                                    destructive=destructive and not p2p)):
        out[n] = h
    if p2p:
        _verify_replicas_p2p(params, names, owner_of, rank, world, group)
    elif world > 1:
        dist.barrier(group)
    theirs = [n for i, n in enumerate(names) if owner_of(i) != rank]  # phase 2: replicas verify or attach
    for n, h in zip(theirs, off.canonical_evict_batch([(params[n], keys[n]) for n in theirs], dedup_policy=policy,
                                                      destructive=destructive, wait_for_creator=True)):
        out[n] = h
    if world > 1:
        dist.barrier(group)  # in p2p mode: no replica reads an owner's copy any more
    if p2p and destructive:
        for i, n in enumerate(names):
            if owner_of(i) == rank:
                torch.cuda.current_stream(params[n].device).synchronize()
                _invalidate_callback(params[n])()
    return out


def verify_p2p(params: Dict[str, torch.Tensor], names: List[str], owner_of, rank: int, world: int,
               group=None) -> List[str]:
    """Exact byte comparison of this rank's copies of the parameters owned by
    other ranks against the owners' GPU copies, over NVLink. Every rank of
    ``group`` calls it together. Returns the names whose bytes differ from the
    owner's on any rank (the same list on every rank)."""
    import torch.distributed as dist

    from .._native import native
    from .fabric import export_tensor

    C = native()
    # 1. every rank exports the allocations behind the parameters it owns
    allocs: List[bytes] = []
    index: Dict[int, tuple] = {}
    for i, n in enumerate(names):
        if owner_of(i) != rank:
            continue
        e = export_tensor(params[n])
        h = bytes(e["handle"])
        if h not in allocs:
            allocs.append(h)
        index[i] = (allocs.index(h), int(e["offset"]), int(e["nbytes"]))
    exports = [None] * world
    dist.all_gather_object(exports, (allocs, index), group=group)
    # 2. compare against each owner's copy with K3 (plain loads of peer memory)
    mine = [i for i, _ in enumerate(names) if owner_of(i) != rank]
    dev = next(iter(params.values())).device
    stream = torch.cuda.current_stream(dev)
    nchunks = [(params[names[i]].numel() * params[names[i]].element_size() + 65535) // 65536 for i in mine]
    dig = torch.empty(max(sum(nchunks), 1), dtype=torch.int64, device=dev)
    mism = torch.zeros(max(len(mine), 1), dtype=torch.int32, device=dev)
    mapped: Dict[tuple, int] = {}
    try:
        dbase = 0
        for k, i in enumerate(mine):
            o = owner_of(i)
            o_allocs, o_index = exports[o]
            a, offset, nbytes = o_index[i]
            local = params[names[i]]
            if local.numel() * local.element_size() != nbytes:
                raise ValueError(f"{names[i]}: {local.numel() * local.element_size()} bytes here, "
                                 f"{nbytes} on rank {o}")
            if (o, a) not in mapped:
                mapped[(o, a)] = C.ipc_open(o_allocs[a], 0)
            C.k_verify_peer(local.data_ptr(), mapped[(o, a)] + offset, nbytes, dig.data_ptr() + 8 * dbase,
                            mism.data_ptr() + 4 * k, stream.cuda_stream, 0)
            dbase += nchunks[k]
        stream.synchronize()
        bad = [names[i] for k, i in enumerate(mine) if int(mism[k].item()) != 0] if mine else []
    finally:
        dist.barrier(group)  # every replica finished reading the owners' memory
        for ptr in mapped.values():
            C.ipc_close(ptr)
    everyone = [None] * world
    dist.all_gather_object(everyone, bad, group=group)
    return sorted({n for b in everyone for n in b})


def _verify_replicas_p2p(params, names, owner_of, rank, world, group) -> None:
    import torch.distributed as dist

    dist.barrier(group)  # the owners' objects exist and their copies are complete
    bad = verify_p2p(params, names, owner_of, rank, world, group)
    if bad:
        raise RuntimeError(f"p2p_verified: {len(bad)} parameter(s) differ between DP replicas: {bad[:8]}")
