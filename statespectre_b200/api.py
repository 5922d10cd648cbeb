"""User API of the offload runtime.

Surface and semantics follow StateSpectre's ``state_spectre`` package
(reference: python_api/state_spectre/__init__.py:25-946) so existing user code
switches by changing the import:

    with offload_context(device="cuda:0") as off:
        h = off.evict(x, name="x")        # VRAM freed once the copy lands
        x = h.restore()                   # new tensor, byte-identical

Differences that are additions, not changes:
  * ``device="cpu"`` opens a host-mode session for CPU tensors;
  * restores can cast on the fly (``cast="fp8_block128"`` returns
    ``(fp8 tensor, fp32 scales)``) and re-verify content hashes;
  * every evict carries a 128-bit content hash computed on the GPU in the
    same pass as the copy (``OffloadHandle.content_hash``);
  * ``evict_batch`` / ``restore_batch`` move many small tensors (KV-cache
    blocks) with one reservation round trip;
  * ``PrefetchHandle.wait`` waits for the restore copy itself (StateSpectre
    waited on the evict flag, reference: __init__.py:272-274);
  * bf16 tensors of 4 MiB and more cross PCIe in zbf16 coding (lossless
    exponent coding, about 0.75 of the bytes; ``OffloadHandle.coded``);
    ``offload_context(..., compress=False)`` moves them uncoded.
"""

from __future__ import annotations

import contextlib
import itertools
import json
import os
import threading
import time
from typing import Iterable, List, Optional, Sequence, Tuple, Union

import torch

from . import _wire
from ._native import native

__all__ = [
    "offload_context", "Off", "OffloadHandle", "PrefetchHandle", "ManagedRecord", "CanonicalKey",
    "DedupPolicy", "ModelRole", "CanonicalHandle", "INTERNAL_STREAM",
]

INTERNAL_STREAM = (1 << 64) - 1


class ModelRole:
    UNKNOWN = 0
    POLICY_TRAINABLE = 1
    POLICY_ROLLOUT = 2
    POLICY_REFERENCE = 3
    REWARD_MODEL = 4
    VALUE_MODEL = 5
    AUXILIARY = 6
    _BY_NAME = {"unknown": 0, "policy_trainable": 1, "policy_rollout": 2, "policy_reference": 3,
                "reward_model": 4, "value_model": 5, "auxiliary": 6}

    @classmethod
    def parse(cls, role) -> int:
        if isinstance(role, int):
            return role
        r = str(role).lower()
        if r not in cls._BY_NAME:
            raise ValueError(f"unknown model_role {role!r}; one of {list(cls._BY_NAME)}")
        return cls._BY_NAME[r]


# 4 and 5 are additions of this runtime: "device_hash_verified" replicas hash
# their own GPU copy for the daemon to compare; "p2p_verified" replicas have
# compared their bytes with the owner's GPU copy over NVLink
# (parallel.dp_dedup) and attach.
DEDUP_MODES = {"disabled": 0, "semantic_trusted": 1, "hash_verified": 2, "sampled_hash": 3,
               "device_hash_verified": 4, "p2p_verified": 5}
ACTION_NAMES = {0: "ATTACHED_EXISTING", 1: "NEED_D2H_CREATE", 2: "WAIT_FOR_CREATOR", 3: "DUPLICATE_CANDIDATE",
                4: "REJECTED_STALE_VERSION", 5: "QUOTA_EXCEEDED", 6: "VERIFIED_BY_DEVICE_HASH",
                7: "VERIFIED_BY_P2P", 255: "ERROR"}
CASTS = {None: 0, "none": 0, "fp8_block128": 1, "bf16": 2, "fp32": 3}
# evict data hints: payloads the agent may code for transfer (zbf16 / zf32)
_FMT_HINTS = {torch.bfloat16: 1, torch.float32: 2}

# c10::ScalarType numbering: the dtype field of a canonical key carries it so
# keys match ranks that report tensor.scalar_type() from C++.
_SCALAR_TYPE = {
    torch.uint8: 0, torch.int8: 1, torch.int16: 2, torch.int32: 3, torch.int64: 4, torch.float16: 5,
    torch.float32: 6, torch.float64: 7, torch.complex64: 9, torch.complex128: 10, torch.bool: 11,
    torch.bfloat16: 15,
}
for _name, _code in (("float8_e5m2", 23), ("float8_e4m3fn", 24)):
    if hasattr(torch, _name):
        _SCALAR_TYPE[getattr(torch, _name)] = _code


def fnv1a64(data: bytes, seed: int = 1469598103934665603) -> int:
    """64-bit FNV-1a (stable parameter-id / shape hashing)."""
    h = seed
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def hash_ints(values) -> int:
    buf = bytearray()
    for v in values:
        buf += (int(v) & 0xFFFFFFFFFFFFFFFF).to_bytes(8, "little")
    return fnv1a64(bytes(buf))


def _stream_handle(stream, device: torch.device) -> int:
    if stream is None:
        return torch.cuda.current_stream(device).cuda_stream if device.type == "cuda" else 0
    if isinstance(stream, int):
        return stream
    if hasattr(stream, "cuda_stream"):
        return int(stream.cuda_stream)
    raise TypeError("stream must be None, a torch.cuda.Stream or an int handle")


def _validate_destructive(t: torch.Tensor, unsafe_autograd: bool) -> None:
    if not t.is_contiguous():
        raise RuntimeError("evict: tensor must be contiguous for destructive eviction "
                           "(use allow_views=True, compact=True to copy a view)")
    if t.storage_offset() != 0:
        raise RuntimeError("evict: tensor.storage_offset() must be 0 for destructive eviction "
                           "(use allow_views=True, compact=True to copy a view)")
    logical = t.numel() * t.element_size()
    storage = t.untyped_storage().nbytes()
    if logical != storage:
        raise RuntimeError(f"evict: logical nbytes ({logical}) != underlying storage nbytes ({storage}); "
                           "tensor does not own its full storage. Use allow_views=True, compact=True.")
    if t.requires_grad and not unsafe_autograd:
        raise RuntimeError("evict: tensor.requires_grad is True; destructive eviction would invalidate an "
                           "autograd-tracked tensor. Pass unsafe_autograd=True (inside "
                           "off.unsafe_destructive_mode()) to accept responsibility.")


def _invalidate_callback(t: torch.Tensor):
    """Replace the storage (not just the shape) once the copy has landed."""
    opts = {"dtype": t.dtype, "device": t.device}

    def cb(t=t):
        t.data = torch.empty(0, **opts)  # Tensor::set_data: storage swapped, old one freed

    return cb


class OffloadHandle:
    """Handle to an offloaded tensor; carries what restore needs."""

    __slots__ = ("tensor_id", "version", "name", "shape", "stride", "dtype", "device_origin", "nbytes", "_off",
                 "_prefetched", "_discarded", "coded")

    def __init__(self, off, tensor_id, version, name, shape, stride, dtype, device_origin, nbytes):
        self._off = off
        self.tensor_id = int(tensor_id)
        self.version = int(version)
        self.name = name
        self.shape = torch.Size(shape)
        self.stride = tuple(stride)
        self.dtype = dtype
        self.device_origin = device_origin
        self.nbytes = int(nbytes)
        self._prefetched = None
        self._discarded = False
        self.coded = False  # moved zbf16-coded (lossless) when True

    def ready(self) -> bool:
        """True once the copy into the pinned slot has completed."""
        return self._off._agent.is_offloaded(self.tensor_id, self.version)

    def wait_offloaded(self) -> None:
        self._off._agent.wait_offloaded(self.tensor_id, self.version)

    @property
    def content_hash(self) -> Optional[tuple]:
        """(lo, hi) ssh128 content hash of the offloaded bytes, once known."""
        return self._off._agent.tensor_hash(self.tensor_id, self.version)

    def location(self) -> str:
        return self._off._agent.location(self.tensor_id, self.version)

    def prefetch(self, device=None, stream=None) -> "PrefetchHandle":
        """Start the restore now (asynchronously); ``restore()`` then returns it."""
        if self._discarded:
            raise RuntimeError("prefetch: handle has been discarded")
        t = self._restore_new(device, stream, wait=False, cast=None, verify=False)
        self._prefetched = t
        return PrefetchHandle(self, t)

    def _restore_new(self, device, stream, wait, cast, verify, keep_pinned=False):
        dev = self._off._resolve_device(device)
        code = CASTS[cast]
        numel = self.shape.numel()
        scales = None
        if code == 1:
            if self.dtype != torch.bfloat16:
                raise ValueError("fp8_block128 cast needs a bfloat16 tensor")
            out = torch.empty(self.shape, dtype=torch.float8_e4m3fn, device=dev)
            scales = torch.empty((numel + 127) // 128, dtype=torch.float32, device=dev)
        elif code == 2:
            if self.dtype != torch.float32:
                raise ValueError("bf16 cast needs a float32 tensor")
            out = torch.empty(self.shape, dtype=torch.bfloat16, device=dev)
        elif code == 3:
            if self.dtype != torch.bfloat16:
                raise ValueError("fp32 cast needs a bfloat16 tensor")
            out = torch.empty(self.shape, dtype=torch.float32, device=dev)
        else:
            out = torch.empty(self.shape, dtype=self.dtype, device=dev)
        nbytes = self.nbytes if code == 0 else out.numel() * out.element_size()
        ok, msg, bad = self._off._agent.restore(
            self.tensor_id, self.version, out.data_ptr(), nbytes, _stream_handle(stream, dev), bool(wait), code,
            scales.data_ptr() if scales is not None else 0, bool(verify), bool(keep_pinned))
        if not ok:
            raise RuntimeError(f"restore failed: {msg}")
        return (out, scales) if code == 1 else out

    def restore(self, device=None, stream=None, wait: bool = True, cast: Optional[str] = None,
                verify: bool = False, keep_pinned: bool = False):
        """Restore into a NEW tensor (or ``(fp8, scales)`` for fp8 casts)."""
        if self._discarded:
            raise RuntimeError("restore: handle has been discarded")
        if self._prefetched is not None and cast is None:
            out, self._prefetched = self._prefetched, None
            if wait:
                self._off._agent.wait_restored(self.tensor_id, self.version)
            return out
        return self._restore_new(device, stream, wait, cast, verify, keep_pinned)

    def restore_into(self, dst: torch.Tensor, stream=None, wait: bool = True, verify: bool = False) -> torch.Tensor:
        """Restore into an existing tensor's storage (no allocation).

        For aliased flat buffers the cycle is: ``h = off.copy(buf, wait=True)``,
        ``buf.untyped_storage().resize_(0)``, later ``resize_(h.nbytes)`` and
        ``h.restore_into(buf)``; resizing keeps the Storage object so aliases stay valid.
        """
        if self._discarded:
            raise RuntimeError("restore_into: handle has been discarded")
        if not dst.is_contiguous():
            raise RuntimeError("restore_into: dst must be contiguous")
        n = dst.numel() * dst.element_size()
        if n != self.nbytes:
            raise ValueError(f"restore_into: dst has {n} bytes but the offloaded tensor is {self.nbytes} bytes "
                             "(resize the storage to match before restoring)")
        ok, msg, _ = self._off._agent.restore(self.tensor_id, self.version, dst.data_ptr(), n,
                                              _stream_handle(stream, dst.device), bool(wait), 0, 0, bool(verify),
                                              False)
        if not ok:
            raise RuntimeError(f"restore_into failed: {msg}")
        return dst

    def discard(self) -> None:
        """Drop every daemon-side copy of this tensor (pinned and cold)."""
        if self._discarded:
            return
        self._off._agent.discard(self.tensor_id, self.version)
        self._prefetched = None
        self._discarded = True

    def __repr__(self) -> str:
        return (f"OffloadHandle(tensor_id={self.tensor_id}, version={self.version}, name={self.name!r}, "
                f"shape={tuple(self.shape)}, dtype={self.dtype}, nbytes={self.nbytes})")


class PrefetchHandle:
    __slots__ = ("_handle", "_tensor")

    def __init__(self, handle: OffloadHandle, tensor: torch.Tensor):
        self._handle = handle
        self._tensor = tensor

    def wait(self) -> torch.Tensor:
        """Block until the restore copy itself has completed."""
        h = self._handle
        h._off._agent.wait_restored(h.tensor_id, h.version)
        return self._tensor

    @property
    def tensor(self) -> torch.Tensor:
        return self._tensor


class ManagedRecord:
    """A tensor tracked for later eviction."""

    __slots__ = ("_off", "tensor", "name")

    def __init__(self, off, tensor, name):
        self._off = off
        self.tensor = tensor
        self.name = name

    def evict(self, stream=None, invalidate="set_empty", wait=False, allow_views=False, unsafe_autograd=False,
              compact=False) -> OffloadHandle:
        h = self._off.evict(self.tensor, name=self.name, stream=stream, invalidate=invalidate, wait=wait,
                            allow_views=allow_views, unsafe_autograd=unsafe_autograd, compact=compact)
        self.tensor = None
        return h

    def copy(self, stream=None, wait=False) -> OffloadHandle:
        return self._off.copy(self.tensor, name=self.name, stream=stream, wait=wait)


class DedupPolicy:
    __slots__ = ("mode", "creating_policy", "cross_job_dedup")

    def __init__(self, mode: str = "semantic_trusted", creating_policy: str = "wait", cross_job_dedup: bool = False):
        if mode not in DEDUP_MODES:
            raise ValueError(f"mode must be one of {list(DEDUP_MODES)}; got {mode!r}")
        if creating_policy not in ("wait", "duplicate_candidate_on_pressure"):
            raise ValueError("creating_policy must be 'wait' or 'duplicate_candidate_on_pressure'")
        self.mode = mode
        self.creating_policy = creating_policy
        self.cross_job_dedup = bool(cross_job_dedup)

    @property
    def mode_int(self) -> int:
        return DEDUP_MODES[self.mode]

    @property
    def allow_duplicate_candidate(self) -> bool:
        return self.creating_policy == "duplicate_candidate_on_pressure"


class CanonicalKey:
    """Identity of one logical model-state shard at one model version (dp excluded)."""

    __slots__ = ("model_role", "model_version", "param_id", "param_fqn_hash", "param_fqn_debug", "layout",
                 "shape_hash", "stride_hash", "pp_rank", "tp_rank", "ep_rank", "etp_rank", "expert_id",
                 "shard_offset", "shard_nbytes", "dtype")

    def __init__(self, *, model_role, model_version, param_id, param_fqn_hash, param_fqn_debug, layout, shape_hash,
                 stride_hash, pp_rank, tp_rank, ep_rank, etp_rank, expert_id, shard_offset, shard_nbytes, dtype=0):
        self.model_role = int(model_role)
        self.model_version = int(model_version)
        self.param_id = int(param_id)
        self.param_fqn_hash = int(param_fqn_hash)
        self.param_fqn_debug = param_fqn_debug
        self.layout = int(layout)
        self.shape_hash = int(shape_hash)
        self.stride_hash = int(stride_hash)
        self.pp_rank = int(pp_rank)
        self.tp_rank = int(tp_rank)
        self.ep_rank = int(ep_rank)
        self.etp_rank = int(etp_rank)
        self.expert_id = int(expert_id)
        self.shard_offset = int(shard_offset)
        self.shard_nbytes = int(shard_nbytes)
        self.dtype = int(dtype)

    def to_wire(self, job: dict, nbytes: int) -> dict:
        return {"job": job, "model_role": self.model_role, "model_version": self.model_version,
                "param_id": self.param_id, "param_fqn_hash": self.param_fqn_hash,
                "param_fqn_debug": self.param_fqn_debug, "dtype": self.dtype, "layout": self.layout,
                "nbytes": nbytes, "shape_hash": self.shape_hash, "stride_hash": self.stride_hash,
                "pp_rank": self.pp_rank, "tp_rank": self.tp_rank, "ep_rank": self.ep_rank,
                "etp_rank": self.etp_rank, "expert_id": self.expert_id, "shard_offset": self.shard_offset,
                "shard_nbytes": self.shard_nbytes or nbytes}

    def __repr__(self) -> str:
        return (f"CanonicalKey(role={self.model_role}, version={self.model_version}, param_id={self.param_id}, "
                f"fqn={self.param_fqn_debug!r}, pp={self.pp_rank}, tp={self.tp_rank}, ep={self.ep_rank}, "
                f"expert={self.expert_id})")


class CanonicalHandle:
    """Outcome of a canonical evict: the daemon object id and what happened."""

    __slots__ = ("object_id", "action", "action_name", "did_d2h", "attached", "key", "message", "content_hash", "_off")

    def __init__(self, object_id, action, did_d2h, key, message, off=None, content_hash=None):
        self.object_id = int(object_id)
        self.action = int(action)
        self.action_name = ACTION_NAMES.get(int(action), str(action))
        self.did_d2h = bool(did_d2h)
        self.attached = int(action) in (0, 6)
        self.key = key
        self.message = message
        self.content_hash = content_hash
        self._off = off

    def restore_into(self, dst: torch.Tensor, stream=None, wait: bool = True) -> torch.Tensor:
        """Reload this object's bytes into ``dst`` (works for replicas that only attached)."""
        if self._off is None:
            raise RuntimeError("restore_into: handle not bound to a session")
        if not dst.is_contiguous():
            raise RuntimeError("canonical_restore_into: dst must be contiguous")
        ok, msg = self._off._agent.canonical_restore(self.object_id, dst.data_ptr(), dst.numel() * dst.element_size(),
                                                     _stream_handle(stream, dst.device), bool(wait))
        if not ok:
            raise RuntimeError(f"canonical_restore_into failed: {msg}")
        return dst

    def release(self) -> dict:
        """Drop this session's reference; the object is freed after the last holder."""
        if self._off is None:
            raise RuntimeError("release: handle not bound to a session")
        return self._off._release(self.key.model_role, self.key.model_version, self.object_id)

    def __repr__(self) -> str:
        return f"CanonicalHandle(object_id={self.object_id}, action={self.action_name}, did_d2h={self.did_d2h})"


class Off:
    """Session handle yielded by :func:`offload_context`."""

    def __init__(self, agent, device: torch.device, rank: int):
        self._agent = agent
        self._device = device
        self._rank = int(rank)
        self._ids = itertools.count(1)
        self._unsafe_default = False
        self._lock = threading.Lock()
        self.tenant_id = None
        self.job_id = None
        self.launch_epoch = None
        self.job_name = None
        self._dedup_policy = DedupPolicy()
        self.nvlink_options: dict = {}  # the daemon config's `nvlink:` section

    # ---- identity ----
    @property
    def device(self) -> torch.device:
        return self._device

    @property
    def rank(self) -> int:
        return self._rank

    def _next_tensor_id(self) -> int:
        # rank in the top 24 bits, a per-process counter in the low 40 (bit 63 stays clear)
        return ((self._rank & 0x7FFFFF) << 40) | (next(self._ids) & 0xFFFFFFFFFF)

    def _resolve_device(self, device) -> torch.device:
        if device is None:
            return self._device
        if isinstance(device, int):
            return torch.device("cuda", device)
        return torch.device(device)

    def _job(self) -> dict:
        if self.job_id is None:
            raise RuntimeError("no job registered; pass job_name to offload_context()")
        return {"tenant_id": self.tenant_id, "job_id": self.job_id, "launch_epoch": self.launch_epoch,
                "job_name": self.job_name or ""}

    def _raw(self, opcode: int, values: dict) -> dict:
        req, resp = _wire.OPS[opcode]
        return _wire.decode(resp, self._agent.call_raw(opcode, _wire.encode(req, values)))

    # ---- job registration ----
    def _register_job(self, tenant_id: int, job_name: str, scheduler_job_id: int, labels: dict | None = None) -> None:
        labels = labels or {}
        r = self._raw(_wire.Op.REGISTER_JOB, {"tenant_id": tenant_id, "job_name": job_name,
                                              "scheduler_job_id": scheduler_job_id,
                                              "label_keys": list(labels), "label_values": list(labels.values())})
        if not r["ok"]:
            raise RuntimeError(f"register_job failed: {r['message']}")
        j = r["job"]
        self.tenant_id, self.job_id, self.launch_epoch, self.job_name = (
            j["tenant_id"], j["job_id"], j["launch_epoch"], j["job_name"])

    def set_dedup_policy(self, policy: DedupPolicy) -> None:
        self._dedup_policy = policy

    # ---- canonical model state ----
    def canonical_key(self, *, model_role, model_version, param_name, param_id=None, tensor=None, pp_rank=0,
                      tp_rank=0, ep_rank=0, etp_rank=0, expert_id=-1, shape=None, dtype=None, shard_offset=0,
                      shard_nbytes=None) -> CanonicalKey:
        """Build a canonical key; dp rank is deliberately not an argument."""
        if tensor is not None:
            shape = tuple(tensor.shape) if shape is None else tuple(shape)
            stride = tuple(tensor.stride())
            if shard_nbytes is None:
                shard_nbytes = tensor.numel() * tensor.element_size()
            dtype = tensor.dtype if dtype is None else dtype
        else:
            shape = tuple(shape or ())
            stride = ()
        fqn = fnv1a64(param_name.encode("utf-8"))
        return CanonicalKey(model_role=ModelRole.parse(model_role), model_version=int(model_version),
                            param_id=fqn if param_id is None else int(param_id), param_fqn_hash=fqn,
                            param_fqn_debug=param_name, layout=0, shape_hash=hash_ints(shape),
                            stride_hash=hash_ints(stride), pp_rank=pp_rank, tp_rank=tp_rank, ep_rank=ep_rank,
                            etp_rank=etp_rank, expert_id=expert_id, shard_offset=shard_offset,
                            shard_nbytes=int(shard_nbytes or 0), dtype=_SCALAR_TYPE.get(dtype, 0))

    def canonical_evict(self, tensor: torch.Tensor, canonical_key: CanonicalKey, dedup: str = "attach_or_create",
                        destructive: bool = True, stream=None, wait: bool = True, allow_views: bool = False,
                        unsafe_autograd: bool = False, compact: bool = False, local_tensor_id: int = 0,
                        local_version: int = 1, dedup_policy: Optional[DedupPolicy] = None,
                        wait_for_creator: bool = False, timeout_s: float = 600.0) -> CanonicalHandle:
        """Attach-or-create the canonical object of ``tensor``.

        Actions: ATTACHED_EXISTING (no copy), NEED_D2H_CREATE (this rank copies,
        hashing in the same pass), WAIT_FOR_CREATOR (retried here when
        ``wait_for_creator``), DUPLICATE_CANDIDATE, or VERIFIED_BY_DEVICE_HASH
        for ``device_hash_verified`` replicas (hash of the local GPU copy
        compared by the daemon; nothing crosses PCIe).
        """
        src, nbytes, body, cb = self._canonical_request(tensor, canonical_key, dedup, destructive, allow_views,
                                                        unsafe_autograd, compact, local_tensor_id, local_version,
                                                        dedup_policy)
        stream_h = _stream_handle(stream, src.device)
        deadline = time.monotonic() + timeout_s
        while True:
            ok, action, oid, did_d2h, msg, hlo, hhi = self._agent.canonical_evict(
                src.data_ptr(), nbytes, stream_h, bool(destructive), body, cb, bool(wait))
            if ok and action == 2 and wait_for_creator and time.monotonic() < deadline:
                time.sleep(0.002)
                continue
            break
        if not ok:
            raise RuntimeError(f"canonical_evict failed (action={ACTION_NAMES.get(action, action)}): {msg}")
        return CanonicalHandle(oid, action, did_d2h, canonical_key, msg, off=self,
                               content_hash=(hlo, hhi) if (hlo or hhi) else None)

    def _canonical_request(self, tensor, key, dedup, destructive, allow_views, unsafe_autograd, compact,
                           local_tensor_id, local_version, dedup_policy):
        """Source tensor, byte count, encoded RequestCanonicalEvict body and
        invalidate callback of one canonical evict."""
        job = self._job()
        pol = dedup_policy or self._dedup_policy
        mode = 0 if dedup == "disabled" else pol.mode_int
        unsafe = unsafe_autograd or self._unsafe_default
        src = tensor
        if not destructive and tensor.is_contiguous():
            pass  # a copy that leaves the tensor alone reads a contiguous view in place
        elif compact or allow_views:
            src = tensor.clone(memory_format=torch.contiguous_format)
        else:
            _validate_destructive(tensor, unsafe)
        nbytes = src.numel() * src.element_size()
        if key.dtype == 0:
            key.dtype = _SCALAR_TYPE.get(src.dtype, 0)
        body = _wire.encode("RequestCanonicalEvictRequest", {
            "key": key.to_wire(job, nbytes), "local_tensor_id": local_tensor_id, "local_version": local_version,
            "destructive": destructive, "attach_if_exists": True, "create_if_missing": True, "dedup_mode": mode,
            "allow_duplicate_candidate": pol.allow_duplicate_candidate, "alignment": 256})
        cb = _invalidate_callback(tensor) if destructive and not (compact or allow_views) else None
        return src, nbytes, body, cb

    def canonical_evict_batch(self, items: Sequence[Tuple[torch.Tensor, CanonicalKey]],
                              dedup: str = "attach_or_create", destructive: bool = True, stream=None,
                              allow_views: bool = False, unsafe_autograd: bool = False, compact: bool = False,
                              dedup_policy: Optional[DedupPolicy] = None, max_inflight_bytes: int = 0,
                              wait_for_creator: bool = False, timeout_s: float = 600.0) -> List[CanonicalHandle]:
        """``canonical_evict`` of many ``(tensor, key)`` pairs on one stream.

        Every item's attach-or-create round trip and copy are issued before
        the first copy is awaited, so the round trips of later items and the
        commits of earlier ones overlap the copies in flight (at most
        ``max_inflight_bytes`` of copies outstanding; 0 = no limit). The
        outcome of each item is that of ``canonical_evict``; items answered
        WAIT_FOR_CREATOR are retried one by one when ``wait_for_creator``.
        Additive to StateSpectre's API (its sealed versions record one tensor
        per call: python_api/state_spectre/__init__.py canonical_evict).
        """
        if not items:
            return []
        reqs = []
        keep = []
        dev = None
        for tensor, key in items:
            src, nbytes, body, cb = self._canonical_request(tensor, key, dedup, destructive, allow_views,
                                                            unsafe_autograd, compact, 0, 1, dedup_policy)
            dev = dev or src.device
            keep.append(src)
            reqs.append((src.data_ptr(), nbytes, body, cb))
        stream_h = _stream_handle(stream, dev)
        outs = self._agent.canonical_evict_batch(reqs, stream_h, bool(destructive), int(max_inflight_bytes))
        handles = []
        for (tensor, key), (ok, action, oid, did_d2h, msg, hlo, hhi) in zip(items, outs):
            if ok and action == 2 and wait_for_creator:
                handles.append(self.canonical_evict(tensor, key, dedup=dedup, destructive=destructive, stream=stream,
                                                    allow_views=allow_views, unsafe_autograd=unsafe_autograd,
                                                    compact=compact, dedup_policy=dedup_policy,
                                                    wait_for_creator=True, timeout_s=timeout_s))
                continue
            if not ok:
                raise RuntimeError(f"canonical_evict failed (action={ACTION_NAMES.get(action, action)}): {msg}")
            handles.append(CanonicalHandle(oid, action, did_d2h, key, msg, off=self,
                                           content_hash=(hlo, hhi) if (hlo or hhi) else None))
        del keep
        return handles

    def seal_model_version(self, model_role, model_version: int, fail_if_missing: bool = True,
                           promote: bool = False, expected_param_ids: Sequence[int] = ()) -> dict:
        r = self._raw(_wire.Op.SEAL_MODEL_VERSION, {
            "job": self._job(), "model_role": ModelRole.parse(model_role), "model_version": int(model_version),
            "fail_if_missing": fail_if_missing, "expected_param_ids": list(expected_param_ids), "promote": promote})
        if not r["ok"]:
            raise RuntimeError(f"seal_model_version failed: {r['message']}")
        return {"state": r["state"], "tensor_count": r["tensor_count"], "total_nbytes": r["total_nbytes"],
                "manifest_hash": (r["manifest_hash_lo"], r["manifest_hash_hi"]), "message": r["message"]}

    def promote_rollout_version(self, model_version: int, fail_if_missing: bool = True) -> dict:
        return self.seal_model_version(ModelRole.POLICY_ROLLOUT, model_version, fail_if_missing=fail_if_missing,
                                       promote=True)

    def drop_canonical_version(self, model_role, model_version: int) -> dict:
        r = self._raw(_wire.Op.DROP_CANONICAL_VERSION, {"job": self._job(), "model_role": ModelRole.parse(model_role),
                                                         "model_version": int(model_version)})
        if not r["ok"]:
            raise RuntimeError(f"drop_canonical_version failed: {r['message']}")
        return {"dropped": r["dropped_count"], "skipped_inflight": r["skipped_inflight"],
                "bytes_freed": r["bytes_freed"], "message": r["message"]}

    def carry_forward_version(self, model_role, from_version: int, to_version: int,
                              param_ids: Optional[Sequence[int]] = None, *, pp_rank: Optional[int] = None,
                              tp_rank: Optional[int] = None, ep_rank: int = 0, etp_rank: int = 0,
                              expert_id: int = -1) -> dict:
        """Make `to_version` objects for unchanged params that share the
        storage (and content hash) of `from_version`'s objects; nothing is
        copied. `param_ids=None` carries every object of `from_version`.
        Keys already present at `to_version` are left alone (`existing`).
        With `tp_rank` / `pp_rank` only that partition's objects are carried
        (a TP rank carrying its own shards); without, every partition of each
        listed parameter is.
        (No reference counterpart: the reference re-evicts every object of
        each version, python_api/state_spectre/__init__.py:575.)"""
        shard = tp_rank is not None or pp_rank is not None
        r = self._raw(_wire.Op.CARRY_FORWARD, {
            "rank_id": 0, "rank_epoch": 0, "job": self._job(), "model_role": ModelRole.parse(model_role),
            "from_version": int(from_version), "to_version": int(to_version),
            "param_ids": [int(p) for p in (param_ids or [])], "shard": shard, "pp_rank": int(pp_rank or 0),
            "tp_rank": int(tp_rank or 0), "ep_rank": int(ep_rank), "etp_rank": int(etp_rank),
            "expert_id": int(expert_id)})
        if not r["ok"]:
            raise RuntimeError(f"carry_forward failed: {r['message']}")
        return {"carried": r["carried_count"], "existing": r["existing_count"], "missing": r["missing_count"],
                "bytes_shared": r["bytes_shared"]}

    def _release(self, role: int, version: int, object_id: int) -> dict:
        r = self._raw(_wire.Op.RELEASE_CANONICAL, {
            "rank_id": self._agent.rank_id(), "rank_epoch": self._agent.rank_epoch(), "job": self._job(),
            "model_role": role, "model_version": int(version), "object_id": int(object_id)})
        if not r["ok"]:
            raise RuntimeError(f"release_canonical failed: {r['message']}")
        return {"released": r["released_count"], "freed": r["freed_count"], "bytes_freed": r["bytes_freed"],
                "message": r["message"]}

    def release_canonical_version(self, model_role, model_version: int) -> dict:
        return self._release(ModelRole.parse(model_role), model_version, 0)

    def get_manifest(self, model_role, model_version: int, **flt) -> dict:
        f = {}
        for axis in ("pp", "tp", "ep", "etp"):
            if f"{axis}_rank" in flt:
                f[f"{axis}_present"] = True
                f[f"{axis}_rank"] = flt[f"{axis}_rank"]
        if "expert_id" in flt:
            f["expert_present"] = True
            f["expert_id"] = flt["expert_id"]
        r = self._raw(_wire.Op.GET_MANIFEST, {"job": self._job(), "model_role": ModelRole.parse(model_role),
                                              "model_version": int(model_version), "filter": f})
        if not r["ok"]:
            raise RuntimeError(f"get_manifest failed: {r['message']}")
        return r

    def export_manifest(self, model_role, model_version: int, path: str) -> dict:
        """Write a sealed manifest in the fixed ABI record format (header + entries)."""
        r = self._raw(_wire.Op.EXPORT_MANIFEST, {"job": self._job(), "model_role": ModelRole.parse(model_role),
                                                 "model_version": int(model_version), "path": path})
        if not r["ok"]:
            raise RuntimeError(f"export_manifest failed: {r['message']}")
        return r

    def job_stats(self) -> List[dict]:
        return self._raw(_wire.Op.GET_JOB_STATS, {"all_tenants": True})["jobs"]

    def daemon_stats(self) -> dict:
        r = self._raw(_wire.Op.GET_STATS, {"rank_id": 0xFFFFFFFF})
        return {e["key"]: e["value"] for e in r["stats"]}

    # ---- kernel timing (device-side %globaltimer stamps) ----
    def enable_kernel_timing(self, capacity: int = 4096) -> None:
        """Stamp every transfer/hash/push kernel launched on this session's GPU
        (also ``offload_context(kernel_timing=True)`` or ``kernels.timing`` in
        the daemon config)."""
        if self._device.type == "cuda":
            native().kernel_timing_enable(self._device.index, int(capacity))

    def kernel_timings(self, since: int = 0):
        """(records, next): finished launches with sequence >= ``since``; each
        record has ``kernel``, ``bytes``, ``ns`` (first CTA start to last CTA
        end, measured on the device) and ``seq``."""
        if self._device.type != "cuda":
            return [], 0
        return native().kernel_timings(self._device.index, int(since))

    def kernel_profile(self, since: int = 0) -> dict:
        """Per kernel: launches, total device ms, bytes and median GB/s."""
        recs, _ = self.kernel_timings(since)
        out: dict = {}
        for r in recs:
            e = out.setdefault(r["kernel"], {"launches": 0, "ms": 0.0, "bytes": 0, "_gbs": []})
            e["launches"] += 1
            e["ms"] += r["ns"] / 1e6
            e["bytes"] += r["bytes"]
            if r["ns"] > 0:
                e["_gbs"].append(r["bytes"] / r["ns"])
        for e in out.values():
            g = sorted(e.pop("_gbs"))
            e["median_gbs"] = round(g[len(g) // 2], 3) if g else None
            e["ms"] = round(e["ms"], 4)
        return out

    # ---- v1 offload ----
    @staticmethod
    def _invalidate_to_flags(invalidate) -> bool:
        if invalidate in (None, "none", "off", False):
            return False
        if invalidate in ("set_empty", "zero", "empty"):
            return True
        raise ValueError(f"invalidate must be one of 'set_empty', 'zero', or None; got {invalidate!r}")

    def _check_device(self, t: torch.Tensor) -> None:
        if self._device.type == "cpu":
            if t.device.type != "cpu":
                raise RuntimeError("evict: this session serves CPU tensors (device='cpu')")
        elif t.device.type != "cuda":
            raise RuntimeError("evict: tensor must be a CUDA tensor (open the session with device='cpu' for CPU tensors)")

    def _evict_impl(self, tensor, name, stream, destructive, allow_views, unsafe_autograd, compact, wait,
                    tensor_id=0, version=0) -> OffloadHandle:
        if tensor is None:
            raise RuntimeError("evict: tensor is None (already evicted/consumed?)")
        self._check_device(tensor)
        shape, stride, dtype = tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype
        unsafe = unsafe_autograd or self._unsafe_default
        if compact or allow_views:
            src = tensor.clone(memory_format=torch.contiguous_format)
            cb = None  # the clone is dropped after the copy; the caller's base storage stays
            keep = src
        else:
            _validate_destructive(tensor, unsafe) if destructive else None
            src = tensor
            cb = _invalidate_callback(tensor) if destructive else None
            keep = None
        if keep is not None:
            # Keep the clone alive until the copy has landed.
            def cb(keep=keep):  # noqa: F811
                del keep
        nbytes = src.numel() * src.element_size()
        tid = int(tensor_id) or self._next_tensor_id()
        ver = int(version) or 1
        # bf16 and fp32 payloads may travel coded (zbf16 / zf32, lossless; the
        # agent decides per object)
        hint = _FMT_HINTS.get(src.dtype, 0)
        ok, msg, _lease, _slot, _lo, _hi, coded = self._agent.evict(
            src.data_ptr(), nbytes, _stream_handle(stream, src.device), bool(destructive), tid, ver, name or "",
            cb, bool(wait), hint)
        if not ok:
            raise RuntimeError(f"evict failed: {msg}")
        h = OffloadHandle(self, tid, ver, name, shape, stride, dtype, tensor.device, nbytes)
        h.coded = bool(coded)
        return h

    def evict(self, tensor, name=None, stream=None, invalidate="set_empty", wait=False, allow_views=False,
              unsafe_autograd=False, compact=False, tensor_id: int = 0, version: int = 0) -> OffloadHandle:
        """Destructive eviction: copy to pinned memory, then release the tensor's storage."""
        return self._evict_impl(tensor, name, stream, self._invalidate_to_flags(invalidate), allow_views,
                                unsafe_autograd, compact, wait, tensor_id, version)

    def copy(self, tensor, name=None, stream=None, wait=False, allow_views=False, compact=False,
             tensor_id: int = 0, version: int = 0) -> OffloadHandle:
        """Non-destructive copy: the tensor stays valid."""
        return self._evict_impl(tensor, name, stream, False, allow_views, False, compact, wait, tensor_id, version)

    def manage(self, tensor, name=None) -> ManagedRecord:
        return ManagedRecord(self, tensor, name)

    def evict_many(self, tensors, names=None, stream=None, invalidate="set_empty", require_own_storage=True,
                   unsafe_autograd=False) -> List[OffloadHandle]:
        tensors = list(tensors)
        if names is not None and len(list(names)) != len(tensors):
            raise ValueError("evict_many: len(names) must match len(tensors)")
        names = list(names) if names is not None else [None] * len(tensors)
        destructive = self._invalidate_to_flags(invalidate)
        return [self._evict_impl(t, n, stream, destructive, not require_own_storage, unsafe_autograd,
                                 not require_own_storage, False) for t, n in zip(tensors, names)]

    def discard_batch(self, handles: Sequence["OffloadHandle"]) -> None:
        """``h.discard()`` for many handles with one daemon round trip."""
        todo = [h for h in handles if not h._discarded]
        if not todo:
            return
        self._agent.discard_batch([(h.tensor_id, h.version) for h in todo])
        for h in todo:
            h._prefetched = None
            h._discarded = True

    def evict_batch(self, tensors: Sequence[torch.Tensor], stream=None, wait: bool = True,
                    versions: Optional[Sequence[int]] = None) -> List[OffloadHandle]:
        """Non-destructive copy of many contiguous tensors with one reservation round trip.

        Items the daemon answers as blocked (pinned window full) are retried,
        after the batch's earlier copies are published so they can drain, for
        up to the session's ``blocked_wait_ms``."""
        tensors = list(tensors)
        if not tensors:
            return []
        for t in tensors:
            self._check_device(t)
            if not t.is_contiguous():
                raise RuntimeError("evict_batch: tensors must be contiguous")
        ids = [self._next_tensor_id() for _ in tensors]
        vers = list(versions) if versions is not None else [1] * len(tensors)
        items = [(t.data_ptr(), t.numel() * t.element_size(), i, v, _FMT_HINTS.get(t.dtype, 0))
                 for t, i, v in zip(tensors, ids, vers)]
        res = self._agent.evict_batch(items, _stream_handle(stream, tensors[0].device), bool(wait))
        out = []
        for t, (ok, msg, coded), i, v in zip(tensors, res, ids, vers):
            if not ok:
                raise RuntimeError(f"evict_batch failed for tensor {i}: {msg}")
            h = OffloadHandle(self, i, v, None, tuple(t.shape), tuple(t.stride()), t.dtype, t.device,
                              t.numel() * t.element_size())
            h.coded = bool(coded)
            out.append(h)
        return out

    def restore_batch(self, handles: Sequence[OffloadHandle], dsts: Optional[Sequence[torch.Tensor]] = None,
                      stream=None, wait: bool = True) -> List[torch.Tensor]:
        """Restore many handles with batched prefetch round trips."""
        handles = list(handles)
        if dsts is None:
            dsts = [torch.empty(h.shape, dtype=h.dtype, device=self._device) for h in handles]
        items = [(d.data_ptr(), h.nbytes, h.tensor_id, h.version) for h, d in zip(handles, dsts)]
        res = self._agent.restore_batch(items, _stream_handle(stream, self._device), bool(wait))
        for h, (ok, msg) in zip(handles, res):
            if not ok:
                raise RuntimeError(f"restore_batch failed for tensor {h.tensor_id}: {msg}")
        return list(dsts)

    def wait(self, handles: Iterable[OffloadHandle]) -> None:
        for h in handles:
            h.wait_offloaded()

    def restore_many(self, handles, device=None, stream=None, wait=True) -> List[torch.Tensor]:
        return [h.restore(device=device, stream=stream, wait=wait) for h in handles]

    def hash_tensor(self, t: torch.Tensor, stream=None) -> tuple:
        """ssh128 (lo, hi) of a tensor's bytes, computed on its device."""
        if not t.is_contiguous():
            t = t.contiguous()
        return self._agent.hash_buffer(t.data_ptr(), t.numel() * t.element_size(), _stream_handle(stream, t.device))

    # ---- debugging ----
    def summary(self) -> str:
        return self._agent.summary_string()

    def summary_dict(self) -> dict:
        return self._agent.stats()

    def assert_no_inflight(self) -> None:
        self._agent.assert_no_inflight()

    def synchronize(self) -> None:
        """Wait until every asynchronous transfer of this session has retired."""
        self._agent.synchronize()

    def slot_table(self, limit: int = 20) -> str:
        s = self._agent.stats()
        d = self.daemon_stats()
        return "\n".join([
            "slot_table:",
            f"  num_slots={s['num_slots']} used={d.get('used_slots', 0)} slot_bytes={d.get('slot_bytes', 0)} "
            f"limit={limit}",
            f"  registered_pinned_bytes={s['registered_pinned_bytes']}",
            f"  inflight_d2h_bytes={s['inflight_d2h_bytes']} inflight_h2d_bytes={s['inflight_h2d_bytes']}",
            f"  evict_count={s['evict_count']} restore_count={s['restore_count']} "
            f"d2h_done={s['d2h_completed']} h2d_done={s['h2d_completed']}",
        ])

    @contextlib.contextmanager
    def unsafe_destructive_mode(self):
        prev = self._unsafe_default
        self._unsafe_default = True
        try:
            yield self
        finally:
            self._unsafe_default = prev

    @contextlib.contextmanager
    def trace(self, path: str):
        """Write a Chrome-trace JSON of session counters around a block; with
        kernel timing on (``enable_kernel_timing``), every stamped kernel of
        the block is a complete event on a GPU track (device timestamps)."""
        t0 = time.time_ns()
        before = self._agent.stats()
        _, stamp0 = self.kernel_timings()
        ev = [{"name": "offload_session", "ph": "B", "ts": t0 / 1000.0, "pid": before["rank_id"],
               "tid": max(before["gpu_id"], 0), "args": before}]
        try:
            yield self
        finally:
            t1 = time.time_ns()
            after = self._agent.stats()
            ev.append({"name": "offload_session", "ph": "E", "ts": t1 / 1000.0, "pid": after["rank_id"],
                       "tid": max(after["gpu_id"], 0), "args": after})
            ev.append({"name": "delta", "ph": "i", "s": "g", "ts": t1 / 1000.0, "pid": after["rank_id"],
                       "tid": max(after["gpu_id"], 0),
                       "args": {k: after[k] - before[k] for k in ("d2h_completed", "h2d_completed", "evict_count",
                                                                  "restore_count", "d2h_bytes", "h2d_bytes",
                                                                  "kernel_launches", "rpc_count")}})
            recs, _ = self.kernel_timings(stamp0)
            for r in recs:
                ev.append({"name": r["kernel"], "ph": "X", "ts": r["t0"] / 1000.0, "dur": r["ns"] / 1000.0,
                           "pid": f"gpu{max(after['gpu_id'], 0)}", "tid": "kernels",
                           "args": {"bytes": r["bytes"], "GB/s": round(r["bytes"] / max(r["ns"], 1), 3),
                                    "seq": r["seq"]}})
            with open(path, "w") as f:
                json.dump({"traceEvents": ev, "displayTimeUnit": "ms"}, f)


_LIVE_SESSIONS: "weakref.WeakSet" = None  # type: ignore[assignment]


def _close_live_sessions() -> None:
    """atexit: stop agent threads before the interpreter finalizes, so no
    native thread tries to take the GIL of a dying interpreter."""
    for s in list(_LIVE_SESSIONS or ()):
        try:
            s.close()
        except Exception:  # noqa: BLE001
            pass


def _track(session) -> None:
    global _LIVE_SESSIONS
    if _LIVE_SESSIONS is None:
        import atexit
        import weakref

        _LIVE_SESSIONS = weakref.WeakSet()
        atexit.register(_close_live_sessions)
    _LIVE_SESSIONS.add(session)


def _as_bool(v: str) -> bool:
    t = str(v).strip().lower()
    if t in ("1", "true", "yes", "on"):
        return True
    if t in ("0", "false", "no", "off"):
        return False
    raise ValueError(v)


# `kernels:` keys of the daemon config -> agent option (name, parser)
_AGENT_OPTION_KEYS = {
    "kernels.evict_ctas": ("evict_ctas", int),
    "kernels.restore_ctas": ("restore_ctas", int),
    "kernels.hash_ctas": ("hash_ctas", int),
    "kernels.stage_ctas": ("stage_ctas", int),
    "kernels.stage_depth": ("stage_depth", int),
    "kernels.stage_piece_chunks": ("stage_piece_chunks", int),
    "kernels.engine": ("engine", str),
    "kernels.uncoded": ("uncoded", str),
    "kernels.coded_restore": ("coded_restore", str),
    "kernels.coded_evict": ("coded_evict", str),
    "kernels.compress": ("compress", _as_bool),
    "kernels.compress_canonical": ("compress_canonical", _as_bool),
    "kernels.compress_min_mb": ("compress_min_bytes", lambda v: int(float(v) * (1 << 20))),
    "kernels.batch_group_mb": ("batch_group_bytes", lambda v: int(float(v) * (1 << 20))),
    "kernels.timing": ("kernel_timing", _as_bool),
    "kernels.stream_priority": ("stream_priority", int),
    "kernels.host_hash_max_kb": ("host_hash_max_bytes", lambda v: int(float(v) * 1024)),
}


def _daemon_agent_options(path: str, rank: int, gpu: int) -> Optional[dict]:
    """The daemon's forwarded ``kernels:`` / ``nvlink:`` settings (empty when
    the daemon does not offer them; None when it left the request unanswered,
    as StateSpectre's own offloadd does with every opcode it does not know)."""
    if not path.startswith("tcp://") and not os.path.exists(path):
        return {}  # no daemon there; the session's own connect reports it
    try:
        # StateSpectre's own offloadd logs an unknown opcode and sends nothing back
        conn = native().RawConn(path, 5000, 5000)
    except Exception:  # noqa: BLE001 - the agent reports connection errors itself
        return {}
    try:
        _, body, _ = conn.call(_wire.Op.GET_AGENT_OPTIONS,
                               _wire.encode("GetAgentOptionsRequest", {"rank_id": rank, "gpu_id": gpu}))
        r = _wire.decode("GetAgentOptionsResponse", body)
        return {e["key"]: e["value"] for e in r["options"]} if r["ok"] else {}
    except Exception:  # noqa: BLE001 - no answer within the reply timeout
        return None
    finally:
        conn.close()


class _OffloadSession:
    """Context manager returned by :func:`offload_context` (a plain object, so a
    session used without ``with`` is closed only explicitly)."""

    def __init__(self, *, daemon_addr, device, rank, local_rank, world_rank, numa_node, register_policy,
                 registration_chunk_mb, eager_register, job_name, tenant_id, scheduler_job_id, dedup_policy,
                 job_labels=None, **agent_opts):
        dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", 0)
        self._device = dev
        path = daemon_addr[len("unix://"):] if daemon_addr.startswith("unix://") else daemon_addr
        opts = {"socket_path": path, "device": dev.index if dev.type == "cuda" else -1, "rank_id": int(rank),
                "local_rank": int(local_rank), "world_rank": int(world_rank), "numa_node": int(numa_node),
                "eager_register": bool(eager_register or register_policy in ("eager", "eager_all"))}
        daemon_opts = _daemon_agent_options(path, int(rank), dev.index if dev.type == "cuda" else 0)
        if daemon_opts is None:
            # StateSpectre's own offloadd: speak its opcodes 1-30 only
            opts["v1_only"] = True
            daemon_opts = {}
        for k, v in daemon_opts.items():
            if k in _AGENT_OPTION_KEYS and _AGENT_OPTION_KEYS[k][0] not in agent_opts:
                name, conv = _AGENT_OPTION_KEYS[k]
                try:
                    opts[name] = conv(v)
                except ValueError:
                    pass
        opts.update(agent_opts)
        self._agent = native().Agent(opts)
        off = Off(self._agent, dev, rank)
        off.nvlink_options = {k[len("nvlink."):]: v for k, v in daemon_opts.items() if k.startswith("nvlink.")}
        if dedup_policy is not None:
            off.set_dedup_policy(dedup_policy)
        if job_name is not None:
            off._register_job(tenant_id, job_name, 0 if scheduler_job_id is None else int(scheduler_job_id),
                              job_labels)
        self._off = off
        self._closed = False
        _track(self)

    def __enter__(self) -> Off:
        return self._off

    @property
    def off(self) -> Off:
        return self._off

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        if self._device.type == "cuda":
            try:
                torch.cuda.synchronize(self._device)
            except Exception:  # noqa: BLE001
                pass
        self._agent.close()

    def __exit__(self, *exc):
        self.close()
        return False


def offload_context(daemon_addr: str = "unix:///tmp/state_spectre.sock",
                    device: Union[str, int, torch.device] = "cuda:0", rank: int = 0, local_rank: int = 0,
                    world_rank: int = 0, numa_node: int = -1, register_policy: str = "lazy_chunked",
                    registration_chunk_mb: int = 512, target_tier: str = "pageable_then_nvme",
                    invalidate_mode: str = "set_empty", eager_register: bool = False,
                    job_name: Optional[str] = None, tenant_id: int = 0, scheduler_job_id=None,
                    dedup_policy: Optional[DedupPolicy] = None, job_labels: Optional[dict] = None,
                    **agent_opts) -> _OffloadSession:
    """Open an offload session with the node daemon.

    Maps the daemon's arenas, registers them with CUDA (lazily or eagerly) and
    starts the completion and heartbeat threads. With ``job_name`` the session
    registers a job and canonical evicts become available. Extra keyword
    arguments tune the agent (``engine``, ``evict_ctas``, ``restore_ctas``,
    ``hash_on_evict``, ``use_ring``, ``fast_submit``, ...). ``target_tier`` and
    ``invalidate_mode`` are accepted for compatibility; tiering policy lives in
    the daemon config.
    """
    return _OffloadSession(daemon_addr=daemon_addr, device=device, rank=rank, local_rank=local_rank,
                           world_rank=world_rank, numa_node=numa_node, register_policy=register_policy,
                           registration_chunk_mb=registration_chunk_mb, eager_register=eager_register,
                           job_name=job_name, tenant_id=tenant_id, scheduler_job_id=scheduler_job_id,
                           dedup_policy=dedup_policy, job_labels=job_labels, **agent_opts)
