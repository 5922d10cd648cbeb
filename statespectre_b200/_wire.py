"""Pure-Python mirror of the control-plane wire schema.

Every message is a list of ``(field, type)`` pairs in wire order; one generic
encoder/decoder walks it. The field lists mirror ``csrc/include/ofld/protocol.h``
(``fields()`` overloads) and, for opcodes 1-30, StateSpectre's codec
(reference: src/common/wire.cpp:66-412, wire_v2.cpp:11-438), so a Python
client speaks the daemon's protocol without the native module. Types:
``bool`` (1 byte), ``u8/u16/u32/u64`` little-endian, ``i32`` (two's
complement u32), ``str`` (u32 length + UTF-8), ``[T]`` (u32 count + items) and
nested message names.

Frame: ``[u32 magic 'OFRP'][u16 opcode][u16 flags][u32 len][body]``.
"""

from __future__ import annotations

import socket
import struct
from typing import Any, Dict, List, Optional, Tuple

RPC_MAGIC = 0x4F465250
FRAME_HEADER = struct.Struct("<IHHI")
EXPORT_MAGIC = 0x4F464558
EXPORT_HEADER = struct.Struct("<IIQQQQ")
EXPORT_HEADER_SIZE = EXPORT_HEADER.size  # 40
MAX_PAYLOAD = 256 << 20


class Op:
    REGISTER_RANK = 1
    HEARTBEAT = 2
    REQUEST_OFFLOAD = 3
    MARK_D2H_SUBMITTED = 4
    MARK_D2H_COMPLETE = 5
    REQUEST_PREFETCH = 6
    MARK_H2D_SUBMITTED = 7
    MARK_H2D_COMPLETE = 8
    RELEASE_LEASE = 9
    QUERY_LOCATION = 10
    BATCH_COMPLETE = 11
    SHUTDOWN = 12
    GET_STATS = 13
    REGISTER_JOB = 20
    REQUEST_CANONICAL_EVICT = 21
    COMMIT_CANONICAL_OBJECT = 22
    SEAL_MODEL_VERSION = 23
    GET_LATEST_SEALED_VERSION = 24
    GET_MANIFEST = 25
    PULL_TENSOR = 26
    REQUEST_CANONICAL_RESTORE = 27
    RELEASE_CANONICAL_RESTORE = 28
    DROP_CANONICAL_VERSION = 29
    RELEASE_CANONICAL = 30
    BATCH_REQUEST_OFFLOAD = 40
    BATCH_REQUEST_PREFETCH = 41
    PUBLISH_PEER_BUFFER = 42
    LOOKUP_PEER_BUFFER = 43
    GET_JOB_STATS = 44
    EXPORT_MANIFEST = 45
    DISCARD_TENSOR = 46
    CARRY_FORWARD = 47
    GET_AGENT_OPTIONS = 48
    BATCH_DISCARD_TENSOR = 49
    SET_RUN_FORMAT = 50


# Backward-compatible names used by rollout engines.
OP_GET_LATEST_SEALED_VERSION = Op.GET_LATEST_SEALED_VERSION
OP_GET_MANIFEST = Op.GET_MANIFEST
OP_PULL_TENSOR = Op.PULL_TENSOR

TK_TCP = 1
TK_FILE = 2
TK_LIBFABRIC_SEND = 3
TK_RDMA_READ = 4
TK_RDMA_WRITE = 5

S = "str"
STATUS = [("ok", "bool"), ("message", S)]
TRANSFER_MARK = [("rank_id", "u32"), ("rank_epoch", "u64"), ("lease_id", "u64"), ("tensor_id", "u64"),
                 ("version", "u64"), ("slot_id", "u32"), ("seq", "u64"), ("timestamp_ns", "u64")]

SCHEMA: Dict[str, List[Tuple[str, Any]]] = {
    "Status": STATUS,
    "ArenaFd": [("arena_id", "u64"), ("numa_node", "u32"), ("kind", "u32"), ("size", "u64"),
                ("base_offset", "u64"), ("preferred_gpu", "u32"), ("flags", "u64"), ("fd_index", "u32"),
                ("registration_granularity", "u32"), ("allocation_granularity", "u32")],
    "RegisterRankRequest": [("rank_id", "u32"), ("local_rank", "u32"), ("world_rank", "u32"), ("gpu_id", "u32"),
                            ("numa_node", "u32"), ("pid", "u64"), ("capabilities", "u64")],
    "RegisterRankResponse": STATUS + [("rank_epoch", "u64"), ("control_generation", "u64"),
                                      ("arenas", ["ArenaFd"]), ("control_fd_index", "u32"),
                                      ("control_size", "u64"), ("num_slots", "u32"), ("ring_index", "u32")],
    "HeartbeatRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("timestamp_ns", "u64")],
    "RequestOffloadRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("tensor_id", "u64"), ("version", "u64"),
                              ("nbytes", "u64"), ("gpu_id", "u32"), ("numa_node", "u32"), ("alignment", "u32"),
                              ("priority", "u32"), ("flags", "u64"), ("debug_name", S)],
    "RequestOffloadResponse": STATUS + [("lease_id", "u64"), ("slot_id", "u32"), ("arena_id", "u64"),
                                        ("arena_offset", "u64"), ("capacity", "u64"), ("state", "u32"),
                                        ("blocked", "bool")],
    "TransferMark": TRANSFER_MARK,
    "MarkD2HCompleteResponse": STATUS + [("latest_version", "bool"), ("drain_enqueued", "bool")],
    "RequestPrefetchRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("tensor_id", "u64"), ("version", "u64"),
                               ("nbytes", "u64"), ("gpu_id", "u32"), ("numa_node", "u32"), ("priority", "u32"),
                               ("flags", "u64")],
    "RequestPrefetchResponse": STATUS + [("lease_id", "u64"), ("slot_id", "u32"), ("arena_id", "u64"),
                                         ("arena_offset", "u64"), ("nbytes", "u64"), ("state", "u32"),
                                         ("ready", "bool"), ("version", "u64")],
    "MarkH2DCompleteRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("lease_id", "u64"), ("tensor_id", "u64"),
                               ("version", "u64"), ("slot_id", "u32"), ("keep_pinned", "bool"), ("seq", "u64"),
                               ("timestamp_ns", "u64")],
    "ReleaseLeaseRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("lease_id", "u64"), ("slot_id", "u32"),
                            ("reason", S)],
    "LocationQueryRequest": [("tensor_id", "u64"), ("version", "u64")],
    "LocationQueryResponse": STATUS + [("location_kind", "u32"), ("slot_id", "u32"), ("nbytes", "u64"),
                                       ("version", "u64")],
    "BatchCompletion": [("event_type", "u32"), ("lease_id", "u64"), ("tensor_id", "u64"), ("version", "u64"),
                        ("slot_id", "u32"), ("seq", "u64"), ("timestamp_ns", "u64"), ("keep_pinned", "bool")],
    "BatchCompleteRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("completions", ["BatchCompletion"])],
    "BatchCompleteResponse": STATUS + [("accepted", "u32"), ("rejected", "u32")],
    "GetStatsRequest": [("rank_id", "u32")],
    "StatEntry": [("key", S), ("value", "u64")],
    "GetStatsResponse": STATUS + [("stats", ["StatEntry"])],
    "ShutdownRequest": [("token", "u64")],
    # ---- canonical v2 ----
    "JobKey": [("tenant_id", "u64"), ("job_id", "u64"), ("launch_epoch", "u64"), ("job_name", S)],
    "RegisterJobRequest": [("tenant_id", "u64"), ("job_name", S), ("scheduler_job_id", "u64"),
                           ("label_keys", [S]), ("label_values", [S])],
    "RegisterJobResponse": STATUS + [("job", "JobKey"), ("control_generation", "u64")],
    "CanonicalKey": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"), ("param_id", "u64"),
                     ("param_fqn_hash", "u64"), ("param_fqn_debug", S), ("dtype", "u32"), ("layout", "u32"),
                     ("nbytes", "u64"), ("shape_hash", "u64"), ("stride_hash", "u64"), ("pp_rank", "u32"),
                     ("tp_rank", "u32"), ("ep_rank", "u32"), ("etp_rank", "u32"), ("expert_id", "i32"),
                     ("shard_offset", "u64"), ("shard_nbytes", "u64")],
    "RequestCanonicalEvictRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("key", "CanonicalKey"),
                                     ("local_tensor_id", "u64"), ("local_version", "u64"), ("destructive", "bool"),
                                     ("attach_if_exists", "bool"), ("create_if_missing", "bool"),
                                     ("dedup_mode", "u32"), ("allow_duplicate_candidate", "bool"),
                                     ("alignment", "u32"), ("priority", "u32"), ("gpu_id", "u32"),
                                     ("numa_node", "u32")],
    "RequestCanonicalEvictResponse": STATUS + [("action", "u32"), ("object_id", "u64"), ("lease_id", "u64"),
                                               ("slot_id", "u32"), ("arena_id", "u64"), ("arena_offset", "u64"),
                                               ("capacity", "u64"), ("synthetic_tid", "u64")],
    "CommitCanonicalObjectRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("object_id", "u64"),
                                     ("lease_id", "u64"), ("slot_id", "u32"), ("content_hash_lo", "u64"),
                                     ("content_hash_hi", "u64")],
    "CommitCanonicalObjectResponse": STATUS + [("object_id", "u64"), ("won", "bool")],
    "SealModelVersionRequest": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"),
                                ("fail_if_missing", "bool"), ("expected_param_ids", ["u64"]), ("promote", "bool")],
    "SealModelVersionResponse": STATUS + [("state", "u32"), ("tensor_count", "u64"), ("total_nbytes", "u64"),
                                          ("manifest_hash_lo", "u64"), ("manifest_hash_hi", "u64")],
    "GetLatestSealedVersionRequest": [("job", "JobKey"), ("model_role", "u32")],
    "GetLatestSealedVersionResponse": STATUS + [("found", "bool"), ("model_version", "u64")],
    "ManifestFilter": [("pp_present", "bool"), ("pp_rank", "u32"), ("tp_present", "bool"), ("tp_rank", "u32"),
                       ("ep_present", "bool"), ("ep_rank", "u32"), ("etp_present", "bool"), ("etp_rank", "u32"),
                       ("expert_present", "bool"), ("expert_id", "i32")],
    "GetManifestRequest": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"),
                           ("filter", "ManifestFilter")],
    "TensorManifestEntry": [("key", "CanonicalKey"), ("object_id", "u64"), ("nbytes", "u64"),
                            ("content_hash_lo", "u64"), ("content_hash_hi", "u64"), ("location_hint", S)],
    "GetManifestResponse": STATUS + [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"),
                                     ("state", "u32"), ("tensors", ["TensorManifestEntry"])],
    "PullTensorRequest": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"), ("object_id", "u64"),
                          ("transport", "u32"), ("target_descriptor", S)],
    "PullTensorResponse": STATUS + [("object_id", "u64"), ("nbytes", "u64"), ("transport", "u32"),
                                    ("content_hash_lo", "u64"), ("content_hash_hi", "u64"),
                                    ("transport_metadata", S)],
    "RequestCanonicalRestoreRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("object_id", "u64"),
                                       ("gpu_id", "u32"), ("numa_node", "u32")],
    "RequestCanonicalRestoreResponse": STATUS + [("retriable", "bool"), ("object_id", "u64"), ("nbytes", "u64"),
                                                 ("arena_id", "u64"), ("arena_offset", "u64")],
    "ReleaseCanonicalRestoreRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("object_id", "u64")],
    "DropCanonicalVersionRequest": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64")],
    "DropCanonicalVersionResponse": STATUS + [("dropped_count", "u64"), ("skipped_inflight", "u64"),
                                              ("bytes_freed", "u64")],
    "ReleaseCanonicalRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("job", "JobKey"), ("model_role", "u32"),
                                ("model_version", "u64"), ("object_id", "u64")],
    "ReleaseCanonicalResponse": STATUS + [("released_count", "u64"), ("freed_count", "u64"), ("bytes_freed", "u64")],
    # ---- extensions ----
    "BatchRequestOffloadRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("items", ["RequestOffloadRequest"])],
    "BatchRequestOffloadResponse": STATUS + [("grants", ["RequestOffloadResponse"])],
    "BatchRequestPrefetchRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("items", ["RequestPrefetchRequest"])],
    "BatchRequestPrefetchResponse": STATUS + [("results", ["RequestPrefetchResponse"])],
    "PeerBufferDesc": [("key", S), ("owner_rank", "u32"), ("device", "u32"), ("kind", "u32"), ("nbytes", "u64"),
                       ("offset", "u64"), ("handle", "bytes")],
    "PublishPeerBufferRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("desc", "PeerBufferDesc")],
    "LookupPeerBufferRequest": [("key", S), ("wait_ms", "u32")],
    "LookupPeerBufferResponse": STATUS + [("found", "bool"), ("desc", "PeerBufferDesc")],
    "JobStatsEntry": [("job", "JobKey"), ("pinned_bytes", "u64"), ("pageable_bytes", "u64"), ("nvme_bytes", "u64"),
                      ("inflight_d2h_bytes", "u64"), ("inflight_export_bytes", "u64"),
                      ("canonical_object_count", "u64"), ("dedup_bytes_saved", "u64")],
    "GetJobStatsRequest": [("tenant_id", "u64"), ("all_tenants", "bool")],
    "GetJobStatsResponse": STATUS + [("jobs", ["JobStatsEntry"])],
    "ExportManifestRequest": [("job", "JobKey"), ("model_role", "u32"), ("model_version", "u64"), ("path", S)],
    "ExportManifestResponse": STATUS + [("bytes_written", "u64"), ("tensor_count", "u64")],
    "DiscardTensorRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("tensor_id", "u64"), ("version", "u64")],
    "CarryForwardRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("job", "JobKey"), ("model_role", "u32"),
                            ("from_version", "u64"), ("to_version", "u64"), ("param_ids", ["u64"]),
                            ("shard", "bool"), ("pp_rank", "u32"), ("tp_rank", "u32"), ("ep_rank", "u32"),
                            ("etp_rank", "u32"), ("expert_id", "i32")],
    "CarryForwardResponse": STATUS + [("carried_count", "u32"), ("existing_count", "u32"), ("missing_count", "u32"),
                                      ("bytes_shared", "u64")],
    "OptionEntry": [("key", S), ("value", S)],
    "GetAgentOptionsRequest": [("rank_id", "u32"), ("gpu_id", "u32")],
    "GetAgentOptionsResponse": STATUS + [("options", ["OptionEntry"])],
    "TensorVersion": [("tensor_id", "u64"), ("version", "u64")],
    "BatchDiscardTensorRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("items", ["TensorVersion"])],
    "BatchDiscardTensorResponse": STATUS + [("results", ["Status"])],
    "SetRunFormatRequest": [("rank_id", "u32"), ("rank_epoch", "u64"), ("lease_id", "u64"), ("slot_id", "u32"),
                            ("format", "u64")],
}

# opcode -> (request message, response message)
OPS: Dict[int, Tuple[str, str]] = {
    Op.REGISTER_RANK: ("RegisterRankRequest", "RegisterRankResponse"),
    Op.HEARTBEAT: ("HeartbeatRequest", "Status"),
    Op.REQUEST_OFFLOAD: ("RequestOffloadRequest", "RequestOffloadResponse"),
    Op.MARK_D2H_SUBMITTED: ("TransferMark", "Status"),
    Op.MARK_D2H_COMPLETE: ("TransferMark", "MarkD2HCompleteResponse"),
    Op.REQUEST_PREFETCH: ("RequestPrefetchRequest", "RequestPrefetchResponse"),
    Op.MARK_H2D_SUBMITTED: ("TransferMark", "Status"),
    Op.MARK_H2D_COMPLETE: ("MarkH2DCompleteRequest", "Status"),
    Op.RELEASE_LEASE: ("ReleaseLeaseRequest", "Status"),
    Op.QUERY_LOCATION: ("LocationQueryRequest", "LocationQueryResponse"),
    Op.BATCH_COMPLETE: ("BatchCompleteRequest", "BatchCompleteResponse"),
    Op.SHUTDOWN: ("ShutdownRequest", "Status"),
    Op.GET_STATS: ("GetStatsRequest", "GetStatsResponse"),
    Op.REGISTER_JOB: ("RegisterJobRequest", "RegisterJobResponse"),
    Op.REQUEST_CANONICAL_EVICT: ("RequestCanonicalEvictRequest", "RequestCanonicalEvictResponse"),
    Op.COMMIT_CANONICAL_OBJECT: ("CommitCanonicalObjectRequest", "CommitCanonicalObjectResponse"),
    Op.SEAL_MODEL_VERSION: ("SealModelVersionRequest", "SealModelVersionResponse"),
    Op.GET_LATEST_SEALED_VERSION: ("GetLatestSealedVersionRequest", "GetLatestSealedVersionResponse"),
    Op.GET_MANIFEST: ("GetManifestRequest", "GetManifestResponse"),
    Op.PULL_TENSOR: ("PullTensorRequest", "PullTensorResponse"),
    Op.REQUEST_CANONICAL_RESTORE: ("RequestCanonicalRestoreRequest", "RequestCanonicalRestoreResponse"),
    Op.RELEASE_CANONICAL_RESTORE: ("ReleaseCanonicalRestoreRequest", "Status"),
    Op.DROP_CANONICAL_VERSION: ("DropCanonicalVersionRequest", "DropCanonicalVersionResponse"),
    Op.RELEASE_CANONICAL: ("ReleaseCanonicalRequest", "ReleaseCanonicalResponse"),
    Op.BATCH_REQUEST_OFFLOAD: ("BatchRequestOffloadRequest", "BatchRequestOffloadResponse"),
    Op.BATCH_REQUEST_PREFETCH: ("BatchRequestPrefetchRequest", "BatchRequestPrefetchResponse"),
    Op.PUBLISH_PEER_BUFFER: ("PublishPeerBufferRequest", "Status"),
    Op.LOOKUP_PEER_BUFFER: ("LookupPeerBufferRequest", "LookupPeerBufferResponse"),
    Op.GET_JOB_STATS: ("GetJobStatsRequest", "GetJobStatsResponse"),
    Op.EXPORT_MANIFEST: ("ExportManifestRequest", "ExportManifestResponse"),
    Op.DISCARD_TENSOR: ("DiscardTensorRequest", "Status"),
    Op.CARRY_FORWARD: ("CarryForwardRequest", "CarryForwardResponse"),
    Op.GET_AGENT_OPTIONS: ("GetAgentOptionsRequest", "GetAgentOptionsResponse"),
    Op.BATCH_DISCARD_TENSOR: ("BatchDiscardTensorRequest", "BatchDiscardTensorResponse"),
    Op.SET_RUN_FORMAT: ("SetRunFormatRequest", "Status"),
}

_PRIM = {"u8": struct.Struct("<B"), "u16": struct.Struct("<H"), "u32": struct.Struct("<I"),
         "u64": struct.Struct("<Q"), "i32": struct.Struct("<i")}
_MASK = {"u8": 0xFF, "u16": 0xFFFF, "u32": 0xFFFFFFFF, "u64": 0xFFFFFFFFFFFFFFFF}


class WireError(ValueError):
    """Malformed or truncated wire data."""


def _default(t):
    if isinstance(t, list):
        return []
    if t in ("str",):
        return ""
    if t == "bytes":
        return b""
    if t == "bool":
        return False
    if t in _PRIM:
        return -1 if False else 0
    return defaults(t)


def defaults(msg: str) -> dict:
    """A message dict with every field at its zero value (expert_id = -1)."""
    out = {}
    for name, t in SCHEMA[msg]:
        out[name] = _default(t)
    if msg == "CanonicalKey":
        out["expert_id"] = -1
    return out


def _put(buf: bytearray, t, v) -> None:
    if isinstance(t, list):
        v = list(v or [])
        buf += _PRIM["u32"].pack(len(v))
        for e in v:
            _put(buf, t[0], e)
    elif t == "bool":
        buf.append(1 if v else 0)
    elif t == "str":
        data = (v or "").encode("utf-8")
        buf += _PRIM["u32"].pack(len(data))
        buf += data
    elif t == "bytes":
        data = bytes(v or b"")
        buf += _PRIM["u32"].pack(len(data))
        buf += data
    elif t == "i32":
        buf += _PRIM["u32"].pack(int(v) & 0xFFFFFFFF)
    elif t in _PRIM:
        buf += _PRIM[t].pack(int(v) & _MASK[t])
    else:
        encode_into(buf, t, v or {})


def encode_into(buf: bytearray, msg: str, values: dict) -> None:
    for name, t in SCHEMA[msg]:
        _put(buf, t, values.get(name, _default(t) if not (msg == "CanonicalKey" and name == "expert_id") else -1))


def encode(msg: str, values: dict | None = None, **kw) -> bytes:
    """Encode ``values`` (missing fields default to zero) as message ``msg``."""
    v = dict(values or {})
    v.update(kw)
    buf = bytearray()
    encode_into(buf, msg, v)
    return bytes(buf)


class _Reader:
    def __init__(self, data: bytes):
        self.d = memoryview(data)
        self.p = 0

    def take(self, n: int) -> memoryview:
        if self.p + n > len(self.d):
            raise WireError("truncated wire message")
        v = self.d[self.p:self.p + n]
        self.p += n
        return v

    def get(self, t):
        if isinstance(t, list):
            n = _PRIM["u32"].unpack(self.take(4))[0]
            if n > len(self.d) - self.p:
                raise WireError("truncated wire message")
            return [self.get(t[0]) for _ in range(n)]
        if t == "bool":
            return self.take(1)[0] != 0
        if t in ("str", "bytes"):
            n = _PRIM["u32"].unpack(self.take(4))[0]
            raw = bytes(self.take(n))
            return raw.decode("utf-8", errors="replace") if t == "str" else raw
        if t in _PRIM:
            s = _PRIM[t]
            return s.unpack(self.take(s.size))[0]
        return {name: self.get(ft) for name, ft in SCHEMA[t]}


def decode(msg: str, data: bytes) -> dict:
    """Decode ``data`` as message ``msg``; raises WireError when truncated."""
    return _Reader(data).get(msg)


def make_frame(opcode: int, body: bytes, flags: int = 0) -> bytes:
    return FRAME_HEADER.pack(RPC_MAGIC, opcode, flags, len(body)) + body


def parse_frame_header(data: bytes) -> Tuple[int, int, int]:
    if len(data) < FRAME_HEADER.size:
        raise WireError("short frame header")
    magic, op, flags, n = FRAME_HEADER.unpack(data[:FRAME_HEADER.size])
    if magic != RPC_MAGIC:
        raise WireError("bad frame magic")
    return op, flags, n


def recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = sock.recv_into(view[got:], n - got)
        if k == 0:
            raise ConnectionError("connection closed mid-message")
        got += k
    return bytes(buf)


def recv_frame(sock: socket.socket) -> Tuple[int, bytes]:
    op, _flags, n = parse_frame_header(recv_exact(sock, FRAME_HEADER.size))
    if n > MAX_PAYLOAD:
        raise WireError("frame payload too large")
    return op, recv_exact(sock, n) if n else b""


def parse_export_header(hdr: bytes) -> dict:
    magic, ver, oid, nbytes, hlo, hhi = EXPORT_HEADER.unpack(hdr[:EXPORT_HEADER_SIZE])
    if magic != EXPORT_MAGIC:
        raise WireError("bad export header magic")
    return {"version": ver, "object_id": oid, "nbytes": nbytes, "content_hash_lo": hlo, "content_hash_hi": hhi}


# ---------------------------------------------------------------------------
# Message helpers under StateSpectre's names (reference:
# python_api/state_spectre/_wire.py), thin wrappers of the schema codec above
# for tools written against them.
# ---------------------------------------------------------------------------
OFLD_RPC_MAGIC = RPC_MAGIC
EXPORT_HEADER_FMT = EXPORT_HEADER.format


def _job(tenant_id, job_id, launch_epoch, job_name) -> dict:
    return {"tenant_id": int(tenant_id), "job_id": int(job_id), "launch_epoch": int(launch_epoch),
            "job_name": job_name or ""}


def encode_get_latest(tenant_id, job_id, launch_epoch, job_name, model_role) -> bytes:
    return encode("GetLatestSealedVersionRequest", job=_job(tenant_id, job_id, launch_epoch, job_name),
                  model_role=int(model_role))


def decode_get_latest_resp(payload: bytes) -> dict:
    return decode("GetLatestSealedVersionResponse", payload)


def manifest_filter(flt: Optional[dict] = None) -> dict:
    """Filter dict (keys ``pp``, ``tp``, ``ep``, ``etp``, ``expert``) as the
    ManifestFilter message; absent keys match everything."""
    flt = flt or {}
    out = {}
    for axis in ("pp", "tp", "ep", "etp"):
        out[f"{axis}_present"] = axis in flt
        out[f"{axis}_rank"] = int(flt.get(axis, 0))
    out["expert_present"] = "expert" in flt
    out["expert_id"] = int(flt.get("expert", 0))
    return out


def encode_get_manifest(tenant_id, job_id, launch_epoch, job_name, model_role, model_version, flt=None) -> bytes:
    return encode("GetManifestRequest", job=_job(tenant_id, job_id, launch_epoch, job_name),
                  model_role=int(model_role), model_version=int(model_version), filter=manifest_filter(flt))


def decode_get_manifest_resp(payload: bytes) -> dict:
    return decode("GetManifestResponse", payload)


def encode_pull(tenant_id, job_id, launch_epoch, job_name, model_role, model_version, object_id, transport,
                target_descriptor) -> bytes:
    return encode("PullTensorRequest", job=_job(tenant_id, job_id, launch_epoch, job_name),
                  model_role=int(model_role), model_version=int(model_version), object_id=int(object_id),
                  transport=int(transport), target_descriptor=target_descriptor or "")


def decode_pull_resp(payload: bytes) -> dict:
    return decode("PullTensorResponse", payload)


class Connection:
    """One control connection (UDS path, ``unix://path`` or ``tcp://host:port``).

    Reused for any number of round trips; a lock serialises them.
    """

    def __init__(self, addr: str, timeout: float = 30.0):
        import threading

        self.addr = addr
        if addr.startswith("tcp://"):
            host, _, port = addr[6:].rpartition(":")
            self.sock = socket.create_connection((host, int(port)), timeout=timeout)
            self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        else:
            path = addr[7:] if addr.startswith("unix://") else addr
            self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            self.sock.settimeout(timeout)
            self.sock.connect(path)
        self._lock = threading.Lock()

    def call(self, opcode: int, values: dict | None = None, **kw) -> dict:
        req_name, resp_name = OPS[opcode]
        body = encode(req_name, values, **kw)
        with self._lock:
            self.sock.sendall(make_frame(opcode, body))
            rop, payload = recv_frame(self.sock)
        if rop != opcode:
            raise WireError(f"reply opcode mismatch: sent {opcode} got {rop}")
        return decode(resp_name, payload)

    def close(self) -> None:
        try:
            self.sock.close()
        except OSError:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
