"""Wire format: golden vectors, cross-language parity, framing and truncation.

Golden vectors pack the fields in the order StateSpectre's codec writes them
(reference: src/common/wire.cpp:66-412, wire_v2.cpp:11-438), so a byte match
here means frames interoperate with it.
"""

import random
import struct

import pytest

from statespectre_b200 import _wire
from statespectre_b200._native import native
from statespectre_b200._wire import Op


def s(text: str) -> bytes:
    b = text.encode()
    return struct.pack("<I", len(b)) + b


def test_golden_register_rank_request():
    body = _wire.encode("RegisterRankRequest", rank_id=3, local_rank=1, world_rank=7, gpu_id=2, numa_node=1,
                        pid=4242, capabilities=9)
    assert body == struct.pack("<IIIIIQQ", 3, 1, 7, 2, 1, 4242, 9)


def test_golden_request_offload_and_response():
    body = _wire.encode("RequestOffloadRequest", rank_id=1, rank_epoch=5, tensor_id=77, version=2, nbytes=4096,
                        gpu_id=0, numa_node=1, alignment=256, priority=0, flags=9, debug_name="w")
    assert body == struct.pack("<IQQQQIIIIQ", 1, 5, 77, 2, 4096, 0, 1, 256, 0, 9) + s("w")
    resp = _wire.encode("RequestOffloadResponse", ok=True, message="ok", lease_id=11, slot_id=4, arena_id=0,
                        arena_offset=8 << 20, capacity=2 << 20, state=1, blocked=False)
    assert resp == b"\x01" + s("ok") + struct.pack("<QIQQQI", 11, 4, 0, 8 << 20, 2 << 20, 1) + b"\x00"


def test_golden_canonical_key_expert_twos_complement():
    key = _wire.defaults("CanonicalKey")
    key.update(model_role=2, model_version=9, param_id=1, param_fqn_hash=2, param_fqn_debug="p", dtype=15,
               nbytes=64, pp_rank=1, tp_rank=2, ep_rank=3, etp_rank=4, expert_id=-1, shard_nbytes=64)
    key["job"] = {"tenant_id": 1, "job_id": 2, "launch_epoch": 3, "job_name": "j"}
    body = _wire.encode("CanonicalKey", key)
    expect = (struct.pack("<QQQ", 1, 2, 3) + s("j") + struct.pack("<IQQQ", 2, 9, 1, 2) + s("p") +
              struct.pack("<IIQQQIIIIIQQ", 15, 0, 64, 0, 0, 1, 2, 3, 4, 0xFFFFFFFF, 0, 64))
    assert body == expect
    assert _wire.decode("CanonicalKey", body)["expert_id"] == -1  # u32 two's complement on the wire


def test_golden_get_stats_response_interleaves_key_value():
    body = _wire.encode("GetStatsResponse", ok=True, message="ok",
                        stats=[{"key": "a", "value": 1}, {"key": "bb", "value": 2}])
    assert body == b"\x01" + s("ok") + struct.pack("<I", 2) + s("a") + struct.pack("<Q", 1) + s("bb") + \
        struct.pack("<Q", 2)


def test_frame_header():
    f = _wire.make_frame(Op.GET_STATS, b"\x01\x02")
    assert f[:12] == struct.pack("<IHHI", 0x4F465250, 13, 0, 2)
    assert _wire.parse_frame_header(f) == (13, 0, 2)
    with pytest.raises(_wire.WireError):
        _wire.parse_frame_header(b"XXXX" + f[4:])


def _random_value(t, rng):
    if isinstance(t, list):
        return [_random_value(t[0], rng) for _ in range(rng.randint(0, 3))]
    if t == "bool":
        return rng.random() < 0.5
    if t == "str":
        return "".join(rng.choice("abcxyz_0123") for _ in range(rng.randint(0, 9)))
    if t == "bytes":
        return bytes(rng.randint(0, 255) for _ in range(rng.randint(0, 70)))
    bits = {"u8": 8, "u16": 16, "u32": 32, "i32": 32, "u64": 64}[t] if t in ("u8", "u16", "u32", "i32", "u64") else None
    if bits:
        return rng.getrandbits(bits)
    return {name: _random_value(ft, rng) for name, ft in _wire.SCHEMA[t]}


@pytest.mark.parametrize("opcode", sorted(_wire.OPS))
def test_cpp_python_codec_parity(opcode):
    C = native()
    rng = random.Random(opcode)
    for response, msg in ((False, _wire.OPS[opcode][0]), (True, _wire.OPS[opcode][1])):
        for _ in range(5):
            v = _random_value(msg, rng)
            body = _wire.encode(msg, v)
            assert C.reencode(opcode, response, body) == body
            assert _wire.encode(msg, _wire.decode(msg, body)) == body


@pytest.mark.parametrize("opcode", [Op.REGISTER_RANK, Op.REQUEST_CANONICAL_EVICT, Op.GET_MANIFEST])
def test_truncation_rejected(opcode):
    C = native()
    msg = _wire.OPS[opcode][0]
    body = _wire.encode(msg, _random_value(msg, random.Random(1)))
    for cut in (1, len(body) // 2, len(body) - 1):
        with pytest.raises(_wire.WireError):
            _wire.decode(msg, body[:cut])
        with pytest.raises(Exception):
            C.reencode(opcode, False, body[:cut])


def test_export_header():
    hdr = struct.pack("<IIQQQQ", 0x4F464558, 1, 5, 100, 7, 8)
    assert _wire.parse_export_header(hdr) == {"version": 1, "object_id": 5, "nbytes": 100, "content_hash_lo": 7,
                                              "content_hash_hi": 8}


def test_op_names_cover_all_opcodes():
    C = native()
    for op in _wire.OPS:
        assert C.op_name(op) != "Unknown"


def test_proto_schema_docs_are_current():
    """rpc/*.proto are generated from the wire schema and must match it."""
    from statespectre_b200 import _proto

    assert _proto.main(["--check"]) == 0, "run: python -m statespectre_b200._proto"


def test_reference_named_helpers_and_compat_modules():
    """StateSpectre's message helpers keep their names and byte layout
    (job key, then the message's fields in order)."""
    import struct

    import state_spectre._rollout as R
    import state_spectre._wire as W

    assert R.RolloutWeightClient is not None
    job = struct.pack("<QQQI", 1, 42, 3, 2) + b"j0"
    assert W.encode_get_latest(1, 42, 3, "j0", 2) == job + struct.pack("<I", 2)
    filt = b"".join(struct.pack("<?I", k == "tp", 5 if k == "tp" else 0) for k in ("pp", "tp", "ep", "etp"))
    filt += struct.pack("<?i", False, 0)
    assert W.encode_get_manifest(1, 42, 3, "j0", 2, 7, {"tp": 5}) == job + struct.pack("<IQ", 2, 7) + filt
    pull = W.encode_pull(1, 42, 3, "j0", 2, 7, 99, 1, "127.0.0.1:5")
    assert pull == job + struct.pack("<IQQI", 2, 7, 99, 1) + struct.pack("<I", 11) + b"127.0.0.1:5"
    resp = W.encode("PullTensorResponse", ok=True, message="", object_id=99, nbytes=8, transport=1,
                    content_hash_lo=1, content_hash_hi=2, transport_metadata="")
    assert W.decode_pull_resp(resp)["nbytes"] == 8
    assert W.OFLD_RPC_MAGIC == 0x4F465250 and struct.calcsize(W.EXPORT_HEADER_FMT) == 40
