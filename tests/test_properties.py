"""Property tests (hypothesis) of the wire codec and the zbf16 host coder.

* Arbitrary bytes given to the C++ decoder of any message are either
  rejected with an error or decoded; a decoded body re-encodes to a fixed
  point. A daemon parses whatever a peer sends, so no input may crash it.
* Any message the Python schema can express, with random field values, is
  encoded byte for byte alike by both codecs.
* zbf16 coding is lossless on every bf16 input it accepts, and decoding
  damaged coded bytes fails cleanly.
"""

import numpy as np
import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from statespectre_b200 import _wire
from statespectre_b200._native import native

SETTINGS = settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.too_slow])
MESSAGES = sorted({(op, False) for op in _wire.OPS} | {(op, True) for op in _wire.OPS})


def _value(t, depth=0):
    if isinstance(t, list):
        return st.lists(_value(t[0], depth + 1), max_size=3 if depth < 2 else 0)
    if t == "u32":
        return st.integers(0, 2 ** 32 - 1)
    if t == "u64":
        return st.integers(0, 2 ** 64 - 1)
    if t == "i32":
        return st.integers(-2 ** 31, 2 ** 31 - 1)
    if t == "bool":
        return st.booleans()
    if t == "str":
        return st.text(max_size=12)
    if t == "bytes":
        return st.binary(max_size=24)
    return _message(t, depth + 1)


def _message(name, depth=0):
    return st.fixed_dictionaries({f: _value(t, depth) for f, t in _wire.SCHEMA[name]})


@SETTINGS
@given(msg=st.sampled_from(MESSAGES), body=st.binary(max_size=96))
def test_decoder_rejects_or_reaches_a_fixed_point_on_arbitrary_bytes(msg, body):
    op, response = msg
    try:
        once = native().reencode(op, response, body)
    except Exception:  # WireError surfaces as a Python exception; the process lives on
        return
    assert native().reencode(op, response, once) == once


@SETTINGS
@given(data=st.data(), msg=st.sampled_from(MESSAGES))
def test_python_and_cpp_codecs_agree_on_random_messages(data, msg):
    op, response = msg
    name = _wire.OPS[op][1 if response else 0]
    values = data.draw(_message(name))
    body = _wire.encode(name, values)
    assert native().reencode(op, response, body) == body
    assert _wire.encode(name, _wire.decode(name, body)) == body


def _bf16(words: np.ndarray) -> np.ndarray:
    return words.astype(np.uint16)


@SETTINGS
@given(nchunks=st.integers(1, 3), tail=st.sampled_from([0, 16, 4096, 8192 + 48]), spread=st.integers(0, 40),
       seed=st.integers(0, 2 ** 32 - 1))
def test_zbf16_round_trip_is_exact(nchunks, tail, spread, seed):
    rng = np.random.default_rng(seed)
    n = (nchunks * 65536 + tail) // 2
    # sign and mantissa random; exponents clustered around 120 with `spread` binades of scatter
    sign_mant = rng.integers(0, 1 << 16, n, dtype=np.uint32) & 0x807F
    exp = np.clip(120 + rng.integers(-spread, spread + 1, n), 0, 255).astype(np.uint32)
    words = _bf16(sign_mant | (exp << 7))
    raw = words.tobytes()
    coded = native().zbf16_encode(words)
    if coded is None:  # a chunk whose coding would not fit: stored raw by the caller
        return
    assert len(coded) == len(raw)
    assert native().zbf16_coded_bytes(coded) <= len(raw)
    assert native().zbf16_decode(coded) == raw


@SETTINGS
@given(seed=st.integers(0, 2 ** 32 - 1), flips=st.integers(1, 8))
def test_zbf16_decode_of_damaged_bytes_fails_cleanly(seed, flips):
    rng = np.random.default_rng(seed)
    n = 65536
    words = _bf16((rng.integers(0, 1 << 16, n, dtype=np.uint32) & 0x807F) | (np.uint32(121) << 7))
    coded = bytearray(native().zbf16_encode(words))
    for _ in range(flips):
        i = int(rng.integers(0, 16))  # the chunk header: tag, mode, ebase, escape count, lengths
        coded[i] ^= 1 << int(rng.integers(0, 8))
    try:
        out = native().zbf16_decode(bytes(coded))
    except RuntimeError:
        return
    assert len(out) == len(coded)  # a damaged ebase still decodes, to other values of the same size


def test_schema_covers_every_opcode():
    assert native().op_name(999) == "Unknown"
    for op in _wire.OPS:
        assert native().op_name(op) != "Unknown", op
    with pytest.raises(RuntimeError, match="unknown opcode"):
        native().reencode(999, False, b"")


@SETTINGS
@given(mode=st.sampled_from([1, 2]), ebase=st.integers(0, 255), n_esc=st.integers(0, 3000),
       len_kib=st.sampled_from([4, 16, 64]), seed=st.integers(0, 2**32 - 1), flip=st.integers(0, 65535))
def test_export_decoder_survives_arbitrary_chunks(mode, ebase, n_esc, len_kib, seed, flip):
    """The daemon's export decoder on chunks with a self-consistent header and
    arbitrary contents (random planes, any escape count, one flipped byte):
    it returns bytes or refuses, and it never reads or writes outside the
    chunk, whatever the codes say."""
    import struct

    import numpy as np

    from statespectre_b200._native import native

    length = len_kib * 1024
    n = length // 2
    plane = (n // 8) * 3 if mode == 2 else n // 2
    comp = 16 + n + plane + n_esc
    if comp > length:
        comp, n_esc = length, max(0, length - 16 - n - plane)
    rng = np.random.default_rng(seed)
    body = bytearray(rng.integers(0, 256, length, dtype=np.uint8).tobytes())
    body[:16] = struct.pack("<HBBIII", 0x425A, mode, ebase, n_esc, length, 16 + n + plane + n_esc)
    if flip >= 16 and flip < length:
        body[flip] ^= 0x5A
    try:
        out = native().zcoded_decode_range(1, bytes(body), 0, length)
        assert len(out) == length
    except RuntimeError:
        pass
