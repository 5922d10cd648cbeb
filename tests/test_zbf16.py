"""zbf16 chunk coding: host reference codec (no GPU).

The GPU kernels are checked against this codec in test_zbf16_gpu.py.
"""

import numpy as np
import pytest
import torch

from statespectre_b200._native import native

CHUNK = 65536


def _bf16_bytes(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.uint8).numpy()


@pytest.mark.parametrize("std", [1.0, 0.02, 1e-3])
@pytest.mark.parametrize("nbytes", [4096, 65536, 3 * 65536 + 4096, 5 * 65536 + 1024 * 16])
def test_gaussian_round_trip_and_ratio(std, nbytes):
    C = native()
    g = torch.Generator().manual_seed(nbytes)
    x = torch.randn(nbytes // 2, generator=g) * std
    raw = _bf16_bytes(x)
    coded = C.zbf16_encode(raw)
    assert coded is not None and len(coded) == nbytes
    assert C.zbf16_decode(coded) == raw.tobytes()
    ratio = C.zbf16_coded_bytes(coded) / nbytes
    tail = nbytes % CHUNK
    if tail == 0 or tail >= 4096:
        assert ratio < 0.73, ratio  # 11 bits per value (3-bit codes) + the escapes below 7 binades


def test_zeros_and_constants_code():
    C = native()
    for fill in (0.0, 1.0, -3.5):
        raw = _bf16_bytes(torch.full((1 << 16,), fill))
        coded = C.zbf16_encode(raw)
        assert coded is not None
        assert C.zbf16_decode(coded) == raw.tobytes()


def test_random_bits_are_not_codable():
    C = native()
    raw = np.random.default_rng(0).integers(0, 256, size=1 << 17, dtype=np.uint8)
    assert C.zbf16_encode(raw) is None


def test_wide_range_values_escape_and_still_round_trip():
    C = native()
    g = torch.Generator().manual_seed(3)
    # most values N(0,1), 5 % spread over 40 binades: many escapes, still fits
    x = torch.randn(1 << 16, generator=g)
    mask = torch.rand(1 << 16, generator=g) < 0.05
    x[mask] = torch.exp2(torch.randint(-40, 0, (int(mask.sum()),), generator=g).float())
    raw = _bf16_bytes(x)
    coded = C.zbf16_encode(raw)
    assert coded is not None
    assert C.zbf16_decode(coded) == raw.tobytes()
    plain = C.zbf16_encode(_bf16_bytes(torch.randn(1 << 16, generator=torch.Generator().manual_seed(3))))
    assert C.zbf16_coded_bytes(coded) > C.zbf16_coded_bytes(plain)  # the escapes cost bytes


def _modes(coded: bytes, nbytes: int):
    return [coded[c * CHUNK + 2] for c in range(nbytes // CHUNK)]


def test_each_chunk_takes_the_shorter_code_width():
    """Gaussian-like chunks store 3-bit codes over the top 7 binades (mode
    2); values spread evenly over 14 binades keep 4-bit codes (mode 1), and
    so do chunks whose largest exponent is too small for a mode-2 window."""
    C = native()
    g = torch.Generator().manual_seed(11)
    gauss = _bf16_bytes(torch.randn(4 * CHUNK // 2, generator=g))
    wide = _bf16_bytes(torch.exp2(torch.rand(4 * CHUNK // 2, generator=g) * 14 - 7)
                       * torch.sign(torch.randn(4 * CHUNK // 2, generator=g)))
    tiny = _bf16_bytes(torch.randn(4 * CHUNK // 2, generator=g) * 1e-36)
    for raw, mode in ((gauss, 2), (wide, 1), (tiny, 1)):
        coded = C.zbf16_encode(raw)
        assert coded is not None and set(_modes(coded, len(raw))) == {mode}
        assert C.zbf16_decode(coded) == raw.tobytes()


def test_three_bit_code_layout():
    """Mode 2 byte layout of a chunk of 1.0s (exponent 127): base = 127 - 6,
    every code 6, a vector's eight codes as one little-endian 24-bit value
    (0b110 repeated: bytes B6 6D DB), no escapes."""
    C = native()
    raw = _bf16_bytes(torch.ones(CHUNK // 2))
    coded = C.zbf16_encode(raw)
    n = CHUNK // 2
    assert coded[2] == 2 and coded[3] == 121  # mode, base
    assert int.from_bytes(coded[4:8], "little") == 0  # escapes
    assert int.from_bytes(coded[12:16], "little") == 16 + n + 3 * n // 8
    assert coded[16:16 + n] == bytes(n)  # sign + mantissa of 1.0 are all zero
    assert coded[16 + n:16 + n + 6] == bytes([0xB6, 0x6D, 0xDB] * 2)
    assert C.zbf16_decode(coded) == raw.tobytes()


def test_ineligible_sizes():
    C = native()
    assert C.zbf16_encode(np.zeros(2048, dtype=np.uint8)) is None  # below one raw tail
    assert C.zbf16_encode(np.zeros(65536 + 8, dtype=np.uint8)) is None  # not a 16-byte multiple


def test_raw_tail_chunk_is_stored_verbatim():
    C = native()
    g = torch.Generator().manual_seed(5)
    raw = _bf16_bytes(torch.randn(65536 // 2 + 1024, generator=g))  # 64 KiB + 2 KiB tail
    coded = C.zbf16_encode(raw)
    assert coded is not None
    assert coded[65536:] == raw[65536:].tobytes()  # tail below 4 KiB: raw by rule
    assert C.zbf16_decode(coded) == raw.tobytes()


def test_decoder_rejects_corruption():
    C = native()
    raw = _bf16_bytes(torch.randn(1 << 15))
    coded = bytearray(C.zbf16_encode(raw))
    coded[0] ^= 0xFF  # header tag
    with pytest.raises(RuntimeError):
        C.zbf16_decode(bytes(coded))


@pytest.mark.parametrize("nbytes", [4096, 65536, 3 * 65536 + 4096, 7 * 65536 + 2048, 9 * 65536 + 16 * 1000])
def test_export_decoder_matches_the_reference_decoder(nbytes):
    """The daemon's allocation-free decoder (element-order pass, sorted escape
    patch) gives the reference decoder's bytes, for whole objects and for
    chunk-aligned sub-ranges, in both code widths and with many escapes."""
    C = native()
    g = torch.Generator().manual_seed(nbytes + 1)
    x = torch.randn(nbytes // 2, generator=g)
    x[::97] *= 1e-6  # deep escapes (mode 1)
    x[::13] *= 300.0  # widen the window so some chunks pick mode 2 and some mode 1
    raw = _bf16_bytes(x)
    coded = C.zbf16_encode(raw)
    assert coded is not None
    assert C.zcoded_decode_range(1, coded, 0, nbytes) == raw.tobytes()
    for off in range(0, nbytes, 2 * CHUNK):
        n = min(2 * CHUNK, nbytes - off)
        assert C.zcoded_decode_range(1, coded, off, n) == raw[off:off + n].tobytes()
    if nbytes > CHUNK:
        with pytest.raises(RuntimeError):
            C.zcoded_decode_range(1, coded, 16, CHUNK)  # not chunk-aligned


@pytest.mark.parametrize("rows", [1, 3])
def test_export_decoder_handles_zf32_rows(rows):
    C = native()
    g = torch.Generator().manual_seed(rows)
    x = torch.randn(rows * 32768, generator=g) * 0.02
    raw = x.contiguous().view(torch.uint8).numpy()
    coded = C.zf32_encode(raw)
    assert coded is not None
    assert C.zcoded_decode_range(2, coded, 0, len(raw)) == raw.tobytes()
    assert C.zcoded_decode_range(2, coded, 131072 * (rows - 1), 131072) == raw[131072 * (rows - 1):].tobytes()


def test_export_decoder_rejects_corruption():
    C = native()
    x = torch.randn(65536)
    coded = bytearray(C.zbf16_encode(_bf16_bytes(x)))
    coded[8] ^= 0xFF  # escape count no longer matches the codes
    with pytest.raises(RuntimeError):
        C.zcoded_decode_range(1, bytes(coded), 0, len(coded))
