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
        assert ratio < 0.77, ratio  # 12 bits per value + a few escapes


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
    assert C.zbf16_coded_bytes(coded) > 0.75 * len(raw)


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
