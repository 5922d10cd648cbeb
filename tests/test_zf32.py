"""zf32 coding of fp32 objects: host reference codec (no GPU).

A 128 KiB row of fp32 values is stored as its 64 KiB low-half plane
followed by the zbf16 coded chunk of its top halves; the GPU kernels are
checked against this codec in test_zf32_gpu.py.
"""

import numpy as np
import pytest
import torch

from statespectre_b200._native import native

ROW = 131072
CHUNK = 65536


def _f32_bytes(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.float32).contiguous().view(torch.uint8).numpy()


def _halves(raw: np.ndarray):
    w = raw.view("<u4")
    return (w >> 16).astype("<u2").tobytes(), (w & 0xFFFF).astype("<u2").tobytes()


@pytest.mark.parametrize("std", [1.0, 0.02, 1e-4])
@pytest.mark.parametrize("rows", [1, 3, 8])
def test_gaussian_round_trip_and_ratio(std, rows):
    C = native()
    g = torch.Generator().manual_seed(rows * 7 + int(std * 1000))
    raw = _f32_bytes(torch.randn(rows * ROW // 4, generator=g) * std)
    coded = C.zf32_encode(raw)
    assert coded is not None and len(coded) == len(raw)
    assert C.zf32_decode(coded) == raw.tobytes()
    ratio = C.zf32_coded_bytes(coded) / len(raw)
    assert ratio < 0.86, ratio  # 16 raw bits + ~11 coded bits of the top half per value


def test_row_layout_is_low_plane_then_zbf16_chunk_of_top_halves():
    C = native()
    g = torch.Generator().manual_seed(5)
    raw = _f32_bytes(torch.randn(2 * ROW // 4, generator=g))
    coded = C.zf32_encode(raw)
    for r in range(2):
        row = raw[r * ROW:(r + 1) * ROW]
        hi, lo = _halves(row)
        out = coded[r * ROW:(r + 1) * ROW]
        assert out[:CHUNK] == lo
        zb = C.zbf16_encode(np.frombuffer(hi, dtype=np.uint8))
        stored = C.zbf16_coded_bytes(zb)
        assert out[CHUNK:CHUNK + stored] == zb[:stored]


def test_adam_second_moment_like_values_round_trip():
    """Positive values over many binades (squared gradients): more escapes,
    still lossless and smaller than the raw bytes."""
    C = native()
    g = torch.Generator().manual_seed(9)
    v = (torch.randn(4 * ROW // 4, generator=g) * 1e-3) ** 2 + 1e-12
    raw = _f32_bytes(v)
    coded = C.zf32_encode(raw)
    assert coded is not None
    assert C.zf32_decode(coded) == raw.tobytes()
    assert C.zf32_coded_bytes(coded) < len(raw)


def test_zeros_and_subnormals_round_trip_but_inf_and_nan_keep_the_object_raw():
    """Zeros and subnormals are exponent-0 escapes; an inf or NaN puts the
    row's window at the top binade, every finite value escapes, the row no
    longer fits and the object moves uncoded."""
    C = native()
    x = torch.randn(2 * ROW // 4)
    x[::97] = 0.0
    x[1::89] = -0.0
    x[4::1005] = 1e-40  # subnormal
    raw = _f32_bytes(x)
    coded = C.zf32_encode(raw)
    assert coded is not None
    assert C.zf32_decode(coded) == raw.tobytes()
    for special in (float("inf"), float("nan")):
        y = x.clone()
        y[ROW // 4 + 3] = special  # second row only
        assert C.zf32_encode(_f32_bytes(y)) is None


def test_random_bits_are_not_codable():
    C = native()
    raw = np.random.default_rng(0).integers(0, 256, size=2 * ROW, dtype=np.uint8)
    assert C.zf32_encode(raw) is None


def test_only_whole_rows_are_eligible():
    C = native()
    assert C.zf32_encode(np.zeros(ROW + 4096, dtype=np.uint8)) is None
    assert C.zf32_encode(np.zeros(ROW // 2, dtype=np.uint8)) is None
    assert C.zf32_encode(np.zeros(ROW, dtype=np.uint8)) is not None


def test_decoder_rejects_corruption():
    C = native()
    raw = _f32_bytes(torch.randn(ROW // 4))
    coded = bytearray(C.zf32_encode(raw))
    coded[CHUNK] ^= 0xFF  # the top-half chunk's header tag
    with pytest.raises(RuntimeError):
        C.zf32_decode(bytes(coded))
