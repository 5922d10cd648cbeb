"""ssh128 in numpy, written from the written definition of the hash (the
"Definition" comment of csrc/include/ofld/chunk_hash.h), not from its code.

The structure is deliberately different from the C++ and CUDA forms: every
chunk of an object is processed at once as an array of shape
(chunks, 16 rounds, 256 lanes, 4 words), the lane rounds are array
operations, and the tree levels are strided array folds. Only the object
fold, a short sequential chain, is plain Python integers.
"""

from __future__ import annotations

import numpy as np

CHUNK = 64 * 1024
LANES = 256
ROUNDS = 16  # vectors per lane in a full chunk

P1, P2, P3, P4, P5 = 2654435761, 2246822519, 3266489917, 668265263, 374761393
G = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1

_u32 = np.uint32
_u64 = np.uint64


def _rotl32(x, r):
    return (x << _u32(r)) | (x >> _u32(32 - r))


def _avalanche32(h):
    h = h ^ (h >> _u32(15))
    h = h * _u32(P2)
    h = h ^ (h >> _u32(13))
    h = h * _u32(P3)
    return h ^ (h >> _u32(16))


def _fmix64(k):
    k = k ^ (k >> _u64(33))
    k = k * _u64(0xFF51AFD7ED558CCD)
    k = k ^ (k >> _u64(33))
    k = k * _u64(0xC4CEB9FE1A85EC53)
    return k ^ (k >> _u64(33))


def _fold(a, b):
    return _fmix64(a ^ (b * _u64(G)))


def chunk_digests(data) -> list:
    """Chunk digests (u64 ints) of a bytes-like object."""
    buf = np.frombuffer(bytes(data), dtype=np.uint8)
    n = buf.size
    nchunks = (n + CHUNK - 1) // CHUNK
    if nchunks == 0:
        return []
    padded = np.zeros(nchunks * CHUNK, dtype=np.uint8)
    padded[:n] = buf
    # vector v of a chunk is words [4v, 4v+4); lane t takes v = r*256 + t
    words = padded.view("<u4").reshape(nchunks, ROUNDS, LANES, 4)
    lens = np.full(nchunks, CHUNK, dtype=np.int64)
    lens[-1] = n - (nchunks - 1) * CHUNK
    nvec = (lens + 15) // 16  # vectors present in each chunk (last one zero-padded)
    vidx = (np.arange(ROUNDS)[:, None] * LANES + np.arange(LANES)[None, :])  # (16, 256)
    present = vidx[None, :, :] < nvec[:, None, None]                        # (chunks, 16, 256)

    with np.errstate(over="ignore"):
        t = np.arange(LANES, dtype=_u32)
        seed = t * _u32(P5) + _u32(0x9E3779B9)
        acc = np.stack([seed + _u32(P1) + _u32(P2), seed + _u32(P2), seed, seed - _u32(P1)], axis=-1)
        acc = np.broadcast_to(acc, (nchunks, LANES, 4)).copy()
        for r in range(ROUNDS):
            upd = _rotl32(acc + words[:, r] * _u32(P2), 13) * _u32(P1)
            acc = np.where(present[:, r, :, None], upd, acc)
        a0, a1, a2, a3 = (acc[..., i] for i in range(4))
        lo = _avalanche32((_rotl32(a0, 1) + _rotl32(a1, 7) + _rotl32(a2, 12) + _rotl32(a3, 18)) ^ (t * _u32(P3)))
        hi = _avalanche32((_rotl32(a0, 3) ^ _rotl32(a1, 11) ^ _rotl32(a2, 17) ^ _rotl32(a3, 25)) + _u32(P4) + t)
        x = (hi.astype(_u64) << _u64(32)) | lo.astype(_u64)  # (chunks, 256) lane digests
        s = 1
        while s < LANES:
            x = x.copy()
            x[:, 0::2 * s] = _fold(x[:, 0::2 * s], x[:, s::2 * s])
            s *= 2
        dig = _fold(x[:, 0], lens.astype(_u64))
    return [int(d) for d in dig]


def object_hash(data) -> tuple:
    """(lo, hi) object hash of a bytes-like object."""
    n = len(bytes(data))
    lo, hi = 0xCBF29CE484222325, 0x6A09E667F3BCC909
    for d in chunk_digests(data):
        lo = ((lo ^ d) * 0x100000001B3) & M64
        x = hi ^ d
        hi = ((((x << 29) | (x >> 35)) & M64) * G + 0x94D049BB133111EB) & M64
    with np.errstate(over="ignore"):
        out = (int(_fmix64(_u64(lo ^ n))), int(_fmix64(_u64((hi + n) & M64))))
    return (1, 0) if out == (0, 0) else out
