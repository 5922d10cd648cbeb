"""The allocation-free hash entry point, called through its exported C symbol.

`ofld_hash_noalloc` serves callers that cannot allocate device memory at the
moment they need a checksum (allocator hooks, pre-reserved memory pools,
latency-critical paths, out-of-memory handlers). It keeps its chunk digests
in a fixed device array inside the library, so this test checks that its
results equal the regular entry point's (hash_device + fold_digests, which
uses a caller-provided digest buffer) on two calls in a row, and that sizes
beyond its 8 GiB limit are refused before anything is launched.

This file is collected last so that a run stopping at its first failure has
already run every other test.
"""

import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "statespectre_b200")


def _lib():
    from statespectre_b200._native import native

    native()  # the extension is what carries the symbol
    path = glob.glob(os.path.join(PKG, "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.ofld_hash_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _regular_hash(x: torch.Tensor) -> tuple:
    from statespectre_b200._native import native

    C = native()
    n = x.numel() * x.element_size()
    nd = max((n + 65535) // 65536, 1)
    dig = torch.zeros(nd, dtype=torch.int64, device=x.device)
    out = torch.zeros(2, dtype=torch.int64, device=x.device)
    s = torch.cuda.current_stream().cuda_stream
    if n:
        C.k_hash_device(x.data_ptr(), n, dig.data_ptr(), s, 0)
    C.k_fold_digests(dig.data_ptr(), (n + 65535) // 65536, n, out.data_ptr(), s)
    torch.cuda.synchronize()
    return tuple(int(v) & 0xFFFFFFFFFFFFFFFF for v in out.cpu().tolist())


def _noalloc_hash(fn, x: torch.Tensor) -> tuple:
    out = torch.zeros(2, dtype=torch.int64, device=x.device)
    n = x.numel() * x.element_size()
    rc = fn(x.data_ptr() if n else None, n, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return tuple(int(v) & 0xFFFFFFFFFFFFFFFF for v in out.cpu().tolist())


def test_noalloc_hash_matches_regular_entry_point_twice():
    fn = _lib()
    torch.manual_seed(3)
    a = torch.randint(0, 256, ((5 << 20) + 37,), dtype=torch.uint8, device="cuda")
    b = torch.randn(3 << 20, device="cuda")  # a second, larger call reusing the same scratch
    assert _noalloc_hash(fn, a) == _regular_hash(a)
    assert _noalloc_hash(fn, b) == _regular_hash(b)
    # the first call's digests left in the scratch array do not leak into a smaller call
    assert _noalloc_hash(fn, a[:1000]) == _regular_hash(a[:1000])


def test_noalloc_hash_unaligned_and_empty_inputs():
    """Any alignment and any size: a source one byte past an allocation
    boundary with a ragged length takes the per-thread hash form through the
    same scratch array; zero bytes runs only the fold."""
    fn = _lib()
    torch.manual_seed(5)
    a = torch.randint(0, 256, ((3 << 20) + 64,), dtype=torch.uint8, device="cuda")
    odd = a[1:1 + (1 << 20) + 5]
    assert odd.data_ptr() % 16 == 1
    assert _noalloc_hash(fn, odd) == _regular_hash(odd)
    empty = a[:0]
    assert _noalloc_hash(fn, empty) == _regular_hash(empty)
    assert _noalloc_hash(fn, odd) == _regular_hash(odd)  # and once more after the empty call


def test_noalloc_rejects_oversize_and_null_without_launching():
    fn = _lib()
    x = torch.zeros(16, dtype=torch.uint8, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert fn(x.data_ptr(), (8 << 30) + 1, out.data_ptr(), s) == 1
    assert fn(None, 16, out.data_ptr(), s) == 2
    assert fn(x.data_ptr(), 16, None, s) == 2
    torch.cuda.synchronize()
    assert out.abs().sum().item() == 0
