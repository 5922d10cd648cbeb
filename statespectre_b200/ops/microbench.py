"""Kernel-level host<->device bandwidth sweep for tuning a node.

    python -m statespectre_b200.ops.microbench [--mb 1024] [--out sweep.json]

For each pinned-memory kind (cudaHostAlloc, memfd with 4 KiB pages, memfd
with transparent huge pages, anonymous THP) it times K1 (device -> host with
the fused hash) over store forms and CTA counts and K2 (host -> device) over
load forms and CTA counts, with CUDA events (median of 6 after a warm-up).
The results pick `kernels.evict_ctas` / `kernels.restore_ctas` and the
access policy for a node.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import mmap
import os

import torch

from .._native import native


def _memfd(n: int, huge: bool):
    fd = os.memfd_create("ofld-mb", 0)
    os.ftruncate(fd, n)
    mm = mmap.mmap(fd, n, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
    os.close(fd)
    if huge:
        try:
            mm.madvise(mmap.MADV_HUGEPAGE)
        except OSError:
            pass
    addr = ctypes.addressof(ctypes.c_char.from_buffer(mm))
    ctypes.memset(addr, 0, n)
    return mm, addr


def _anon(n: int):
    mm = mmap.mmap(-1, n, mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS, mmap.PROT_READ | mmap.PROT_WRITE)
    mm.madvise(mmap.MADV_HUGEPAGE)
    addr = ctypes.addressof(ctypes.c_char.from_buffer(mm))
    ctypes.memset(addr, 0, n)
    return mm, addr


def sweep(nbytes: int = 1 << 30, device: int = 0) -> dict:
    C = native()
    dev = torch.device("cuda", device)
    torch.cuda.set_device(dev)
    src = torch.randint(0, 255, (nbytes,), dtype=torch.uint8, device=dev)
    back = torch.empty_like(src)
    dig = torch.zeros((nbytes + 65535) // 65536, dtype=torch.int64, device=dev)
    s = torch.cuda.Stream(priority=-1)
    keep = []

    def timeit(fn, iters=6):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ts = []
        for _ in range(iters):
            e0.record(s)
            fn()
            e1.record(s)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return round(nbytes / (ts[len(ts) // 2] / 1e3) / 1e9, 2)

    pinned = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    regions = {"cudaHostAlloc": pinned.data_ptr()}
    for name, make in (("memfd4k", lambda: _memfd(nbytes, False)), ("memfd_thp", lambda: _memfd(nbytes, True)),
                       ("anon_thp", lambda: _anon(nbytes))):
        mm, addr = make()
        C.host_register(addr, nbytes)
        keep.append((mm, addr))
        regions[name] = addr
    out = {}
    for name, addr in regions.items():
        for st in (0, 1, 2):
            for ctas in (8, 16, 32, 64, 128):
                C.set_access_policy(0, st)
                out[f"{name}/k1 store{st} ctas{ctas}"] = timeit(
                    lambda: C.k_evict_hash(src.data_ptr(), addr, nbytes, dig.data_ptr(), s.cuda_stream, ctas))
        for ld in (0, 1, 2):
            for ctas in (16, 32, 64, 128, 256):
                C.set_access_policy(ld, 0)
                out[f"{name}/k2 load{ld} ctas{ctas}"] = timeit(
                    lambda: C.k_restore_cast(addr, back.data_ptr(), nbytes, 0, 0, 0, 0, s.cuda_stream, ctas))
    C.set_access_policy(0, 0)
    torch.cuda.synchronize()
    for _, addr in keep:
        C.host_unregister(addr)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mb", type=int, default=1024)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--out", default="")
    a = ap.parse_args()
    res = sweep(a.mb << 20, a.device)
    text = json.dumps(res, indent=1)
    print(text)
    if a.out:
        with open(a.out, "w") as f:
            f.write(text)


if __name__ == "__main__":
    main()
