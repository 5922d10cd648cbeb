"""Launch one data-path kernel a few times on a fixed case (for ncu captures).

    python -m statespectre_b200.ops.profile_case --kernel evict --mb 512 --iters 3

Kernels: evict (K1, device -> pinned + ssh128), restore (K2, pinned ->
device), restore_fp8 (K2 with the bf16 -> fp8 1x128 cast), hash (device
ssh128), verify (K3 local vs second buffer). The case is larger than the
126 MB L2 so DRAM counters are meaningful; it holds about 2x --mb of device
memory and --mb of pinned host memory.
"""

from __future__ import annotations

import argparse

import torch

from .._native import native


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True, choices=["evict", "restore", "restore_fp8", "hash", "verify"])
    ap.add_argument("--mb", type=int, default=512)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--ctas", type=int, default=0)
    a = ap.parse_args()
    C = native()
    n = a.mb << 20
    dev = torch.device("cuda", 0)
    x = torch.randn(n // 2, dtype=torch.bfloat16, device=dev)
    host = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    dig = torch.zeros((n + 65535) // 65536, dtype=torch.int64, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    mism = torch.zeros(1, dtype=torch.int32, device=dev)
    scales = torch.empty(n // 256, dtype=torch.float32, device=dev)
    C.k_evict_hash(x.data_ptr(), host.data_ptr(), n, dig.data_ptr(), s, a.ctas)  # fill the host copy
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.iters):
        if a.kernel == "evict":
            C.k_evict_hash(x.data_ptr(), host.data_ptr(), n, dig.data_ptr(), s, a.ctas)
        elif a.kernel == "restore":
            C.k_restore_cast(host.data_ptr(), out.data_ptr(), n, 0, 0, 0, 0, s, a.ctas)
        elif a.kernel == "restore_fp8":
            C.k_restore_cast(host.data_ptr(), out.data_ptr(), n, 1, scales.data_ptr(), 0, 0, s, a.ctas)
        elif a.kernel == "hash":
            C.k_hash_device(x.data_ptr(), n, dig.data_ptr(), s, a.ctas)
        else:
            C.k_verify_peer(x.data_ptr(), out.data_ptr(), n, dig.data_ptr(), mism.data_ptr(), s, a.ctas)
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / a.iters
    print(f"{a.kernel}: {n / (ms / 1e3) / 1e9:.2f} GB/s ({ms:.3f} ms per launch, {n} bytes)")


if __name__ == "__main__":
    main()
