"""Launch one data-path kernel a few times on a fixed case (for ncu captures).

    python -m statespectre_b200.ops.profile_case --kernel evict --mb 512 --iters 3

Kernels: evict (K1, device -> pinned + ssh128), restore (K2, pinned ->
device), restore_fp8 (K2 with the bf16 -> fp8 1x128 cast), evict_z /
restore_z (coded K1 / K2 to and from host memory), evict_z_stage /
restore_z_stage (the same coding into and decoding from device memory, the
passes of the copy-engine coded paths), zscan_f32 / evict_zf32 / restore_zf32
and their _stage forms (zf32 coding of an fp32 tensor), evict_bulk /
restore_bulk (K1 / K2 as bulk copies through shared memory), hash (device
ssh128, the library's choice of form), hash_onepass (the per-thread-load
hash kernel), hash_stream (ssh128 through the K4 bulk-copy pipeline), verify (K3
local vs second buffer), push / push_fp8 (K4 into a second buffer, raw or
quantized; --peer 1 puts that buffer on cuda:1 so the stores cross NVLink).
The case is larger than the 126 MB L2 so DRAM counters are meaningful; it
holds about 2x --mb of device memory and --mb of pinned host memory.
"""

from __future__ import annotations

import argparse

import torch

from .._native import native


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True, choices=["evict", "restore", "restore_fp8", "hash", "hash_onepass",
                                                          "hash_stream", "verify", "push", "push_fp8", "zscan",
                                                          "evict_z", "restore_z", "evict_bulk", "restore_bulk",
                                                          "evict_z_stage", "restore_z_stage", "zscan_f32",
                                                          "evict_zf32", "restore_zf32", "evict_zf32_stage",
                                                          "restore_zf32_stage"])
    ap.add_argument("--mb", type=int, default=512)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--ctas", type=int, default=0)
    ap.add_argument("--stages", type=int, default=0, help="hash_stream: 2, 3 or 4 staged halves per CTA (0: default)")
    ap.add_argument("--peer", type=int, default=-1,
                    help="device of the push destination or of the copy verify compares against (default: same GPU)")
    ap.add_argument("--items", type=int, default=64, help="push: split the buffer into this many tensors")
    ap.add_argument("--delta", type=int, default=0,
                    help="push: 1 = delta mode with the destination table cleared before each launch "
                         "(every chunk stored after its digest), 2 = delta mode with nothing changed")
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
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    zeb = torch.zeros((n + 65535) // 65536, dtype=torch.uint8, device=dev)
    stage = None
    if a.kernel in ("zscan", "evict_z", "restore_z", "evict_z_stage", "restore_z_stage"):
        # zbf16: window bases, then the coded host copy (and a device copy of it)
        C.k_zscan(x.data_ptr(), n, zeb.data_ptr(), err.data_ptr(), s, 0)
        C.k_evict_z(x.data_ptr(), host.data_ptr(), n, zeb.data_ptr(), dig.data_ptr(), s, a.ctas)
        if a.kernel == "restore_z_stage":
            stage = torch.empty(n, dtype=torch.uint8, device=dev)
            stage.copy_(host)
    xf = None
    if "f32" in a.kernel:
        # zf32: an fp32 tensor of the same byte size (N(0, 0.02): master
        # weights), its row window bases and coded host copy (and a device copy)
        xf = torch.randn(n // 4, device=dev) * 0.02
        C.k_zscan_f32(xf.data_ptr(), n, zeb.data_ptr(), err.data_ptr(), s, 0)
        C.k_evict_zf32(xf.data_ptr(), host.data_ptr(), n, zeb.data_ptr(), s, a.ctas)
        if a.kernel == "restore_zf32_stage":
            stage = torch.empty(n, dtype=torch.uint8, device=dev)
            stage.copy_(host)
    if a.kernel == "verify":
        # K3 compares x with a second copy: on this GPU, or with --peer on that
        # GPU (plain peer loads over NVLink); the copy goes through host memory
        if a.peer >= 0:
            C.enable_peer(a.peer)
            out = torch.empty(n, dtype=torch.uint8, device=torch.device("cuda", a.peer))
        out.copy_(x.view(torch.uint8).cpu())
        torch.cuda.synchronize()
    pusher = None
    if a.kernel.startswith("push"):
        from ..parallel.weight_sync import WeightLayout, WeightPusher
        params = {f"x{i}": v for i, v in enumerate(x.view(a.items, -1))}
        layout = WeightLayout.from_params(params, "fp8" if a.kernel == "push_fp8" else "bf16")
        if a.peer >= 0:
            C.enable_peer(a.peer)
            dst = torch.empty(layout.total_bytes, dtype=torch.uint8, device=torch.device("cuda", a.peer))
        else:
            dst = torch.empty(layout.total_bytes, dtype=torch.uint8, device=dev)
        pusher = WeightPusher(params, layout, dst.data_ptr(), dev, delta=a.delta > 0, ctas=a.ctas)
        if a.delta == 2:
            pusher.push()
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
        elif a.kernel == "hash_onepass":
            C.k_hash_onepass(x.data_ptr(), n, dig.data_ptr(), s, a.ctas)
        elif a.kernel == "evict_bulk":
            C.k_evict_bulk(x.data_ptr(), host.data_ptr(), n, dig.data_ptr(), err.data_ptr(), s, a.ctas)
        elif a.kernel == "restore_bulk":
            C.k_restore_bulk(host.data_ptr(), out.data_ptr(), n, err.data_ptr(), s, a.ctas)
        elif a.kernel == "zscan":
            C.k_zscan(x.data_ptr(), n, zeb.data_ptr(), err.data_ptr(), s, 0)
        elif a.kernel == "evict_z":
            C.k_evict_z(x.data_ptr(), host.data_ptr(), n, zeb.data_ptr(), dig.data_ptr(), s, a.ctas)
        elif a.kernel == "restore_z":
            C.k_restore_z(host.data_ptr(), out.data_ptr(), n, 0, 0, 0, 0, s, a.ctas)
        elif a.kernel == "evict_z_stage":  # coding into device memory (the copy-engine evict's staging pass)
            C.k_evict_z(x.data_ptr(), out.data_ptr(), n, zeb.data_ptr(), dig.data_ptr(), s, a.ctas)
        elif a.kernel == "restore_z_stage":  # decoding from device memory (the copy-engine restore's pass)
            C.k_restore_z(stage.data_ptr(), out.data_ptr(), n, 0, 0, 0, 0, s, a.ctas)
        elif a.kernel == "zscan_f32":
            C.k_zscan_f32(xf.data_ptr(), n, zeb.data_ptr(), err.data_ptr(), s, 0)
        elif a.kernel == "evict_zf32":
            C.k_evict_zf32(xf.data_ptr(), host.data_ptr(), n, zeb.data_ptr(), s, a.ctas)
        elif a.kernel == "restore_zf32":
            C.k_restore_zf32(host.data_ptr(), out.data_ptr(), n, s, a.ctas)
        elif a.kernel == "evict_zf32_stage":
            C.k_evict_zf32(xf.data_ptr(), out.data_ptr(), n, zeb.data_ptr(), s, a.ctas)
        elif a.kernel == "restore_zf32_stage":
            C.k_restore_zf32(stage.data_ptr(), out.data_ptr(), n, s, a.ctas)
        elif a.kernel == "hash_stream":
            C.k_hash_stream(x.data_ptr(), n, dig.data_ptr(), err.data_ptr(), s, a.ctas, a.stages)
        elif pusher is not None:
            if a.delta == 1:
                pusher.invalidate()
            pusher.push()
        else:
            C.k_verify_peer(x.data_ptr(), out.data_ptr(), n, dig.data_ptr(), mism.data_ptr(), s, a.ctas)
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / a.iters
    if a.kernel == "verify" and int(mism.item()) != 0:
        raise SystemExit(f"verify: {int(mism.item())} vectors differ")
    if int(err.item()) != 0 or (pusher is not None and pusher.result()["error"]):
        code = int(err.item()) if pusher is None else pusher.result()["error"]
        raise SystemExit(f"{a.kernel}: device status {code}")
    if a.kernel in ("restore_zf32", "restore_zf32_stage") and not torch.equal(out.view(torch.float32), xf):
        raise SystemExit(f"{a.kernel}: decoded values differ")
    if a.kernel in ("hash", "hash_stream", "evict_bulk"):  # the digests must equal the one-pass kernel's
        ref = torch.zeros_like(dig)
        C.k_hash_onepass(x.data_ptr(), n, ref.data_ptr(), s, 0)
        torch.cuda.synchronize()
        if not torch.equal(ref, dig):
            raise SystemExit(f"{a.kernel}: digests differ from the one-pass hash")
    print(f"{a.kernel}: {n / (ms / 1e3) / 1e9:.2f} GB/s ({ms:.3f} ms per launch, {n} bytes)")


if __name__ == "__main__":
    main()
