"""zf32-coded fp32 evict/restore on the GPU against the host reference codec."""

import time

import pytest
import torch

from statespectre_b200 import in_process_daemon, offload_context
from statespectre_b200._native import native

pytestmark = pytest.mark.gpu

ROW = 131072
CHUNK = 65536


def _case(nbytes, kind, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = nbytes // 4
    if kind == "normal":
        return torch.randn(n, generator=g, device="cuda")
    if kind == "moments":  # Adam second moments: squared gradients
        return (torch.randn(n, generator=g, device="cuda") * 1e-3) ** 2 + 1e-12
    return torch.randn(n, generator=g, device="cuda") * 0.02  # master weights


@pytest.mark.parametrize("kind", ["normal", "moments", "weights"])
@pytest.mark.parametrize("rows", [1, 5, 300])
def test_kernels_match_host_codec(kind, rows):
    """zscan_f32 + evict_zf32 write the host codec's bytes (low plane and the
    stored part of each coded top-half chunk); restore_zf32 brings back the
    original fp32 values; the pre-pass's largest stored length matches."""
    C = native()
    nbytes = rows * ROW
    x = _case(nbytes, kind, seed=rows)
    raw = x.view(torch.uint8).cpu().numpy()
    ref = C.zf32_encode(raw)
    assert ref is not None
    eb = torch.zeros(rows, dtype=torch.uint8, device="cuda")
    fail = torch.zeros(4, dtype=torch.int32, device="cuda")
    maxc = torch.zeros(512, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_zscan_f32(x.data_ptr(), nbytes, eb.data_ptr(), fail.data_ptr(), s, 0, maxc.data_ptr())
    host = torch.zeros(nbytes, dtype=torch.uint8, pin_memory=True)
    C.k_evict_zf32(x.data_ptr(), host.data_ptr(), nbytes, eb.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert int(fail[0].item()) == 0
    got = host.numpy().tobytes()
    longest = 0
    for r in range(rows):
        base = r * ROW
        clen = int.from_bytes(ref[base + CHUNK + 12:base + CHUNK + 16], "little")
        longest = max(longest, clen)
        assert got[base:base + CHUNK + clen] == ref[base:base + CHUNK + clen], r
    assert int(maxc.max().item()) == longest
    assert C.zf32_decode(got) == raw.tobytes()
    out = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    C.k_restore_zf32(host.data_ptr(), out.data_ptr(), nbytes, s, 0)
    # and from device memory (the copy-engine path's staging)
    dev = host.cuda()
    out2 = torch.empty_like(out)
    C.k_restore_zf32(dev.data_ptr(), out2.data_ptr(), nbytes, s, 0)
    torch.cuda.synchronize()
    assert torch.equal(out, x.view(torch.uint8))
    assert torch.equal(out2, x.view(torch.uint8))


def test_scan_fails_on_inf():
    C = native()
    x = torch.randn(4 * ROW // 4, device="cuda")
    x[ROW // 4 * 2 + 17] = float("inf")
    eb = torch.zeros(4, dtype=torch.uint8, device="cuda")
    fail = torch.zeros(4, dtype=torch.int32, device="cuda")
    C.k_zscan_f32(x.data_ptr(), 4 * ROW, eb.data_ptr(), fail.data_ptr(), torch.cuda.current_stream().cuda_stream, 0)
    torch.cuda.synchronize()
    assert int(fail[0].item()) == 1


@pytest.mark.parametrize("coded_evict,coded_restore", [("copy_engine", "copy_engine"), ("sm", "sm"),
                                                         ("copy_engine", "sm"), ("sm", "copy_engine")])
@pytest.mark.parametrize("nbytes", [40 * ROW, 1000 * ROW])
def test_api_forms_are_byte_exact(sock_path, coded_evict, coded_restore, nbytes):
    """fp32 tensors in whole rows move zf32-coded through every transfer
    form; the content hash is that of the fp32 bytes (host oracle); restore,
    restore_into, verified restore and the bf16 cast all agree with the
    original."""
    d = in_process_daemon(socket=sock_path, arena_mb=1024, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", coded_evict=coded_evict,
                             coded_restore=coded_restore) as off:
            x = _case(nbytes, "weights", seed=nbytes // ROW)
            ref = x.clone()
            h = off.evict(x, wait=True)
            assert h.coded
            assert h.content_hash == native().ssh_hash(ref.view(torch.uint8).cpu().numpy())
            assert torch.equal(h.restore().view(torch.int32), ref.view(torch.int32))
            z = torch.empty_like(ref)
            h.restore_into(z, verify=True)
            assert torch.equal(z.view(torch.int32), ref.view(torch.int32))
            assert torch.equal(h.restore(verify=True).view(torch.int32), ref.view(torch.int32))
            b = h.restore(cast="bf16")
            assert b.dtype == torch.bfloat16 and torch.equal(b, ref.to(torch.bfloat16))
            h.discard()
    finally:
        d.stop()


def test_compare_digests_counts_changed_chunks():
    """The check behind a verified zf32 restore: digests of the decoded bytes
    against the evict's, one count per differing 64 KiB chunk."""
    C = native()
    x = _case(16 * ROW, "normal", seed=3)
    y = x.clone()
    y.view(torch.uint8)[5] ^= 0xFF
    y.view(torch.uint8)[7 * CHUNK + 9] ^= 0x01
    s = torch.cuda.current_stream().cuda_stream
    n = 32
    dx = torch.zeros(n, dtype=torch.int64, device="cuda")
    dy = torch.zeros(n, dtype=torch.int64, device="cuda")
    C.k_hash_device(x.data_ptr(), 16 * ROW, dx.data_ptr(), s, 0)
    C.k_hash_device(y.data_ptr(), 16 * ROW, dy.data_ptr(), s, 0)
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.k_compare_digests(dx.data_ptr(), dy.data_ptr(), n, mism.data_ptr(), s)
    C.k_compare_digests(dx.data_ptr(), dx.data_ptr(), n, mism.data_ptr(), s)
    torch.cuda.synchronize()
    assert int(mism.item()) == 2


def test_coded_fp32_survives_drain_and_readback(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0) as off:
            x = _case(64 * ROW, "moments", seed=11)
            ref = x.clone()
            h = off.copy(x, wait=True)
            assert h.coded
            for _ in range(200):
                if h.location() != "pinned":
                    break
                time.sleep(0.01)
            assert h.location() == "pageable"
            assert torch.equal(h.restore().view(torch.int32), ref.view(torch.int32))
    finally:
        d.stop()


def test_batch_restore_of_zf32_runs(sock_path):
    """Runs evicted singly in zf32 come back through restore_batch next to
    zbf16 and raw runs."""
    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0") as off:
            xs = [_case(32 * ROW, "normal", seed=20), torch.randn(8 << 20, device="cuda").to(torch.bfloat16),
                  torch.randint(0, 9, (1 << 20,), dtype=torch.int32, device="cuda"), _case(40 * ROW, "weights", 21)]
            refs = [x.clone() for x in xs]
            hs = [off.copy(x, wait=True) for x in xs]
            assert [h.coded for h in hs] == [True, True, False, True]
            outs = [torch.empty_like(r) for r in refs]
            off.restore_batch(hs, outs)
            torch.cuda.synchronize()
            for o, r in zip(outs, refs):
                assert torch.equal(o.view(torch.uint8), r.view(torch.uint8))
    finally:
        d.stop()


def test_compress_off_and_copy_engine_mode_keep_fp32_raw(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        for kw in ({"compress": False}, {"engine": "copy_engine"}):
            with offload_context(daemon_addr=sock_path, device="cuda:0", **kw) as off:
                x = _case(16 * ROW, "normal", seed=4)
                h = off.copy(x, wait=True)
                assert not h.coded and torch.equal(h.restore(), x)
                h.discard()
    finally:
        d.stop()
