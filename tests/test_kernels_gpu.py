"""Numerics of the sm_100a kernels against host oracles.

Copies must be byte-exact; chunk digests must equal the host implementation
of ssh128; casts are compared with a plain PyTorch fp32 reference of the same
operation.
"""

import numpy as np
import pytest
import torch

from statespectre_b200._native import native

pytestmark = pytest.mark.gpu

SIZES = [1, 15, 16, 17, 4096, 65535, 65536, 65537, 17 * 333 * 4, (1 << 22) + 13, 3 << 20]


def _pinned(n):
    t = torch.empty(max(n, 1), dtype=torch.uint8, pin_memory=True)
    return t


def _dev_ptr_of_pinned(t):
    # torch pinned memory is host-mapped under UVA: the host pointer is valid on the device.
    return t.data_ptr()


def _host_digests(buf: torch.Tensor, n: int):
    return native().ssh_digests(buf[:n].numpy())


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("offset", [0, 3])
def test_evict_hash_bytes_and_digests(n, offset):
    C = native()
    src_full = torch.randint(0, 256, (n + offset,), dtype=torch.uint8, device="cuda")
    src = src_full[offset:]
    dst = _pinned(n + 16)
    nd = (n + 65535) // 65536
    dig = torch.zeros(max(nd, 1), dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_evict_hash(src.data_ptr(), _dev_ptr_of_pinned(dst), n, dig.data_ptr(), s, 0)
    torch.cuda.synchronize()
    host = src.cpu()
    assert torch.equal(dst[:n], host)
    got = [int(v) & 0xFFFFFFFFFFFFFFFF for v in dig.cpu().tolist()[:nd]]
    assert got == _host_digests(host, n)


@pytest.mark.parametrize("n", [65536 * 5 + 4096, 1 << 20, (1 << 24) + 48])
def test_hash_device_and_fold_match_host(n):
    C = native()
    x = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    nd = (n + 65535) // 65536
    dig = torch.zeros(nd, dtype=torch.int64, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_hash_device(x.data_ptr(), n, dig.data_ptr(), s, 0)
    C.k_fold_digests(dig.data_ptr(), nd, n, out.data_ptr(), s)
    torch.cuda.synchronize()
    lo, hi = [int(v) & 0xFFFFFFFFFFFFFFFF for v in out.cpu().tolist()]
    assert (lo, hi) == C.ssh_hash(x.cpu().numpy())


@pytest.mark.parametrize("n", SIZES)
def test_restore_plain_and_verify(n):
    C = native()
    host = torch.randint(0, 256, (n + 16,), dtype=torch.uint8).pin_memory()
    dst = torch.zeros(n, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    expect = torch.tensor(np.array(_host_digests(host, n), dtype=np.uint64).view(np.int64), device="cuda")
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.k_restore_cast(host.data_ptr(), dst.data_ptr(), n, 0, 0, expect.data_ptr(), mism.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), host[:n])
    assert int(mism.item()) == 0
    # corrupt one byte of the source: exactly one chunk must fail verification
    host[n // 2] ^= 0xFF
    mism.zero_()
    C.k_restore_cast(host.data_ptr(), dst.data_ptr(), n, 0, 0, expect.data_ptr(), mism.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert int(mism.item()) == 1


def _fp8_reference(x: torch.Tensor):
    """fp32 reference of 1x128 block quantization (OCP e4m3, saturating)."""
    xf = x.float().reshape(-1)
    pad = (-xf.numel()) % 128
    xp = torch.cat([xf, xf.new_zeros(pad)]).reshape(-1, 128)
    amax = xp.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    inv = torch.where(amax > 0, 448.0 / amax, torch.ones_like(amax))
    q = (xp * inv[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.reshape(-1)[: xf.numel()], scale


@pytest.mark.parametrize("nelem", [128, 4096, 65536 * 3, (1 << 20) + 256])
def test_restore_cast_bf16_to_fp8(nelem):
    C = native()
    x = (torch.randn(nelem, generator=torch.Generator().manual_seed(nelem)) * 3).to(torch.bfloat16)
    host = x.view(torch.uint8).pin_memory()
    out = torch.empty(nelem, dtype=torch.float8_e4m3fn, device="cuda")
    scales = torch.empty((nelem + 127) // 128, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_restore_cast(host.data_ptr(), out.data_ptr(), nelem * 2, 1, scales.data_ptr(), 0, 0, s, 0)
    torch.cuda.synchronize()
    q_ref, s_ref = _fp8_reference(x)
    torch.testing.assert_close(scales.cpu(), s_ref, rtol=0, atol=0)
    got = out.cpu().float()
    # codes equal the fp32 reference's except for rare one-step rounding
    # differences (subnormal and tie cases of the scaled input)
    step = (out.cpu().view(torch.uint8).int() - q_ref.view(torch.uint8).int()).abs()
    assert step.max().item() <= 1
    assert (step != 0).float().mean().item() < 5e-3
    deq = (got.reshape(-1, 128) * scales.cpu()[:, None]).reshape(-1)
    torch.testing.assert_close(deq, x.float(), rtol=0.07, atol=1e-2)


@pytest.mark.parametrize("nelem", [4, 4096, 65536 + 8])
def test_restore_cast_fp32_bf16_roundtrip(nelem):
    C = native()
    s = torch.cuda.current_stream().cuda_stream
    x = torch.randn(nelem)
    host = x.view(torch.uint8).pin_memory()
    out = torch.empty(nelem, dtype=torch.bfloat16, device="cuda")
    C.k_restore_cast(host.data_ptr(), out.data_ptr(), nelem * 4, 2, 0, 0, 0, s, 0)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), x.to(torch.bfloat16))
    if nelem % 8 == 0:
        xb = torch.randn(nelem).to(torch.bfloat16)
        hb = xb.view(torch.uint8).pin_memory()
        out32 = torch.empty(nelem, dtype=torch.float32, device="cuda")
        C.k_restore_cast(hb.data_ptr(), out32.data_ptr(), nelem * 2, 3, 0, 0, 0, s, 0)
        torch.cuda.synchronize()
        assert torch.equal(out32.cpu(), xb.float())


def test_quant_fp8_standalone():
    C = native()
    nelem = 128 * 1000 + 64
    x = (torch.randn(nelem, device="cuda") * 5).to(torch.bfloat16)
    out = torch.empty(nelem, dtype=torch.float8_e4m3fn, device="cuda")
    scales = torch.empty((nelem + 127) // 128, dtype=torch.float32, device="cuda")
    C.k_quant_fp8(x.data_ptr(), out.data_ptr(), scales.data_ptr(), nelem, torch.cuda.current_stream().cuda_stream, 0)
    torch.cuda.synchronize()
    q_ref, s_ref = _fp8_reference(x.cpu())
    torch.testing.assert_close(scales.cpu(), s_ref, rtol=0, atol=0)
    got, ref = out.cpu(), q_ref
    diff = got.float() != ref.float()
    assert diff.float().mean().item() < 5e-3
    # every difference is a one-step rounding difference of the e4m3 code
    codes_g = got.view(torch.uint8)[diff].int() & 0x7F
    codes_r = ref.view(torch.uint8)[diff].int() & 0x7F
    assert (codes_g - codes_r).abs().max().item() <= 1 if diff.any() else True


def test_verify_peer_same_device_counts_mismatches():
    C = native()
    n = (1 << 20) + 64 * 16
    a = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    b = a.clone()
    b[100] ^= 1
    b[n - 1] ^= 1
    nd = (n + 65535) // 65536
    dig = torch.zeros(nd, dtype=torch.int64, device="cuda")
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.k_verify_peer(a.data_ptr(), b.data_ptr(), n, dig.data_ptr(), mism.data_ptr(),
                    torch.cuda.current_stream().cuda_stream, 0)
    torch.cuda.synchronize()
    assert int(mism.item()) == 2
    assert [int(v) & 0xFFFFFFFFFFFFFFFF for v in dig.cpu().tolist()] == native().ssh_digests(a.cpu().numpy())


BULK_SIZES = [16, 4096, 65536, 65536 + 16, 3 * 32768 + 48, (1 << 22) + 4080, 33 << 20]


@pytest.mark.parametrize("n", BULK_SIZES)
@pytest.mark.parametrize("ctas", [0, 3])
def test_evict_bulk_bytes_and_digests(n, ctas):
    """Bulk-copy K1: device -> host-mapped pinned memory through shared
    memory, digests from the staged bytes; equal to the host oracle and to the
    per-thread K1."""
    C = native()
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = _pinned(n + 16)
    dst.fill_(0xA5)
    nd = (n + 65535) // 65536
    dig = torch.zeros(nd, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_evict_bulk(src.data_ptr(), _dev_ptr_of_pinned(dst), n, dig.data_ptr(), err.data_ptr(), s, ctas)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    host = src.cpu()
    assert torch.equal(dst[:n], host)
    assert torch.all(dst[n:] == 0xA5)  # nothing written past the end
    got = [int(v) & 0xFFFFFFFFFFFFFFFF for v in dig.cpu().tolist()]
    assert got == _host_digests(host, n)
    dig2 = torch.zeros_like(dig)
    C.k_evict_hash(src.data_ptr(), _dev_ptr_of_pinned(dst), n, dig2.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert torch.equal(dig, dig2)


@pytest.mark.parametrize("n", BULK_SIZES)
def test_evict_bulk_without_hash_and_restore_bulk(n):
    C = native()
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    host = _pinned(n)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_evict_bulk(src.data_ptr(), _dev_ptr_of_pinned(host), n, 0, err.data_ptr(), s, 0)
    back = torch.full((n + 16,), 0x5A, dtype=torch.uint8, device="cuda")
    C.k_restore_bulk(_dev_ptr_of_pinned(host), back.data_ptr(), n, err.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(host[:n], src.cpu())
    assert torch.equal(back[:n], src)
    assert torch.all(back[n:] == 0x5A)


def test_bulk_forms_reject_unaligned_arguments():
    C = native()
    a = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    h = _pinned(1 << 16)
    s = torch.cuda.current_stream().cuda_stream
    for src, dst, n in ((a.data_ptr() + 1, h.data_ptr(), 4096), (a.data_ptr(), h.data_ptr(), 4095)):
        with pytest.raises(RuntimeError):
            C.k_evict_bulk(src, dst, n, 0, 0, s, 0)
        with pytest.raises(RuntimeError):
            C.k_restore_bulk(dst, src, n, 0, s, 0)


@pytest.mark.parametrize("n", [16, 65536 * 3 + 4096, (1 << 24) + 48, 200 << 20])
@pytest.mark.parametrize("stages", [2, 3, 4])
def test_hash_stream_shapes_match_one_pass_and_host(n, stages):
    """The K4-pipeline hash in each block shape equals the one-pass kernel and
    the host oracle; hash_device (which picks the form) agrees too."""
    C = native()
    x = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    nd = (n + 65535) // 65536
    a, b, c = (torch.zeros(nd, dtype=torch.int64, device="cuda") for _ in range(3))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_hash_stream(x.data_ptr(), n, a.data_ptr(), err.data_ptr(), s, 0, stages)
    C.k_hash_onepass(x.data_ptr(), n, b.data_ptr(), s, 0)
    C.k_hash_device(x.data_ptr(), n, c.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(a, b) and torch.equal(b, c)
    if n <= (1 << 24) + 48:
        assert [int(v) & 0xFFFFFFFFFFFFFFFF for v in b.cpu().tolist()] == _host_digests(x.cpu(), n)
