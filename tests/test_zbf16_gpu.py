"""zbf16-coded evict/restore on the GPU against the host reference codec."""

import pytest
import torch

from statespectre_b200 import in_process_daemon, offload_context
from statespectre_b200._native import native

pytestmark = pytest.mark.gpu

CHUNK = 65536
M = 2**64 - 1


def _case(nbytes, kind, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = nbytes // 2
    if kind == "normal":
        x = torch.randn(n, generator=g, device="cuda")
    elif kind == "weights":
        x = torch.randn(n, generator=g, device="cuda") * 0.02
    else:  # wide: 5 % of the values spread over 40 binades
        x = torch.randn(n, generator=g, device="cuda")
        mask = torch.rand(n, generator=g, device="cuda") < 0.05
        x[mask] = torch.exp2(torch.randint(-40, 0, (int(mask.sum()),), generator=g, device="cuda").float())
    return x.to(torch.bfloat16)


def _scan(x, nbytes):
    C = native()
    nch = (nbytes + CHUNK - 1) // CHUNK
    eb = torch.zeros(nch, dtype=torch.uint8, device="cuda")
    fail = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_zscan(x.data_ptr(), nbytes, eb.data_ptr(), fail.data_ptr(), s, 0)
    torch.cuda.synchronize()
    return eb, int(fail.item())


@pytest.mark.parametrize("kind", ["normal", "weights", "wide"])
@pytest.mark.parametrize("nbytes", [4096, CHUNK, 7 * CHUNK + 4096, 64 << 20])
def test_evict_z_matches_host_codec_and_restores(kind, nbytes):
    C = native()
    x = _case(nbytes, kind, seed=nbytes)
    raw = x.view(torch.uint8).cpu().numpy()
    eb, fail = _scan(x, nbytes)
    ref = C.zbf16_encode(raw)
    assert fail == (ref is None)
    assert ref is not None
    host = torch.zeros(nbytes, dtype=torch.uint8, pin_memory=True)
    dig = torch.zeros((nbytes + CHUNK - 1) // CHUNK, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    C.k_evict_z(x.data_ptr(), host.data_ptr(), nbytes, eb.data_ptr(), dig.data_ptr(), s, 0)
    torch.cuda.synchronize()
    got = host.numpy().tobytes()
    assert C.zbf16_decode(got) == raw.tobytes()
    assert C.zbf16_coded_bytes(got) == C.zbf16_coded_bytes(ref)
    # every chunk's coded bytes equal the reference's (same window, same order)
    nch = (nbytes + CHUNK - 1) // CHUNK
    for c in range(nch):
        base = c * CHUNK
        length = min(CHUNK, nbytes - base)
        clen = length if (c == nch - 1 and length < 4096) else int.from_bytes(ref[base + 12:base + 16], "little")
        assert got[base:base + clen] == ref[base:base + clen], c
    # digests describe the raw bytes
    want = torch.zeros_like(dig)
    C.k_hash_device(x.data_ptr(), nbytes, want.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert torch.equal(dig, want)
    # decode on the GPU, with digest verification
    out = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    mism = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.k_restore_z(host.data_ptr(), out.data_ptr(), nbytes, 0, 0, dig.data_ptr(), mism.data_ptr(), s, 0)
    torch.cuda.synchronize()
    assert mism.item() == 0
    assert torch.equal(out, x.view(torch.uint8))


def test_random_bits_fail_the_scan():
    nbytes = 1 << 20
    x = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda").view(torch.bfloat16)
    _, fail = _scan(x, nbytes)
    assert fail == 1


@pytest.mark.parametrize("cast", [1, 3])
def test_restore_z_casts_match_uncoded_restore(cast):
    C = native()
    nbytes = 4 << 20
    x = _case(nbytes, "weights", seed=11)
    ref = C.zbf16_encode(x.view(torch.uint8).cpu().numpy())
    host = torch.frombuffer(bytearray(ref), dtype=torch.uint8).pin_memory()
    raw_host = x.view(torch.uint8).cpu().pin_memory()
    s = torch.cuda.current_stream().cuda_stream
    n = nbytes // 2
    if cast == 1:
        a = torch.empty(n, dtype=torch.uint8, device="cuda")
        b = torch.empty(n, dtype=torch.uint8, device="cuda")
        sa = torch.empty(n // 128, dtype=torch.float32, device="cuda")
        sb = torch.empty(n // 128, dtype=torch.float32, device="cuda")
        C.k_restore_z(host.data_ptr(), a.data_ptr(), nbytes, 1, sa.data_ptr(), 0, 0, s, 0)
        C.k_restore_cast(raw_host.data_ptr(), b.data_ptr(), nbytes, 1, sb.data_ptr(), 0, 0, s, 0)
        torch.cuda.synchronize()
        assert torch.equal(a, b) and torch.equal(sa, sb)
    else:
        a = torch.empty(n, dtype=torch.float32, device="cuda")
        C.k_restore_z(host.data_ptr(), a.data_ptr(), nbytes, 3, 0, 0, 0, s, 0)
        torch.cuda.synchronize()
        assert torch.equal(a, x.float())


@pytest.fixture
def zsession(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    s = offload_context(daemon_addr=sock_path, device="cuda:0", rank=0)
    yield s.off
    s.close()
    d.stop()


def test_api_codes_bf16_and_round_trips(zsession):
    off = zsession
    x = _case(32 << 20, "weights", seed=2)
    ref = x.clone()
    h = off.evict(x, wait=True)
    assert h.coded
    assert h.content_hash == native().ssh_hash(ref.view(torch.uint8).cpu().numpy())
    y = h.restore()
    assert torch.equal(y, ref)
    z = torch.empty_like(ref)
    h.restore_into(z, verify=True)
    assert torch.equal(z, ref)
    q, sc = h.restore(cast="fp8_block128")
    assert q.dtype == torch.float8_e4m3fn and sc.numel() == ref.numel() // 128
    h.discard()
    # fp32 in whole 128 KiB rows moves zf32-coded; other fp32 sizes, integer
    # and small tensors move uncoded
    f = torch.randn(8 << 20, device="cuda")
    hf = off.copy(f, wait=True)
    assert hf.coded and torch.equal(hf.restore(), f)
    f2 = torch.randn((8 << 20) + 4, device="cuda")
    hf2 = off.copy(f2, wait=True)
    assert not hf2.coded and torch.equal(hf2.restore(), f2)
    i32 = torch.randint(0, 1000, (8 << 20,), dtype=torch.int32, device="cuda")
    hi = off.copy(i32, wait=True)
    assert not hi.coded and torch.equal(hi.restore(), i32)
    small = _case(1 << 20, "weights")
    hs = off.copy(small, wait=True)
    assert not hs.coded and torch.equal(hs.restore(), small)


def test_coded_object_survives_drain_and_readback(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0) as off:
            x = _case(16 << 20, "normal", seed=9)
            ref = x.clone()
            h = off.copy(x, wait=True)
            assert h.coded
            for _ in range(200):  # drain_on_complete moves it to pageable memory
                if h.location() != "pinned":
                    break
                import time
                time.sleep(0.01)
            assert h.location() == "pageable"
            assert torch.equal(h.restore(), ref)
    finally:
        d.stop()


def test_compress_off_moves_uncoded(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, compress=False) as off:
            x = _case(16 << 20, "normal", seed=4)
            h = off.copy(x, wait=True)
            assert not h.coded and torch.equal(h.restore(), x)
    finally:
        d.stop()


def test_batch_evict_codes_kv_blocks(zsession):
    off = zsession
    cache = _case(16 * (4 << 20), "normal", seed=21).view(16, -1)  # 16 KV blocks of 4 MiB
    ref = cache.clone()
    blocks = [cache[i] for i in range(0, 16, 2)]
    hs = off.evict_batch(blocks)
    assert all(h.coded for h in hs)
    for b in blocks:
        b.zero_()
    off.restore_batch(hs, blocks)
    torch.cuda.synchronize()
    assert torch.equal(cache, ref)
    for h in hs:
        h.discard()


def test_batch_groups_mixed_items(sock_path):
    """Several reservation groups, coded and uncoded items side by side."""
    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, batch_group_bytes=8 << 20) as off:
            xs = [_case(4 << 20, "weights", seed=40 + i) for i in range(6)]
            xs.append(torch.randn(1 << 20, device="cuda"))          # fp32: uncoded
            xs.append(_case(1 << 20, "normal", seed=50))            # below the coding floor
            rb = torch.randint(0, 256, (4 << 20,), dtype=torch.uint8, device="cuda")
            xs.append(rb.view(torch.bfloat16))                      # random bits: scan fails
            refs = [x.clone() for x in xs]
            hs = off.evict_batch(xs)
            assert [h.coded for h in hs] == [True] * 6 + [False, False, False]
            for x in xs:
                x.zero_()
            off.restore_batch(hs, xs)
            torch.cuda.synchronize()
            for x, r in zip(xs, refs):  # bytes: the random-bits item holds NaNs
                assert torch.equal(x.view(torch.uint8), r.view(torch.uint8))
            for h in hs:
                h.discard()
    finally:
        d.stop()


@pytest.mark.parametrize("coded_evict,coded_restore", [("sm", "copy_engine"), ("sm", "sm"),
                                                         ("copy_engine", "copy_engine"), ("copy_engine", "sm")])
@pytest.mark.parametrize("n", [(8 << 20), (40 << 20) + 4096 + 16 * 37, 1024 * 65536 + 2048])
def test_coded_transfer_forms_are_byte_exact(sock_path, coded_evict, coded_restore, n):
    """A zbf16-coded run is byte-exact through every combination of the
    transfer forms: K1 coding into the host run or into device staging moved
    by the copy engine, and K2 decoding from host memory or from staging
    filled by the copy engine; the content hash equals the host oracle's.
    Sizes cover several pieces, a ragged last chunk and a short raw tail."""
    from statespectre_b200 import in_process_daemon, offload_context

    d = in_process_daemon(socket=sock_path, arena_mb=4096, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", coded_restore=coded_restore,
                             coded_evict=coded_evict) as off:
            x = torch.randn(n // 2, dtype=torch.bfloat16, device="cuda")
            x.view(-1)[::997] = 1e-30  # a few escapes per chunk
            ref = x.clone()
            h = off.evict(x, wait=True)
            assert h.coded
            assert h.content_hash == native().ssh_hash(ref.cpu().view(torch.uint8).numpy())
            y = h.restore()
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
            z = torch.empty_like(ref)
            h.restore_into(z)
            assert torch.equal(z.view(torch.int16), ref.view(torch.int16))
            h.discard()
    finally:
        d.stop()


@pytest.mark.parametrize("ring", [{}, {"stage_depth": 3, "stage_piece_chunks": 48, "stage_ctas": 37}])
def test_copy_engine_evicts_and_restores_back_to_back_share_staging(sock_path, ring):
    """Asynchronous coded evicts and restores issued back to back on one
    session share the device staging: each waits for the last reader of a
    staging buffer before writing it, so every tensor comes back intact
    (default ring, and an odd-sized ring of small pieces whose turns wrap
    across operations)."""
    from statespectre_b200 import in_process_daemon, offload_context

    d = in_process_daemon(socket=sock_path, arena_mb=2048, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", coded_restore="copy_engine",
                             coded_evict="copy_engine", **ring) as off:
            xs = [torch.randn((48 << 20) // 2 + 4096 * i, dtype=torch.bfloat16, device="cuda") for i in range(4)]
            refs = [x.clone() for x in xs]
            hs = [off.copy(x) for x in xs]  # asynchronous
            outs = [torch.empty_like(r) for r in refs]
            for h, o in zip(hs, outs):
                h.wait_offloaded()
                h.restore_into(o, wait=False)
            h2 = off.copy(xs[0])  # an evict queued behind the restores
            torch.cuda.synchronize()
            h2.wait_offloaded()
            for o, r in zip(outs, refs):
                assert torch.equal(o.view(torch.int16), r.view(torch.int16))
            back = torch.empty_like(refs[0])
            h2.restore_into(back)
            assert torch.equal(back.view(torch.int16), refs[0].view(torch.int16))
    finally:
        d.stop()
