"""End-to-end GPU round trips through the public API and an in-process daemon."""

import pytest
import torch

from statespectre_b200 import DedupPolicy, ModelRole, in_process_daemon, offload_context
from statespectre_b200._native import native

pytestmark = pytest.mark.gpu


@pytest.fixture
def gpu_off(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=1024, drain_on_complete=False)
    s = offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="gpu-test")
    yield s.off
    s.close()
    d.stop()


def test_evict_restore_releases_vram_and_roundtrips(gpu_off):
    off = gpu_off
    x = torch.randn(64 << 20, dtype=torch.bfloat16, device="cuda")  # 128 MiB
    ref = x.clone()
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    h = off.evict(x, wait=True)
    torch.cuda.synchronize()
    assert x.numel() == 0
    assert torch.cuda.memory_allocated() <= before - (128 << 20)
    assert h.location() == "pinned"
    y = h.restore()
    assert torch.equal(y, ref)
    assert h.content_hash == native().ssh_hash(ref.cpu().view(torch.uint8).numpy())
    h.discard()


def test_async_evict_prefetch_restore_into_and_verify(gpu_off):
    off = gpu_off
    x = torch.randn(3 << 20, device="cuda")
    ref = x.clone()
    h = off.copy(x)  # async, non-destructive
    h.wait_offloaded()
    assert h.ready()
    p = h.prefetch()
    y = p.wait()
    assert torch.equal(y, ref)
    z = torch.empty_like(ref)
    h.restore_into(z, verify=True)
    assert torch.equal(z, ref)
    w = h.restore(cast="bf16")
    assert torch.equal(w, ref.to(torch.bfloat16))


def test_odd_sizes_and_views(gpu_off):
    off = gpu_off
    for n in (1, 17, 333, 65537):
        x = torch.randint(0, 255, (n,), dtype=torch.uint8, device="cuda")
        h = off.copy(x, wait=True)
        assert torch.equal(h.restore(), x)
    base = torch.randn(1000, 64, device="cuda")
    view = base[:, 3:40]
    h = off.evict(view, compact=True, wait=True)
    assert torch.equal(h.restore(), view.contiguous())
    with pytest.raises(RuntimeError):
        off.evict(view)  # destructive eviction of a view is refused


def test_fp8_restore_cast(gpu_off):
    off = gpu_off
    x = torch.randn(1 << 20, dtype=torch.bfloat16, device="cuda")
    h = off.copy(x, wait=True)
    q, scales = h.restore(cast="fp8_block128")
    deq = (q.float().reshape(-1, 128) * scales[:, None]).reshape(-1)
    torch.testing.assert_close(deq, x.float(), rtol=0.07, atol=1e-2)


def test_batch_evict_restore(gpu_off):
    off = gpu_off
    blocks = [torch.randn(16, 8, 128, dtype=torch.bfloat16, device="cuda") for _ in range(64)]
    refs = [b.clone() for b in blocks]
    hs = off.evict_batch(blocks)
    outs = off.restore_batch(hs)
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)


def test_canonical_evict_seal_restore(gpu_off):
    off = gpu_off
    w = torch.randn(4096, 512, dtype=torch.bfloat16, device="cuda")
    ref = w.clone()
    key = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1, param_name="layer0.w", tensor=w)
    ch = off.canonical_evict(w, key)
    assert ch.action_name == "NEED_D2H_CREATE" and ch.did_d2h
    assert ch.content_hash == off.hash_tensor(ref)
    sealed = off.promote_rollout_version(1)
    assert sealed["tensor_count"] == 1
    out = torch.empty_like(ref)
    ch.restore_into(out)
    assert torch.equal(out, ref)
    # a second replica verifies by device hash without any copy
    key2 = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=2, param_name="layer0.w", tensor=ref)
    c1 = off.canonical_evict(ref.clone(), key2)
    c2 = off.canonical_evict(ref.clone(), key2, dedup_policy=DedupPolicy("device_hash_verified"))
    assert c1.did_d2h and not c2.did_d2h and c2.action_name == "VERIFIED_BY_DEVICE_HASH"


def test_kernel_timing_stamps_transfers(gpu_off):
    """Device-side %globaltimer stamps: one record per instrumented launch,
    with the launch's bytes and a plausible duration."""
    off = gpu_off
    off.enable_kernel_timing()
    _, start = off.kernel_timings()
    x = torch.randn(32 << 20, dtype=torch.bfloat16, device="cuda")  # 64 MiB: zbf16-coded
    f = torch.randint(-2**31, 2**31 - 1, (8 << 20,), dtype=torch.int32, device="cuda")  # 32 MiB int32: uncoded
    hx, hf = off.copy(x, wait=True), off.copy(f, wait=True)
    hx.restore_into(x, wait=True)
    hf.restore_into(f, wait=True)
    torch.cuda.synchronize()
    recs, nxt = off.kernel_timings(start)
    assert nxt >= start + 4  # zbf16 scan, coded K1, hash beside the int32 copy, coded K2
    kinds = {r["kernel"] for r in recs}
    # bf16 moves coded through the SM kernels; int32 moves on the copy engine
    # with its digests computed by the hash kernel beside it
    assert {"zbf16_scan", "k1_evict_zbf16", "k2_restore_zbf16", "k1_hash"} <= kinds, kinds
    for r in recs:
        assert r["ns"] > 0 and r["bytes"] > 0
        gbs = r["bytes"] / r["ns"]
        assert 1.0 < gbs < 20000.0, r  # PCIe kernels tens of GB/s, the scan HBM-rate
    prof = off.kernel_profile(start)
    assert prof["k1_hash"]["bytes"] == 32 << 20
    # the session trace carries the stamped kernels as device-time events
    import json
    import os
    import tempfile

    tp = os.path.join(tempfile.mkdtemp(), "trace.json")
    with off.trace(tp):
        off.copy(x, wait=True).discard()
    evs = json.load(open(tp))["traceEvents"]
    kev = [e for e in evs if e.get("ph") == "X"]
    assert {"zbf16_scan", "k1_evict_zbf16"} <= {e["name"] for e in kev} and all(e["dur"] > 0 for e in kev)
    hx.discard()
    hf.discard()


@pytest.mark.parametrize("uncoded", ["copy_engine", "bulk", "sm"])
@pytest.mark.parametrize("shape,dtype", [((12 << 20) // 4 + 7, torch.float32), ((1 << 20) + 8, torch.float8_e4m3fn),
                                         ((3 << 20) + 5, torch.int16)])
def test_uncoded_forms_roundtrip_with_host_oracle_hash(sock_path, uncoded, shape, dtype):
    """Every way of moving uncoded bytes (copy engine with the hash beside
    it, bulk copies, per-thread K1/K2) is byte-exact and yields the host
    oracle's content hash; odd sizes take the per-thread form."""
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", uncoded=uncoded) as off:
            if dtype == torch.float8_e4m3fn:
                x = torch.randn(shape, device="cuda").to(dtype)
            elif dtype == torch.int16:
                x = torch.randint(-30000, 30000, (shape,), dtype=dtype, device="cuda")
            else:
                x = torch.randn(shape, dtype=dtype, device="cuda")
            ref = x.clone()
            for _ in range(2):
                h = off.evict(x, wait=True)
                assert h.content_hash == native().ssh_hash(ref.cpu().view(torch.uint8).numpy())
                x = h.restore()
                assert torch.equal(x.view(torch.uint8), ref.view(torch.uint8))
                h.discard()
    finally:
        d.stop()


def test_unknown_uncoded_form_is_rejected(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=64, drain_on_complete=False)
    try:
        with pytest.raises(Exception, match="uncoded"):
            offload_context(daemon_addr=sock_path, device="cuda:0", uncoded="dma")
    finally:
        d.stop()


@pytest.mark.parametrize("host_hash_max", [0, 16384])
def test_small_evicts_hash_on_host_or_device_alike(sock_path, host_hash_max):
    """Small uncoded evicts hash their pinned copy on the host (up to
    host_hash_max_bytes) or on the device beside the copy; both give the host
    oracle's content hash, verify on restore, and the same bytes back."""
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", job_name="small-hash",
                             host_hash_max_bytes=host_hash_max) as off:
            for n in (1, 4096, 4097, 16384, 16400, 65536 + 48):
                x = torch.randint(0, 255, (n,), dtype=torch.uint8, device="cuda")
                ref = x.clone()
                h = off.copy(x, wait=True)
                assert h.content_hash == native().ssh_hash(ref.cpu().numpy()), n
                z = torch.empty_like(ref)
                h.restore_into(z, verify=True)
                assert torch.equal(z, ref), n
                h.discard()
            # canonical objects take the same path
            w = torch.randn(2048, dtype=torch.bfloat16, device="cuda")
            k = off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1, param_name="w", tensor=w)
            c = off.canonical_evict(w, k, destructive=False)
            assert c.content_hash == native().ssh_hash(w.cpu().view(torch.uint8).numpy())
    finally:
        d.stop()


@pytest.mark.parametrize("compress_canonical", [True, False])
def test_coded_canonical_objects_round_trip_and_export_raw(sock_path, compress_canonical):
    """bf16 canonical objects of 4 MiB and more cross PCIe zbf16-coded (one
    batch and one single evict); their content hash is the raw bytes' (host
    oracle), canonical restore decodes them (also with the fp32 cast), and
    TCP / FILE pulls from offloadd get the raw bytes. Small and fp32 objects
    stay raw; with compress_canonical off nothing is coded."""
    from statespectre_b200 import RolloutWeightClient

    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", job_name="coded-canon",
                             compress_canonical=compress_canonical) as off:
            g = torch.Generator(device="cuda").manual_seed(3)
            ts = {"big": torch.randn(6 << 20, device="cuda", generator=g).to(torch.bfloat16) * 0.02,
                  "odd": torch.randn((5 << 20) + 8 * 333, device="cuda", generator=g).to(torch.bfloat16),
                  "small": torch.randn(4096, device="cuda", generator=g).to(torch.bfloat16),
                  "f32": torch.randn(3 << 20, device="cuda", generator=g)}
            refs = {n: t.clone() for n, t in ts.items()}
            keys = {n: off.canonical_key(model_role=ModelRole.POLICY_ROLLOUT, model_version=1, param_name=n, tensor=t)
                    for n, t in ts.items()}
            before = off.summary_dict()["coded_canonical"]
            hs = dict(zip(["big", "small", "f32"],
                          off.canonical_evict_batch([(ts[n], keys[n]) for n in ("big", "small", "f32")],
                                                    destructive=False)))
            hs["odd"] = off.canonical_evict(ts["odd"], keys["odd"], destructive=False)
            coded = off.summary_dict()["coded_canonical"] - before
            assert coded == (2 if compress_canonical else 0)
            for n, h in hs.items():
                assert h.content_hash == native().ssh_hash(refs[n].cpu().view(torch.uint8).numpy()), n
                out = torch.empty_like(refs[n])
                h.restore_into(out)
                torch.cuda.synchronize()
                assert torch.equal(out, refs[n]), n
            # the fp32 cast decodes too
            f32 = torch.empty(refs["big"].numel(), dtype=torch.float32, device="cuda")
            ok, msg = off._agent.canonical_restore(hs["big"].object_id, f32.data_ptr(), f32.numel() * 4,
                                                   torch.cuda.current_stream().cuda_stream, True, 3, 0)
            torch.cuda.synchronize()
            assert ok, msg
            assert torch.equal(f32, refs["big"].float())
            off.promote_rollout_version(1)
            for transport in ("tcp", "file"):
                cl = RolloutWeightClient(sock_path, off.job_id, off.launch_epoch, job_name=off.job_name)
                res = cl.sync_latest(transport=transport)
                for n, h in hs.items():
                    assert res["data"][h.object_id] == refs[n].cpu().view(torch.uint8).numpy().tobytes(), (n, transport)
                cl.close()
    finally:
        d.stop()


@pytest.mark.parametrize("uncoded", ["copy_engine", "sm"])
def test_batch_uncoded_items_on_either_form(sock_path, uncoded):
    """A batch that mixes coded bf16 blocks with uncoded ones (fp32, fp8,
    int and an odd-sized block) round-trips byte for byte, with the host
    oracle's content hashes, whether uncoded items are restored by the copy
    engine or by the group's job kernel."""
    d = in_process_daemon(socket=sock_path, arena_mb=512, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", uncoded=uncoded) as off:
            g = torch.Generator(device="cuda").manual_seed(11)
            blocks = [torch.randn(2 << 20, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3)]
            blocks += [torch.randn(1 << 20, device="cuda", generator=g) for _ in range(3)]
            blocks += [torch.randn(3 << 20, device="cuda", generator=g).to(torch.float8_e4m3fn),
                       torch.randint(-9, 9, ((1 << 20) + 3,), dtype=torch.int32, device="cuda"),
                       torch.randint(0, 255, (4 * 1024 + 7,), dtype=torch.uint8, device="cuda")]
            refs = [b.clone() for b in blocks]
            hs = off.evict_batch(blocks)
            assert [h.coded for h in hs[:3]] == [True] * 3 and not any(h.coded for h in hs[3:])
            for h, r in zip(hs, refs):
                assert h.content_hash == native().ssh_hash(r.cpu().view(torch.uint8).numpy())
            outs = off.restore_batch(hs)
            torch.cuda.synchronize()
            for o, r in zip(outs, refs):
                assert torch.equal(o.view(torch.uint8), r.view(torch.uint8))
    finally:
        d.stop()
