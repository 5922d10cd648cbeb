"""K4 weight-sync push and the pipelined chunk-digest pass on one GPU.

The destination buffer lives on the same GPU here; the kernel's stores are
plain global stores either way. Numerics are checked against plain PyTorch
fp32 references and the host ssh128 oracle.
"""

import pytest
import torch

from statespectre_b200 import in_process_daemon, offload_context
from statespectre_b200._native import native
from statespectre_b200.parallel.weight_sync import (RolloutWeights, TrainerWeightSync, WeightLayout,
                                                     WeightPusher)

pytestmark = pytest.mark.gpu

M = 2**64 - 1


def _params(seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shapes = {"embed": (1000, 256), "q": (512, 512), "bias": (24,), "norm": (256,), "odd": (3, 5, 16),
              "big": (2048, 1536)}
    return {n: (torch.randn(s, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for n, s in shapes.items()}


def _host_hash(t):
    return native().ssh_hash(t.contiguous().view(torch.uint8).cpu().numpy())


def _ref_fp8(x: torch.Tensor):
    """fp32 reference of 1x128 block quantization: scale = amax/448."""
    b = x.float().reshape(-1, 128)
    amax = b.abs().amax(dim=1, keepdim=True)
    inv = torch.where(amax > 0, 448.0 / amax, torch.ones_like(amax))
    q = (b * inv).clamp(-448, 448).to(torch.float8_e4m3fn)
    sc = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax)).reshape(-1)
    return q.reshape(x.shape), sc


def test_hash_stream_matches_hash_device_and_host():
    C = native()
    s = torch.cuda.current_stream().cuda_stream
    for n in (16, 65536, 65536 + 16, 3 * 65536 + 4096, 40 << 20):
        x = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
        nd = (n + 65535) // 65536
        a = torch.zeros(nd, dtype=torch.int64, device="cuda")
        b = torch.zeros(nd, dtype=torch.int64, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        C.k_hash_stream(x.data_ptr(), n, a.data_ptr(), err.data_ptr(), s, 0)
        C.k_hash_device(x.data_ptr(), n, b.data_ptr(), s, 0)
        torch.cuda.synchronize()
        assert err.item() == 0
        assert torch.equal(a, b), n
        host = C.ssh_digests(x.cpu().numpy())
        assert [v & M for v in a.tolist()] == list(host)


def test_push_raw_is_byte_exact_and_hashes_match_oracle():
    params = _params()
    layout = WeightLayout.from_params(params, "bf16")
    rw = RolloutWeights(layout)
    p = WeightPusher(params, layout, rw.buf.data_ptr())
    p.push()
    torch.cuda.synchronize()
    assert p.result()["error"] == 0
    hashes = p.hashes()
    for n, t in params.items():
        assert torch.equal(rw.get(n), t), n
        assert hashes[n] == _host_hash(t), n
    assert rw.content_hashes() == hashes


def test_delta_push_moves_only_changed_chunks():
    params = _params(1)
    layout = WeightLayout.from_params(params, "bf16")
    rw = RolloutWeights(layout)
    p = WeightPusher(params, layout, rw.buf.data_ptr())
    p.push()
    first = p.result()
    assert first["bytes_stored"] == sum(t.numel() * 2 for t in params.values())
    p.push()  # nothing changed
    assert p.result()["bytes_stored"] == first["bytes_stored"]
    params["big"][7, :] += 1  # one row of one tensor: a single 64 KiB chunk
    p.push()
    third = p.result()
    assert third["chunks_stored"] == first["chunks_stored"] + 1
    torch.cuda.synchronize()
    assert torch.equal(rw.get("big"), params["big"])
    p.invalidate()
    p.push()
    assert p.result()["bytes_stored"] == third["bytes_stored"] + first["bytes_stored"]


def test_push_fp8_matches_fp32_reference():
    params = _params(2)
    layout = WeightLayout.from_params(params, "fp8")
    assert layout.by_name["q"].quant and not layout.by_name["bias"].quant
    rw = RolloutWeights(layout)
    p = WeightPusher(params, layout, rw.buf.data_ptr())
    p.push()
    torch.cuda.synchronize()
    for n, t in params.items():
        e = layout.by_name[n]
        if not e.quant:
            assert torch.equal(rw.get(n), t)
            continue
        q, sc = rw.get(n)
        rq, rsc = _ref_fp8(t)
        assert torch.allclose(sc, rsc, rtol=1e-6, atol=0)
        diff = (q.view(torch.uint8).int() - rq.view(torch.uint8).int()).abs()
        assert diff.max().item() <= 1, n
        assert (diff != 0).float().mean().item() < 5e-3, n
        # dequantized values stay within one e4m3 step of the source
        deq = rw.dequantized(n).float()
        assert torch.allclose(deq, t.float(), rtol=0.07, atol=1e-6)
    # the content hash describes the bf16 source, as in the manifest
    assert p.hashes()["q"] == _host_hash(params["q"])


def test_trainer_weight_sync_seals_versions_with_carry_forward(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=2048, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="wsync") as off:
            params = _params(3)
            layout = WeightLayout.from_params(params, "bf16")
            rw = RolloutWeights(layout)
            rw.publish(off, "rollout/0")
            tr = TrainerWeightSync(off, params, ["rollout/0"], mode="bf16")
            r1 = tr.publish_version(1)
            assert r1["changed"] == len(params)
            params["q"].add_(1)
            r2 = tr.publish_version(2)
            assert r2["changed"] == 1
            torch.cuda.synchronize()
            for n, t in params.items():
                assert torch.equal(rw.get(n), t)
            man = off.get_manifest("policy_rollout", 2)
            assert len(man["tensors"]) == len(params)
            by_name = {e["key"]["param_fqn_debug"]: e for e in man["tensors"]}
            for n, t in params.items():
                assert (by_name[n]["content_hash_lo"], by_name[n]["content_hash_hi"]) == _host_hash(t), n
            tr.close()
    finally:
        d.stop()


def test_subset_push_updates_hash_rows_and_digest_table():
    params = _params(4)
    layout = WeightLayout.from_params(params, "bf16")
    rw = RolloutWeights(layout)
    p = WeightPusher(params, layout, rw.buf.data_ptr())
    p.push()
    full = p.result()["bytes_stored"]
    params["q"].mul_(2)
    params["norm"].add_(1)
    p.push(names=["q", "norm"])
    sub = p.result()["bytes_stored"] - full
    assert sub == params["q"].numel() * 2 + params["norm"].numel() * 2
    torch.cuda.synchronize()
    for n, t in params.items():
        assert torch.equal(rw.get(n), t), n
        assert p.hashes()[n] == _host_hash(t), n
    # the digest table now describes the destination: a full delta push moves nothing
    p.push()
    assert p.result()["bytes_stored"] == full + sub


def test_multicast_needs_two_gpus(sock_path):
    from statespectre_b200.parallel import fabric

    if not fabric.vmm_available(0):
        pytest.skip("no CUDA virtual memory management")
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="wsync-mc1") as off:
            params = _params(5)
            rw = RolloutWeights(WeightLayout.from_params(params, "bf16"))
            rw.publish(off, "rollout/mc1")
            with pytest.raises(RuntimeError, match="two or more GPUs"):
                TrainerWeightSync(off, params, ["rollout/mc1"], persist=False, transport="multicast")
            tr = TrainerWeightSync(off, params, ["rollout/mc1"], persist=False)  # auto: one GPU -> p2p
            assert tr.transport == "p2p"
            tr.close()
            rw.close()
    finally:
        d.stop()


def test_vmm_buffer_tensor_view_and_p2p_push(sock_path):
    from statespectre_b200.parallel import fabric

    if not fabric.vmm_available(0):
        pytest.skip("no CUDA virtual memory management")
    buf = fabric.DeviceBuffer(3 << 20, "cuda:0")
    assert buf.size >= 3 << 20 and buf.tensor.numel() == 3 << 20 and buf.tensor.data_ptr() == buf.ptr
    buf.tensor.fill_(7)
    assert int(buf.tensor.sum().item()) == 7 * (3 << 20)
    buf.close()
    d = in_process_daemon(socket=sock_path, arena_mb=256, drain_on_complete=False)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0, job_name="wsync-vmm") as off:
            params = _params(6)
            layout = WeightLayout.from_params(params, "bf16")
            rw = RolloutWeights(layout)
            rw.publish(off, "rollout/vmm")
            tr = TrainerWeightSync(off, params, ["rollout/vmm"], persist=False, transport="p2p")
            tr.publish_version(1)
            torch.cuda.synchronize()
            for n, t in params.items():
                assert torch.equal(rw.get(n), t), n
            tr.close()
            rw.close()
    finally:
        d.stop()


def test_push_reports_a_bad_item_through_its_bounded_waits():
    """The K4 error path, run on purpose and safely: an item whose source is
    not 16-byte aligned is refused by the producer before any copy is issued
    (status 3), the consumers' bounded waits on the stage it never fills run
    out (about two seconds), and the kernel returns. The launch completes,
    the status is read on the host, and the next push on the same context
    works."""
    import struct as _struct
    import time

    C = native()
    s = torch.cuda.current_stream().cuda_stream
    src = torch.randint(0, 256, (2 * 65536 + 64,), dtype=torch.uint8, device="cuda")
    n = 65536
    item = _struct.pack("<QQQQQIIQQ", src.data_ptr() + 8, 0, 0, n, 0, 2, 0, 0, 0)  # PUSH_HASH, misaligned src
    items = torch.frombuffer(bytearray(item), dtype=torch.uint8).to("cuda")
    dig = torch.zeros(1, dtype=torch.int64, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    C.k_push(items.data_ptr(), 1, 1, dig.data_ptr(), out.data_ptr(), 0, err.data_ptr(), s, 1, 0)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert int(err.item()) == 3  # bad item (first writer wins over the expired waits)
    assert waited < 30
    # the context is still usable: a well-formed launch succeeds
    ok_item = _struct.pack("<QQQQQIIQQ", src.data_ptr(), 0, 0, n, 0, 2, 0, 0, 0)
    items.copy_(torch.frombuffer(bytearray(ok_item), dtype=torch.uint8))
    err.zero_()
    C.k_push(items.data_ptr(), 1, 1, dig.data_ptr(), out.data_ptr(), 0, err.data_ptr(), s, 1, 0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert [int(v) & M for v in dig.tolist()] == list(C.ssh_digests(src[:n].cpu().numpy()))
