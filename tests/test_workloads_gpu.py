"""Transformer-style offload on one GPU: per-layer weights and a growing KV
cache move between VRAM and the host tiers, restored on demand, with the
VRAM release checked through torch's allocator (the workload of
StateSpectre's LLM test, reference: tests/python/test_llm_workload.py)."""

import time

import pytest
import torch

from statespectre_b200 import in_process_daemon, offload_context

pytestmark = pytest.mark.gpu

LAYERS = 8
LAYER_BYTES = 32 << 20   # bf16 weights per layer
KV_BLOCK_BYTES = 4 << 20  # one KV-cache block
KV_STEPS = 16
KV_RESIDENT = 4


def _wait_cold(hs, timeout=60.0) -> bool:
    deadline = time.time() + timeout
    while time.time() < deadline:
        if all(h.location() in ("pageable", "nvme") for h in hs):
            return True
        time.sleep(0.01)
    return False


def test_layer_and_kv_offload_releases_vram(sock_path):
    d = in_process_daemon(socket=sock_path, arena_mb=1024, drain_on_complete=True)
    try:
        with offload_context(daemon_addr=sock_path, device="cuda:0", rank=0) as off:
            g = torch.Generator(device="cuda").manual_seed(5)
            layers = [torch.randn(LAYER_BYTES // 2, generator=g, device="cuda").to(torch.bfloat16)
                      for _ in range(LAYERS)]
            refs = [off.hash_tensor(t) for t in layers]
            torch.cuda.synchronize()
            before = torch.cuda.memory_allocated()
            # keep layer 0 (the active one) resident; offload the others destructively
            handles = {i: off.evict(layers[i], wait=True) for i in range(1, LAYERS)}
            torch.cuda.synchronize()
            freed = before - torch.cuda.memory_allocated()
            assert freed >= (LAYERS - 1) * LAYER_BYTES, freed
            assert all(layers[i].numel() == 0 for i in range(1, LAYERS))
            assert _wait_cold(handles.values()), [h.location() for h in handles.values()]
            # decode steps: a new KV block per step, the oldest ones offloaded
            kv, kv_refs, kv_handles = [], [], []
            for step in range(KV_STEPS):
                blk = torch.randn(KV_BLOCK_BYTES // 2, generator=g, device="cuda").to(torch.bfloat16)
                kv_refs.append(off.hash_tensor(blk))
                kv.append(blk)
                if len(kv) > KV_RESIDENT:
                    old = kv.pop(0)
                    kv_handles.append(off.evict(old, wait=True))
            assert len(kv_handles) == KV_STEPS - KV_RESIDENT
            # forward pass: every offloaded layer comes back byte-identical
            for i, h in handles.items():
                t = h.restore()
                assert off.hash_tensor(t) == refs[i], i
                del t
                h.discard()
            restored = off.restore_batch(kv_handles, [torch.empty(KV_BLOCK_BYTES // 2, dtype=torch.bfloat16,
                                                                  device="cuda") for _ in kv_handles])
            torch.cuda.synchronize()
            for j, t in enumerate(restored):
                assert off.hash_tensor(t) == kv_refs[j], j
            off.discard_batch(kv_handles)
            st = off.daemon_stats()
            assert st["used_slots"] == 0 and st["pageable_resident_bytes"] == 0
    finally:
        d.stop()
