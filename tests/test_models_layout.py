"""Model shapes, weight layouts and generated daemon configs (no GPU)."""

import pytest
import torch

from statespectre_b200._native import native
from statespectre_b200.models.shapes import (LLAMA3_8B, QWEN2_5_32B, KVCacheSpec, num_params, param_shapes,
                                             pick_changed, random_init)
from statespectre_b200.parallel.weight_sync import ALIGN, WeightLayout
from statespectre_b200.utils.topology import daemon_yaml


@pytest.mark.parametrize("spec,expect_b", [(QWEN2_5_32B, 32.8), (LLAMA3_8B, 8.0)])
def test_model_sizes_and_tp_shards_cover_the_model(spec, expect_b):
    full = num_params(param_shapes(spec))
    assert abs(full / 1e9 - expect_b) < 0.35, full
    for tp in (2, 4, 8):
        shards = [param_shapes(spec, r, tp) for r in range(tp)]
        assert [n for n, _ in shards[0]] == [n for n, _ in param_shapes(spec)]
        # sharded tensors split exactly; replicated ones (norms) repeat on every shard
        repl = sum(num_params([(n, s)]) for n, s in param_shapes(spec) if "norm" in n)
        assert sum(num_params(s) for s in shards) == full + (tp - 1) * repl
    with pytest.raises(ValueError):
        param_shapes(spec, 0, 3)  # 8 KV heads do not split 3 ways


def test_random_init_and_change_selection_are_seeded():
    shapes = param_shapes(LLAMA3_8B, layers=1)
    small = [(n, s) for n, s in shapes if num_params([(n, s)]) < (1 << 20)][:3]
    a = random_init(small, "cpu", seed=4)
    b = random_init(small, "cpu", seed=4)
    assert all(torch.equal(a[n], b[n]) and a[n].dtype == torch.bfloat16 for n in a)
    names = [n for n, _ in shapes]
    c1, c2 = pick_changed(names, 0.1, seed=9), pick_changed(names, 0.1, seed=9)
    assert c1 == c2 and len(c1) == max(1, round(0.1 * len(names)))


def test_kv_block_geometry():
    spec = KVCacheSpec()
    assert spec.block_bytes == 4 << 20  # 16 tokens x 64 layers x 8 heads x 128 dims x (K, V) x bf16
    assert spec.blocks_for(40 << 30) == 10240


def test_weight_layout_offsets_quantization_and_fingerprint():
    specs = [("embed", (1000, 256), torch.bfloat16), ("norm", (256,), torch.bfloat16),
             ("w", (512, 384), torch.bfloat16), ("f32", (64, 4), torch.float32)]
    bf = WeightLayout(specs, "bf16")
    q = WeightLayout(specs, "fp8")
    assert bf.fingerprint == WeightLayout(specs, "bf16").fingerprint != q.fingerprint
    for lay in (bf, q):
        end = 0
        for e in lay.entries:
            assert e.dst_offset % ALIGN == 0 and e.dst_offset >= end
            end = e.dst_offset + e.dst_nbytes
            if e.quant:
                assert e.scale_offset % ALIGN == 0 and e.nscales * 128 * 2 == e.nbytes
                end = e.scale_offset + 4 * e.nscales
        assert lay.total_bytes >= end
    # fp8 only for 2-D bf16 weights whose size is a multiple of 128 values
    assert [e.quant for e in q.entries] == [True, False, True, False]
    assert q.by_name["w"].dst_nbytes == 512 * 384
    assert q.total_chunks == bf.total_chunks
    with pytest.raises(ValueError):
        WeightLayout([("odd", (3,), torch.bfloat16)])  # 6 bytes: not a multiple of 16


def test_generated_daemon_config_parses():
    text = daemon_yaml("/tmp/x.sock", [0, 0, 1, 1], [8, 8, 0, 4], slot_mb=2, drain_on_complete=True,
                       drain_target="nvme", nvme_dir="/nvme/ofld")
    c = native().parse_config(text)
    assert c["socket_path"] == "/tmp/x.sock" and c["allocation_granularity_bytes"] == 2 << 20
    nodes = {a["numa_node"]: a for a in c["per_numa"]}
    assert nodes[0]["gpu_windows"] == [(0, 8 << 30), (1, 8 << 30)]
    assert nodes[1]["gpu_windows"] == [(3, 4 << 30)]  # GPU 2 has no window
    assert c["drain_target"] == "nvme" and c["nvme_io_engine"] == "io_uring" and c["nvme_direct_io"]
