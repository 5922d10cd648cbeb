"""Benchmark workloads behind ``bench.py --workload``: the evict/restore size
sweep, paged KV-cache offload under load and data-parallel dedup with ZeRO-1
optimizer-state spill. The headline evict/restore point and the in-box
weight sync live in ``bench.py`` and ``parallel/weight_sync_bench.py``."""
