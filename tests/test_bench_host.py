"""Host-side logic of bench.py (no GPU): workload builders, the parity samples, the
unique-byte accounting and the allocator replay the page-table parity uses."""

import numpy as np
import torch

import bench


def test_config3_sample_covers_shared_prefix_groups():
    cfg = bench.decode_config("c3")
    rows = bench.sample_rows(cfg, cfg["B"], 0, seed=7)
    assert len(rows) == 32 and len({int(r) // 16 for r in rows}) == 2
    ctx = bench.sample_context_lens(cfg, 0)
    bt, _ = bench.block_tables(cfg, ctx, 0)
    for g0 in {int(r) // 16 * 16 for r in rows}:
        assert (bt[g0:g0 + 16, :64] == bt[g0, :64]).all()  # 64 shared pages per group


def test_unique_bytes_count_shared_prefix_once():
    cfg = bench.decode_config("c3")
    ctx = bench.sample_context_lens(cfg, 0)
    b = bench.decode_bytes(cfg, ctx, 8, 32)
    per_token = 8 * 128 * 2 * 2
    assert b["kv"] == int(ctx.sum()) * per_token
    assert b["kv"] - b["kv_unique"] == 16 * 15 * 1024 * per_token  # 16 groups, 15 repeats of 1024 tokens
    assert b["total"] - b["total_unique"] == b["kv"] - b["kv_unique"]


def test_allocator_replay_is_sequential():
    ids, lens = bench._replay_allocator(3, 20, 13, 16)
    assert lens == [33, 33, 33]
    assert ids == [[0, 1, 6], [2, 3, 7], [4, 5, 8]]


def test_cpu_sample_keeps_the_workload_tables():
    cfg = bench.decode_config("c1")
    r = bench.cpu_decode_sample(cfg, 2, 0.01)
    assert r["unit"] == "GB/s" and r["value"] > 0 and r["sequences"] >= 1
