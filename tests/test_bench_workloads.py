"""Host-side logic of bench.py: the named workloads' routing, byte/FLOP
accounting, tensor-parallel shard shapes and the cfg4 admission rule."""

from __future__ import annotations

import bench


def test_cfg2_routing_and_bytes():
    wl = bench.WORKLOADS["cfg2"]
    ids, info, lens = bench.routing(wl)
    assert len(ids) == 64 and sum(lens) == 64
    assert len(set(ids)) == 29  # seed 0 draws 29 distinct adapters of 32
    ab = bench.algorithmic_bytes(wl, ids, 1)
    # per layer: 29 adapters x r16 over q,k,v,o (4096 -> 4096), gate/up (4096 -> 11008), down (11008 -> 4096)
    assert abs(ab["lora"] / wl.layers / 1e6 - 87.9) < 0.2
    assert ab["lora_flops"] == wl.layers * sum(2 * 64 * 16 * (i + o) for _, i, o, _ in wl.projs)


def test_cfg3_prefill_routing_matches_the_stated_lengths():
    wl = bench.WORKLOADS["cfg3"]
    ids, info, lens = bench.routing(wl)
    assert lens == [469, 845, 454, 989, 348, 314, 495, 426]  # randint(128, 1025, (8,)) with seed 0
    assert list(info.weight_indices) == list(range(8)) and info.lora_ranks == [64] * 8
    ab = bench.algorithmic_bytes(wl, ids, 1)
    assert abs(ab["lora"] / wl.layers / 1e9 - 1.176) < 0.002
    assert abs(ab["lora_flops"] / wl.layers / 1e9 - 45.5) < 0.1


def test_tp_shards_and_bytes_shrink_with_tp():
    wl = bench.WORKLOADS["cfg5"]
    ids, _, _ = bench.routing(wl)
    assert len(set(ids)) == 128
    per = [bench.algorithmic_bytes(wl, ids, tp)["lora"] / wl.layers for tp in (1, 2, 4, 8)]
    assert abs(per[0] / 1e6 - 914.6) < 1.0
    assert per == sorted(per, reverse=True)
    d8 = bench.shard_dims(wl, 8)
    assert d8["q"] == (8192, 1024, 1024)        # column-parallel: full A, B and y sharded on out
    assert d8["down"] == (28672 // 8, 1024, 8192)  # row-parallel: x/A sharded on in, full-width partial y


def test_launch_counts_per_path():
    wl = bench.WORKLOADS["cfg2"]
    assert bench.launches_per_layer(wl, True, 1, 1) == {"lora": 4, "rmsnorm": 2}    # fused, grouped
    assert bench.launches_per_layer(wl, True, 3, 1) == {"lora": 8, "rmsnorm": 2}    # streaming pair per call
    assert bench.launches_per_layer(wl, False, 2, 1) == {"lora": 14, "rmsnorm": 2}  # split: 2 per projection
    assert bench.launches_per_layer(wl, True, 1, 2)["lora"] == 2 + 2 * 2             # row-parallel o/down: 2 each


def test_admission_rule():
    queue = ["a", "b", "a", "c", "d", "b", "e", "c"]
    admitted, deferred, distinct = bench.admit(queue, 3)
    assert admitted == ["a", "b", "a", "c", "b", "c"]  # d and e would be a 4th and 5th adapter
    assert deferred == ["d", "e"]
    assert distinct == {"a", "b", "c"}
    admitted, deferred, _ = bench.admit(deferred + ["f"], 3)
    assert admitted == ["d", "e", "f"] and deferred == []
