"""CPU tests of the drop-in host logic against the reference's golden fixtures."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json, rerun_under_hashseed0
from multi_lora_b200 import batch_info as bi
from multi_lora_b200.eviction import EvictionPolicy
from multi_lora_b200.pool import LoRAMemoryPool, _RankPlan
from multi_lora_b200.weights import AdapterWeights
from oracle import lora_oracle as O


def test_group_rows_matches_reference():
    for case in load_json("group_rows.json"):
        assert bi.group_rows(case["names"], case["seq_lens"]) == (case["group_names"], case["group_lens"])
    with pytest.raises(ValueError):
        bi.group_rows(["a", "b"], [1])


def test_segment_lens():
    assert bi.segment_lens(3, []) == ([1, 1, 1], [0, 1, 2, 3])
    assert bi.segment_lens(3, [13, 13, 22]) == ([13, 13, 22], [0, 13, 26, 48])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_write_metadata_matches_reference_sequence(dtype):
    """Same columns, padding, bs/max_len and in-place/reallocate decisions as batch_info.py:128-179."""
    meta = bi.empty_kernel_input_metadata(device=torch.device("cpu"), dtype=dtype)
    for step in load_json("metadata.json"):
        info = bi.BatchLoRAInfo(step["weight_indices"], step["lora_ranks"], step["scalings"])
        before = meta
        meta = bi.write_kernel_input_metadata(meta, info, device=torch.device("cpu"), dtype=dtype,
                                              seq_lens=step["seq_lens"])
        assert (meta is before) == step["same_object"]
        assert meta.bs == step["bs"] and meta.max_len == step["max_len"]
        assert meta.seg_lens.tolist() == step["seg_lens"]
        assert meta.seg_indptr.tolist() == step["seg_indptr"]
        assert meta.weight_indices.tolist() == step["out_weight_indices"]
        assert meta.lora_ranks.tolist() == step["out_lora_ranks"]
        assert meta.scalings.dtype == dtype
        want = O.bf16_round(np.array(step["scalings"], np.float32)) if dtype == torch.bfloat16 else step["scalings"]
        np.testing.assert_allclose(meta.scalings.float().numpy(), want, rtol=1e-6)
        assert meta.seg_indptr.dtype == torch.int32 and meta.weight_indices.dtype == torch.int32


def test_write_metadata_keeps_addresses_when_it_fits():
    meta = bi.empty_kernel_input_metadata(device=torch.device("cpu"), dtype=torch.float32)
    big = bi.BatchLoRAInfo([0, 1, 2, 1], [8, 8, 8], [1.0, 2.0, 3.0])
    meta = bi.write_kernel_input_metadata(meta, big, device=torch.device("cpu"), dtype=torch.float32, seq_lens=[])
    ptrs = [t.data_ptr() for t in (meta.seg_lens, meta.seg_indptr, meta.weight_indices, meta.lora_ranks,
                                   meta.scalings)]
    small = bi.BatchLoRAInfo([2], [8, 8, 8], [1.0, 2.0, 3.0])
    m2 = bi.write_kernel_input_metadata(meta, small, device=torch.device("cpu"), dtype=torch.float32,
                                        seq_lens=[5])
    assert m2 is meta
    assert ptrs == [t.data_ptr() for t in (m2.seg_lens, m2.seg_indptr, m2.weight_indices, m2.lora_ranks,
                                           m2.scalings)]
    assert m2.seg_indptr.tolist() == [0, 5, 5, 5, 5]


def test_write_metadata_rejects_bad_routing_on_host():
    meta = bi.empty_kernel_input_metadata(device=torch.device("cpu"), dtype=torch.float32)
    with pytest.raises(ValueError):
        bi.write_kernel_input_metadata(meta, bi.BatchLoRAInfo([3], [8, 8], [1.0, 1.0]),
                                       device=torch.device("cpu"), dtype=torch.float32, seq_lens=[])
    with pytest.raises(ValueError):
        bi.write_kernel_input_metadata(meta, bi.BatchLoRAInfo([0], [-1, 8], [1.0, 1.0]),
                                       device=torch.device("cpu"), dtype=torch.float32, seq_lens=[])


def test_eviction_policy_orders():
    lru = EvictionPolicy("lru")
    for n in ["a", "b", "c", "a"]:
        lru.mark_used(n)
    assert lru.select_victim({"a", "b", "c"}) == "b"
    fifo = EvictionPolicy("fifo")
    for n in ["a", "b", "c", "a"]:
        fifo.mark_used(n)
    assert fifo.select_victim({"a", "b", "c"}) == "a"
    assert fifo.select_victim({None}) is None
    with pytest.raises(RuntimeError):
        fifo.select_victim({"zz"})
    with pytest.raises(ValueError):
        EvictionPolicy("mru")


def test_pool_routing_matches_reference_bit_exact():
    """Slot numbers, residency, evictions and batch info equal the reference pool's
    (under PYTHONHASHSEED=0, the seed of the fixtures)."""
    if not rerun_under_hashseed0("tests/test_host_logic.py::test_pool_routing_matches_reference_bit_exact"):
        return
    g = load_json("pool.json")
    modules = {k: tuple(v) for k, v in g["modules"].items()}
    for policy, trace in g["traces"].items():
        pool = LoRAMemoryPool(3, 8, torch.device("cpu"), torch.float32, policy)
        store = {}
        for name, (r, keys, _seed) in g["specs"].items():
            mods = {k: (torch.zeros(r, modules[k][1]), torch.zeros(modules[k][0], r)) for k in keys}
            store[name] = AdapterWeights(rank=r, scaling=1.0 / r, modules=mods)
            pool.ensure_buffers(store[name])
        for step in trace:
            names = list(step["names"])
            pool.prepare_lora_batch(set(names), weight_store=store)
            info = pool.build_batch_info(names)
            assert {("None" if k is None else k): v for k, v in pool.name_to_slot.items()} == step["name_to_slot"]
            assert pool.eviction_policy.eviction_count == step["eviction_count"]
            assert info.weight_indices == step["weight_indices"]
            assert info.lora_ranks == step["lora_ranks"]
            np.testing.assert_allclose(info.scalings, step["scalings"])


def test_pool_errors_leave_state_consistent():
    pool = LoRAMemoryPool(2, 8, torch.device("cpu"), torch.float32)
    store = {n: AdapterWeights(rank=4, scaling=0.5, modules={"m": (torch.zeros(4, 3), torch.zeros(5, 4))})
             for n in "abc"}
    store["big"] = AdapterWeights(rank=16, scaling=1.0, modules={"m": (torch.zeros(16, 3), torch.zeros(5, 16))})
    pool.prepare_lora_batch({"a", "b"}, weight_store=store)
    snap = dict(pool.name_to_slot)
    with pytest.raises(ValueError):  # three distinct adapters, two slots
        pool.prepare_lora_batch({"a", "b", "c"}, weight_store=store)
    assert set(pool.name_to_slot) <= set(snap) | {"c"}
    pool2 = LoRAMemoryPool(2, 8, torch.device("cpu"), torch.float32)
    with pytest.raises(ValueError):  # rank above max_lora_rank
        pool2.prepare_lora_batch({"big"}, weight_store=store)
    with pytest.raises(KeyError):
        pool2.prepare_lora_batch({"missing"}, weight_store=store)
    with pytest.raises(KeyError):
        pool.get_slot_id("zzz")


def test_rank_plan_layout_tiles_bank():
    """A blocks then B blocks, no gaps or overlaps; rects describe slot-stack strides."""
    dims = {"q": (16, 24), "k": (16, 8), "down": (40, 16)}
    plan = _RankPlan(4, list(dims), dims)
    ref = O.rank_plan(4, list(dims), dims)
    assert plan.total == ref["total"]
    assert plan.a_off == ref["a_off"] and plan.b_off == ref["b_off"]
    spans = sorted([(plan.a_off[k], plan.a_off[k] + 4 * dims[k][0]) for k in dims] +
                   [(plan.b_off[k], plan.b_off[k] + dims[k][1] * 4) for k in dims])
    pos = 0
    for lo, hi in spans:
        assert lo == pos
        pos = hi
    assert pos == plan.total


def test_bank_repacks_from_old_bank_when_modules_grow():
    """An adapter whose module tensors were released follows a growing module set:
    its bank is repacked from the previous bank, with zeros for modules it lacks."""
    from multi_lora_b200.pool import _GpuBuffers

    bufs = _GpuBuffers(4, 4, torch.device("cpu"), torch.float32)
    g = torch.Generator().manual_seed(3)
    a1, b1 = torch.randn(4, 16, generator=g), torch.randn(24, 4, generator=g)
    w = AdapterWeights(rank=4, scaling=1.0, modules={"q": (a1.clone(), b1.clone())})
    bufs.ensure(w)
    plan1 = bufs._plan_for(4)
    bank1 = bufs._bank_for(w, plan1)
    assert w.flattened and w.modules == {}
    assert bufs._bank_for(w, plan1) is bank1  # cached for the same layout
    # another adapter brings a new module: the layout grows, w is repacked from its bank
    a2, b2 = torch.randn(4, 8, generator=g), torch.randn(40, 4, generator=g)
    bufs.ensure(AdapterWeights(rank=4, scaling=1.0, modules={"down": (a2, b2)}))
    plan2 = bufs._plan_for(4)
    assert plan2 is not plan1 and plan2.total > plan1.total
    bank2 = bufs._bank_for(w, plan2)
    assert torch.equal(bank2[plan2.a_off["q"]: plan2.a_off["q"] + 64], a1.reshape(-1))
    assert torch.equal(bank2[plan2.b_off["q"]: plan2.b_off["q"] + 96], b1.reshape(-1))
    assert not bank2[plan2.a_off["down"]: plan2.a_off["down"] + 32].any()
    assert not bank2[plan2.b_off["down"]: plan2.b_off["down"] + 160].any()
    # an adapter with neither tensors nor a bank cannot be packed
    bare = AdapterWeights(rank=4, scaling=1.0, modules={}, flattened=True)
    with pytest.raises(RuntimeError):
        bufs._bank_for(bare, plan2)
