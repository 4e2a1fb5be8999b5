"""Slot-pool loads on the GPU (pinned bank -> stage -> scatter kernel), bit-exact.

* against the reference pool's slot contents (golden, PYTHONHASHSEED=0);
* the reference GPU test's rounds (test_pool_write_many_gpu.py:65-94), including
  more same-rank adapters than one scatter chunk, missing modules and slot reuse.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json, load_npz, rerun_under_hashseed0
from multi_lora_b200.pool import _BANK_CHUNK, LoRAMemoryPool
from multi_lora_b200.weights import AdapterWeights

pytestmark = pytest.mark.gpu


def _weights(modules, rank, keys, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    mods = {}
    for k in keys:
        n_out, n_in = modules[k]
        mods[k] = (torch.randn(rank, n_in, generator=g).to(dtype), torch.randn(n_out, rank, generator=g).to(dtype))
    return AdapterWeights(rank=rank, scaling=1.0 / rank, modules=mods)


def test_pool_slots_match_reference_golden(cuda_dev):
    if not rerun_under_hashseed0("tests/test_pool_gpu.py::test_pool_slots_match_reference_golden"):
        return
    g = load_json("pool.json")
    slots = load_npz("pool_slots.npz")
    modules = {k: tuple(v) for k, v in g["modules"].items()}
    for policy, trace in g["traces"].items():
        pool = LoRAMemoryPool(3, 8, cuda_dev, torch.float32, policy)
        store = {n: _weights(modules, r, k, s) for n, (r, k, s) in g["specs"].items()}
        for w in store.values():
            pool.ensure_buffers(w)
        for i, step in enumerate(trace):
            pool.prepare_lora_batch(set(step["names"]), weight_store=store)
            torch.cuda.synchronize()
            for k in modules:
                a, b = pool.get_module_buffers(k)
                np.testing.assert_array_equal(a.cpu().numpy(), slots[f"{policy}_{i}_{k}_A"], err_msg=f"{policy} {i}")
                np.testing.assert_array_equal(b.cpu().numpy(), slots[f"{policy}_{i}_{k}_B"], err_msg=f"{policy} {i}")
        pool.buffers.check_status()


MODULES = {"m1": (4, 3), "m2": (5, 3), "big": (1000, 520)}


def _check_resident(pool, ref):
    for name, slot in pool.name_to_slot.items():
        if name is None:
            continue
        w = ref[name]
        r = w.rank
        for key in MODULES:
            a, b = pool.get_slot_weights(slot, key)
            if key in w.modules:
                wa, wb = w.modules[key]
                assert torch.equal(a[:r].cpu(), wa), (name, key)
                assert torch.equal(b[:, :r].cpu(), wb), (name, key)
            else:
                assert a[:r].abs().sum() == 0 and b[:, :r].abs().sum() == 0, (name, key)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pool_rounds_like_reference_gpu_test(cuda_dev, dtype):
    specs = {"a": (8, ["m1", "m2", "big"], 1), "b": (8, ["m1"], 2), "c": (4, ["m1", "m2", "big"], 3),
             "d": (4, ["m2"], 4), "e": (8, ["m1", "m2", "big"], 5), "f": (8, ["m1", "m2"], 6),
             "g": (8, ["m2", "big"], 7)}
    store = {n: _weights(MODULES, r, k, s, dtype) for n, (r, k, s) in specs.items()}
    ref = {n: _weights(MODULES, r, k, s, dtype) for n, (r, k, s) in specs.items()}
    pool = LoRAMemoryPool(8, 8, cuda_dev, dtype)
    for w in store.values():
        pool.ensure_buffers(w)
    rounds = [{"a", "b", "c", "d"}, {"e"}, {"a", "c", "e"}, {"b", "d"}, {"a", "b", "e", "f", "g"}]
    assert len(rounds[-1]) > _BANK_CHUNK
    for names in rounds:
        pool.prepare_lora_batch(names, weight_store=store)
        torch.cuda.synchronize()
        _check_resident(pool, ref)
    assert all(store[n].flattened and hasattr(store[n], "_mlora_bank") for n in store)
    pool.buffers.check_status()


def test_load_overlaps_on_copy_stream_and_compute_waits(cuda_dev):
    """The H2D + scatter run on the pool's copy stream; the compute stream waits on its event."""
    pool = LoRAMemoryPool(2, 8, cuda_dev, torch.bfloat16)
    store = {"a": _weights(MODULES, 8, ["big"], 1, torch.bfloat16)}
    ref = _weights(MODULES, 8, ["big"], 1, torch.bfloat16)
    pool.ensure_buffers(store["a"])
    pool.prepare_lora_batch({"a"}, weight_store=store)
    # no explicit synchronize: a compute-stream read must observe the loaded slot
    a, _ = pool.get_slot_weights(pool.get_slot_id("a"), "big")
    first = a[:8].clone()
    torch.cuda.synchronize()
    assert torch.equal(first.cpu(), ref.modules["big"][0])
    assert pool.buffers._copy_stream is not None


def test_load_into_evicted_slot_waits_for_queued_reads(cuda_dev):
    """A load into a slot the previous batch used starts only after the compute
    queued before the new batch was prepared (per-slot event), so that compute
    still sees the old adapter."""
    pool = LoRAMemoryPool(2, 8, cuda_dev, torch.bfloat16)
    seeds = {"a": 1, "b": 2, "c": 3}
    store = {n: _weights(MODULES, 8, ["big"], s, torch.bfloat16) for n, s in seeds.items()}
    refs = {n: _weights(MODULES, 8, ["big"], s, torch.bfloat16) for n, s in seeds.items()}
    pool.ensure_buffers(store["a"])
    pool.prepare_lora_batch({"a", "b"}, weight_store=store)
    slot_a = pool.get_slot_id("a")
    torch.cuda._sleep(100_000_000)  # bounded busy wait: the read below is still queued at the next prepare
    a, _ = pool.get_slot_weights(slot_a, "big")
    seen = a[:8].clone()
    pool.prepare_lora_batch({"b", "c"}, weight_store=store)  # evicts a; c goes into its slot
    assert pool.get_slot_id("c") == slot_a
    torch.cuda.synchronize()
    assert torch.equal(seen.cpu(), refs["a"].modules["big"][0])
    a2, _ = pool.get_slot_weights(slot_a, "big")
    assert torch.equal(a2[:8].cpu(), refs["c"].modules["big"][0])
    pool.buffers.check_status()


def test_load_into_unused_slot_overlaps_queued_compute(cuda_dev):
    """Slots no queued work reads are loaded without waiting for the compute stream."""
    pool = LoRAMemoryPool(2, 8, cuda_dev, torch.bfloat16)
    store = {"a": _weights(MODULES, 8, ["big"], 1, torch.bfloat16)}
    pool.ensure_buffers(store["a"])
    torch.cuda.synchronize()
    torch.cuda._sleep(400_000_000)  # bounded busy wait (~0.2 s) on the compute stream
    pool.prepare_lora_batch({"a"}, weight_store=store)
    pool.buffers._load_event.synchronize()  # the load finished ...
    overlapped = not torch.cuda.current_stream().query()  # ... while the queued compute still runs
    torch.cuda.synchronize()
    assert overlapped


def test_scatter_stage_op_matches_oracle(cuda_dev):
    """torch.ops.mlora.scatter_stage (the slot-load op, scatter_bank.py:68-93) writes
    every staged block into its slot bit-exactly; entries past the rank stay as they were."""
    from multi_lora_b200 import _native
    from multi_lora_b200.pool import _RankPlan
    from oracle import lora_oracle as O

    dims = {"q": (24, 16), "down": (40, 24), "v": (16, 8)}  # key -> (in, out)
    keys, rank, R, K = list(dims), 4, 8, 6
    g = torch.Generator().manual_seed(11)
    A = {k: torch.randn(K, R, dims[k][0], generator=g) for k in keys}
    B = {k: torch.randn(K, dims[k][1], R, generator=g) for k in keys}
    A_dev = {k: v.to(cuda_dev) for k, v in A.items()}
    B_dev = {k: v.to(cuda_dev) for k, v in B.items()}

    class _Bufs:
        pass

    bufs = _Bufs()
    bufs.A, bufs.B = A_dev, B_dev
    plan = _RankPlan(rank, keys, dims)
    rects = torch.tensor(plan.rects(bufs), dtype=torch.int64, device=cuda_dev)
    max_elems = max(r[3] * r[4] for r in plan.rects(bufs))
    slots = [4, 1, 3]
    banks = []
    for i, _ in enumerate(slots):
        mods = {k: (torch.randn(rank, dims[k][0], generator=g), torch.randn(dims[k][1], rank, generator=g))
                for k in keys if not (i == 1 and k == "v")}  # adapter 1 lacks "v": zero blocks
        banks.append(O.build_bank(rank, keys, dims, {k: (a.numpy(), b.numpy()) for k, (a, b) in mods.items()}))
    stage = torch.tensor(np.stack(banks), device=cuda_dev)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    _native.ops().scatter_stage(stage, torch.tensor(slots, dtype=torch.int64, device=cuda_dev), rects, max_elems,
                                status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    A_ref = {k: v.numpy().copy() for k, v in A.items()}
    B_ref = {k: v.numpy().copy() for k, v in B.items()}
    for bank, s in zip(banks, slots):
        O.scatter_bank(bank, rank, keys, dims, A_ref, B_ref, s)
    for k in keys:
        np.testing.assert_array_equal(A_dev[k].cpu().numpy(), A_ref[k], err_msg=k)
        np.testing.assert_array_equal(B_dev[k].cpu().numpy(), B_ref[k], err_msg=k)
    with pytest.raises(RuntimeError):  # slots must be int64
        _native.ops().scatter_stage(stage, torch.tensor(slots, dtype=torch.int32, device=cuda_dev), rects,
                                    max_elems, status)
