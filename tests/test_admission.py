"""Admission of queued tokens into a step (multi_lora_b200.admission): the batch
names at most ``slots`` adapters, deferred tokens go first, resident adapters
before the rest, row order kept. CPU only."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from multi_lora_b200.admission import AdmissionPolicy, TokenQueue
from multi_lora_b200.layers import LinearWithLoRA
from multi_lora_b200.manager import MultiLoRAManager
from multi_lora_b200.weights import AdapterWeights


def test_queue_order_rule():
    pol = AdmissionPolicy(3, resident_first=False)
    q = ["a", "b", "a", "c", "d", "b", "e", "c"]
    adm = pol.admit(q)
    assert [q[i] for i in adm.admitted] == ["a", "b", "a", "c", "b", "c"]
    assert [q[i] for i in adm.deferred] == ["d", "e"]
    assert adm.adapters == {"a", "b", "c"}


def test_resident_first_prefers_loaded_adapters():
    pol = AdmissionPolicy(2)
    q = ["x", "r1", "y", "r2", "r1"]
    adm = pol.admit(q, resident={"r1", "r2"})
    assert adm.adapters == {"r1", "r2"}
    assert adm.admitted == [1, 3, 4]  # queue (row) order kept
    assert [q[i] for i in adm.deferred] == ["x", "y"]


def test_deferred_tokens_go_first_and_cannot_starve():
    pol = AdmissionPolicy(2)
    # "old" was deferred before; it outranks resident adapters
    q = ["old", "r1", "r2"]
    adm = pol.admit(q, resident={"r1", "r2"}, n_deferred=1)
    assert 0 in adm.admitted and adm.adapters == {"old", "r1"}
    # a queue that keeps deferring: every token is admitted within a bounded number of steps
    rng = np.random.default_rng(0)
    tq = TokenQueue(AdmissionPolicy(4), max_tokens=16)
    age = {}
    step = 0
    resident: set = set()
    for step in range(200):
        new = [f"a{int(i)}" for i in rng.zipf(1.3, size=16 - len(tq.pending)) % 40]
        ids = [(step, k) for k in range(len(new))]
        for t in ids:
            age[t] = step
        admitted = tq.step(new, resident=resident)
        resident = set(admitted)
        assert len(set(admitted)) <= 4 and len(admitted) <= 16
    # nothing waits for long: the queue never grows past one step's worth
    assert len(tq.pending) < 16


def test_max_tokens_and_arguments():
    pol = AdmissionPolicy(8)
    adm = pol.admit(["a"] * 10, max_tokens=4)
    assert adm.admitted == [0, 1, 2, 3] and adm.deferred == [4, 5, 6, 7, 8, 9]
    with pytest.raises(ValueError):
        AdmissionPolicy(0)
    with pytest.raises(ValueError):
        pol.admit(["a"], n_deferred=2)


def test_base_model_takes_a_slot():
    adm = AdmissionPolicy(1).admit([None, "a", None])
    assert adm.adapters == {None} and adm.admitted == [0, 2]


def test_manager_admission_uses_pool_residency():
    lin = torch.nn.Linear(8, 8, bias=False)
    mgr = MultiLoRAManager({"m": LinearWithLoRA(lin)}, device=torch.device("cpu"), dtype=torch.float32,
                           max_loras_per_batch=2, max_lora_rank=4)
    for n in ("a", "b", "c"):
        mgr.register_adapter(n, AdapterWeights(rank=4, scaling=1.0,
                                               modules={"m": (torch.zeros(4, 8), torch.zeros(8, 4))}))
    mgr.prepare_lora_batch(["a", "b"])  # a, b resident (routing-only pool on the CPU)
    adm = mgr.admit_tokens(["c", "a", "b", "c"])
    assert adm.adapters == {"a", "b"} and adm.admitted == [1, 2]
    adm = mgr.admit_tokens(["c", "a", "b"], resident_first=False)
    assert adm.adapters == {"c", "a"}
    mgr.prefetch_lora_batch(["c"])
    assert "c" in mgr.pool.name_to_slot
    with pytest.raises(ValueError):
        mgr.prefetch_lora_batch(["a", "b", "c"])
