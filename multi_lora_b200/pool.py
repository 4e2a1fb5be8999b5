"""GPU slot pool with eviction (drop-in for ``multi_lora/pool.py``).

K slots per module: ``A[key]`` is ``[K, max_rank, in]`` and ``B[key]`` is
``[K, out, max_rank]`` (pool.py:97-155 of the reference); slot numbers are what
the kernels index with ``weight_indices``. Residency and victim choice follow
``LoRAMemoryPool.prepare_lora_batch`` / ``_alloc_slot`` (pool.py:382-473).

Loads (pool.py:157-316): each adapter's weights are packed once into a
pinned host "bank" (all A blocks, then all B blocks, one layout per rank);
a swap-in is one contiguous ``cudaMemcpyAsync`` of the bank into a device
stage row on a private copy stream, then one scatter launch per chunk of
adapters writes every block into its slot (``torch.ops.mlora.scatter_stage``
over the C ABI's ``mlora_scatter_stage``). The
compute stream waits on the copy stream's event, so the H2D overlaps
whatever compute was queued before the load.

A pool on a non-CUDA device tracks slots only (routing tests); it holds no
weights and loads nothing.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Set, Tuple

import torch

from multi_lora_b200 import _native
from multi_lora_b200.batch_info import BatchLoRAInfo
from multi_lora_b200.eviction import EvictionPolicy
from multi_lora_b200.weights import AdapterWeights

LoraName = Optional[str]

# adapters staged per scatter launch (pool.py:18-20 uses the same chunking)
_BANK_CHUNK = 4
# attribute under which an AdapterWeights carries (layout, pinned bank)
_BANK_ATTR = "_mlora_bank"


class _RankPlan:
    """Bank layout shared by every adapter of one rank.

    A blocks of all keys in key order, then B blocks in key order; an A
    block is [rank, in] row-major, a B block [out, rank] row-major.
    """

    def __init__(self, rank: int, keys: List[str], dims: Dict[str, Tuple[int, int]]):
        self.rank = rank
        self.keys = list(keys)
        self.a_off: Dict[str, int] = {}
        self.b_off: Dict[str, int] = {}
        self.a_shape: Dict[str, Tuple[int, int]] = {}
        self.b_shape: Dict[str, Tuple[int, int]] = {}
        pos = 0
        for k in self.keys:
            self.a_off[k] = pos
            self.a_shape[k] = (rank, dims[k][0])
            pos += rank * dims[k][0]
        for k in self.keys:
            self.b_off[k] = pos
            self.b_shape[k] = (dims[k][1], rank)
            pos += dims[k][1] * rank
        self.total = pos
        self.tables: Optional[dict] = None

    def rects(self, buffers: "_GpuBuffers") -> List[Tuple[int, int, int, int, int, int]]:
        """Scatter rectangles (src_offset, dst address, slot_stride, rows, cols, dst_row_stride)."""
        out = []
        for k in self.keys:
            a = buffers.A[k]
            r, n_in = self.a_shape[k]
            out.append((self.a_off[k], a.data_ptr(), a.stride(0), r, n_in, a.stride(1)))
        for k in self.keys:
            b = buffers.B[k]
            n_out, r = self.b_shape[k]
            out.append((self.b_off[k], b.data_ptr(), b.stride(0), n_out, r, b.stride(1)))
        return out

    def build_tables(self, buffers: "_GpuBuffers", device: torch.device) -> dict:
        """Device rectangle table for the scatter launch (built once per plan)."""
        rects = self.rects(buffers)
        self.tables = {
            "rects": torch.tensor(rects, dtype=torch.int64).to(device),
            "n": len(rects),
            "max_numel": max(r[3] * r[4] for r in rects),
        }
        return self.tables


class _GpuBuffers:
    """All slots of all modules on the device, plus the load machinery."""

    def __init__(self, max_loras_per_batch: int, max_lora_rank: int, device: torch.device, dtype: torch.dtype):
        self.max_loras_per_batch = max_loras_per_batch
        self.max_lora_rank = max_lora_rank
        self.device = torch.device(device)
        self.dtype = dtype
        self.routing_only = self.device.type != "cuda"
        self.A: Dict[str, torch.Tensor] = {}
        self.B: Dict[str, torch.Tensor] = {}
        self.dims: Dict[str, Tuple[int, int]] = {}  # key -> (in, out)
        self._copy_stream: Optional[torch.cuda.Stream] = None
        self._load_event: Optional[torch.cuda.Event] = None
        self._plans: Dict[tuple, _RankPlan] = {}  # (rank, module keys) -> bank layout
        self.release_modules = True  # drop the per-module host tensors once banked
        self._stage: Optional[torch.Tensor] = None
        self._status: Optional[torch.Tensor] = None
        # per slot: an event on the compute stream after the last work that may read it
        self._slot_event: Dict[int, torch.cuda.Event] = {}
        self._live_slots: Set[int] = set()
        self._loaded: Set[int] = set()  # slots written at least once

    def ensure(self, weights: AdapterWeights) -> None:
        """Create zeroed slot stacks for modules seen for the first time."""
        for key, (a_host, b_host) in weights.modules.items():
            if key in self.dims:
                continue
            n_in, n_out = int(a_host.shape[1]), int(b_host.shape[0])
            self.dims[key] = (n_in, n_out)
            if self.routing_only:
                continue
            k, r = self.max_loras_per_batch, self.max_lora_rank
            self.A[key] = torch.zeros((k, r, n_in), device=self.device, dtype=self.dtype)
            self.B[key] = torch.zeros((k, n_out, r), device=self.device, dtype=self.dtype)

    def begin_batch(self, slots: Set[int]) -> None:
        """A new batch is being prepared: everything enqueued on the compute
        stream so far may read the previous batch's slots, so stamp them with
        an event there; ``slots`` are the new batch's."""
        if self.routing_only:
            return
        if self._live_slots:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            for s in self._live_slots:
                self._slot_event[s] = ev
        self._live_slots = set(slots)

    def write_many(self, pairs: List[Tuple[int, AdapterWeights]]) -> None:
        """Load ``[(slot, weights), ...]`` into their slots (async on the copy stream).

        The copy stream waits only for the compute that last read the target
        slots (their events), not for all queued compute, so a load into a slot
        the previous batch did not use overlaps that batch's kernels.
        """
        if not pairs or self.routing_only:
            return
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
            self._load_event = torch.cuda.Event()
        for slot, _ in pairs:
            ev = self._slot_event.get(slot)
            if ev is not None:
                self._copy_stream.wait_event(ev)
            elif slot in self._loaded:  # written before, outside prepared batches: wait for all queued compute
                self._copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        self._loaded.update(slot for slot, _ in pairs)
        with torch.cuda.stream(self._copy_stream):
            self._load_flat(pairs)
        self._load_event.record(self._copy_stream)

    def _status_word(self) -> torch.Tensor:
        if self._status is None:
            self._status = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._status

    def _load_flat(self, pairs) -> None:
        by_rank: Dict[int, list] = {}
        for slot, w in pairs:
            by_rank.setdefault(w.rank, []).append((slot, w))
        ops = _native.ops()
        stream = torch.cuda.current_stream(self.device)
        for rank, group in by_rank.items():
            plan = self._plan_for(rank)
            stage = self._ensure_stage(plan.total)
            tables = plan.tables or plan.build_tables(self, self.device)
            for lo in range(0, len(group), _BANK_CHUNK):
                chunk = group[lo: lo + _BANK_CHUNK]
                for i, (_, w) in enumerate(chunk):
                    stage[i].copy_(self._bank_for(w, plan), non_blocking=True)
                slots = torch.tensor([s for s, _ in chunk], dtype=torch.int64).pin_memory()
                slots = slots.to(self.device, non_blocking=True)
                ops.scatter_stage(stage[: len(chunk)], slots, tables["rects"], tables["max_numel"],
                                  self._status_word())
                slots.record_stream(stream)

    def _plan_for(self, rank: int) -> _RankPlan:
        """Bank layout for ``rank`` over the modules known now (one object per (rank, module set))."""
        key = (rank, tuple(self.dims))
        plan = self._plans.get(key)
        if plan is None:
            plan = self._plans[key] = _RankPlan(rank, list(key[1]), self.dims)
        return plan

    def _bank_for(self, weights: AdapterWeights, plan: _RankPlan) -> torch.Tensor:
        """The adapter's pinned bank in ``plan``'s layout.

        The adapter object carries its bank with the layout it was packed for.
        A bank for another layout (the pool learned new modules since) is
        repacked block by block from the old bank, so an adapter whose module
        tensors were released can still follow a growing module set; only an
        adapter with neither tensors nor a bank cannot be packed. Modules the
        adapter lacks are zero in the bank, so a load clears the leading
        ``rank`` rows/columns of its slot there (pool.py:260-299 of the
        reference).
        """
        held = getattr(weights, _BANK_ATTR, None)
        if held is not None and held[0] is plan:
            return held[1]
        bank = torch.zeros(plan.total, dtype=self.dtype, pin_memory=not self.routing_only)
        if held is not None:
            old_plan, old = held
            for key in plan.keys:
                if key not in old_plan.a_off:
                    continue
                for off, old_off, (r, c) in ((plan.a_off[key], old_plan.a_off[key], plan.a_shape[key]),
                                             (plan.b_off[key], old_plan.b_off[key], plan.b_shape[key])):
                    bank[off: off + r * c].copy_(old[old_off: old_off + r * c])
        elif weights.flattened:
            raise RuntimeError(f"adapter (rank {plan.rank}) has neither module tensors nor a packed bank")
        else:
            for key, (a, b) in weights.modules.items():
                if key not in plan.a_off:
                    continue
                for off, t in ((plan.a_off[key], a), (plan.b_off[key], b)):
                    bank[off: off + t.numel()].copy_(t.reshape(-1).to(self.dtype))
        object.__setattr__(weights, _BANK_ATTR, (plan, bank))
        if self.release_modules and weights.modules:
            weights.modules = {}
            weights.flattened = True
        return bank

    def _ensure_stage(self, total: int) -> torch.Tensor:
        """Device stage [_BANK_CHUNK, total], one flat buffer reused across ranks."""
        need = _BANK_CHUNK * total
        if self._stage is None or self._stage.numel() < need:
            self._stage = torch.empty(need, device=self.device, dtype=self.dtype)
        return self._stage[:need].view(_BANK_CHUNK, total)

    def wait_load(self) -> None:
        """Make the compute stream wait for the last load."""
        if self._load_event is not None:
            torch.cuda.current_stream(self.device).wait_event(self._load_event)

    def check_status(self) -> None:
        """Raise if a scatter met an out-of-range rectangle (synchronises)."""
        if self._status is not None and int(self._status.item()):
            raise RuntimeError("mlora: slot-load scatter met an out-of-range descriptor")

    def get(self, module_key: str) -> Tuple[torch.Tensor, torch.Tensor]:
        if self.routing_only:
            raise RuntimeError("routing-only pool (non-CUDA device) holds no weights")
        if module_key not in self.A:
            raise KeyError(f"module {module_key!r} not in pool")
        return self.A[module_key], self.B[module_key]


class LoRAMemoryPool:
    """K device slots; each holds nothing, the base model (``None``) or one adapter.

    name_to_slot / slot_names map adapter names to slot numbers and back;
    _slot_rank_scaling keeps each occupied slot's (rank, scaling).
    """

    def __init__(
        self,
        max_loras_per_batch: int,
        max_lora_rank: int,
        device: torch.device,
        dtype: torch.dtype = torch.float16,
        eviction_policy: str = "lru",
    ) -> None:
        self.max_loras_per_batch = max_loras_per_batch
        self.max_lora_rank = max_lora_rank
        self.device = torch.device(device)
        self.dtype = dtype
        self.eviction_policy = EvictionPolicy(eviction_policy)
        self.name_to_slot: Dict[LoraName, int] = {}
        self.slot_names: Dict[int, LoraName] = {}
        self._slot_rank_scaling: Dict[int, Tuple[int, float]] = {}
        self.buffers = _GpuBuffers(max_loras_per_batch, max_lora_rank, self.device, dtype)

    def get_slot_id(self, name: LoraName) -> int:
        if name not in self.name_to_slot:
            raise KeyError(f"lora {name!r} not resident in pool")
        return self.name_to_slot[name]

    def get_module_buffers(self, module_key: str) -> Tuple[torch.Tensor, torch.Tensor]:
        """All slots of one module: (A [K, max_rank, in], B [K, out, max_rank])."""
        return self.buffers.get(module_key)

    def get_slot_weights(self, slot: int, module_key: str) -> Tuple[torch.Tensor, torch.Tensor]:
        a, b = self.buffers.get(module_key)
        return a[slot], b[slot]

    def ensure_buffers(self, weights: AdapterWeights) -> None:
        self.buffers.ensure(weights)

    def prepare_lora_batch(self, lora_names: Set[LoraName], *, weight_store: Dict[LoraName, AdapterWeights]) -> None:
        """Make every name resident, evicting as needed; one batched load at the end.

        Iteration order over ``lora_names`` decides which free slot each new
        adapter gets, exactly as in pool.py:394-415 (a Python set, so it
        depends on PYTHONHASHSEED).
        """
        for name in lora_names:
            self.eviction_policy.mark_used(name)
        pairs = []
        for name in lora_names:
            if name in self.name_to_slot:
                continue
            slot = self._alloc_slot(lora_names)
            self.name_to_slot[name] = slot
            self.slot_names[slot] = name
            if name is None:
                self._slot_rank_scaling[slot] = (0, 0.0)  # base model: rank 0, no weights
                continue
            w = weight_store[name]
            if w.rank > self.max_lora_rank:
                raise ValueError(f"adapter {name!r} rank {w.rank} > max_lora_rank {self.max_lora_rank}")
            self.buffers.ensure(w)
            self._slot_rank_scaling[slot] = (w.rank, w.scaling)
            pairs.append((slot, w))
        self.buffers.begin_batch({self.name_to_slot[n] for n in lora_names})
        self.buffers.write_many(pairs)
        self.buffers.wait_load()

    def build_batch_info(self, lora_names: List[LoraName]) -> BatchLoRAInfo:
        """Slot per segment; rank and scaling per slot (0 for empty/base slots)."""
        weight_indices = [self.get_slot_id(n) for n in lora_names]
        ranks = [0] * self.max_loras_per_batch
        scalings = [0.0] * self.max_loras_per_batch
        for slot, (r, s) in self._slot_rank_scaling.items():
            ranks[slot] = r
            scalings[slot] = s
        return BatchLoRAInfo(weight_indices=weight_indices, lora_ranks=ranks, scalings=scalings)

    def _alloc_slot(self, keep_names: Set[LoraName]) -> int:
        """First empty slot, else evict an adapter outside this batch (base last)."""
        for slot in range(self.max_loras_per_batch):
            if slot not in self.slot_names:
                return slot
        candidates: Set[LoraName] = set()
        base_evictable = False
        for slot, name in self.slot_names.items():
            if name in keep_names:
                continue
            if name is None:
                base_evictable = True
            else:
                candidates.add(name)
        if not candidates:
            if not base_evictable:
                raise ValueError("no evictable slot: batch needs more adapters than max_loras_per_batch")
            candidates.add(None)
        victim = self.eviction_policy.select_victim(candidates)
        slot = self.name_to_slot.pop(victim)
        self.eviction_policy.remove(victim)
        self.slot_names.pop(slot)
        self._slot_rank_scaling.pop(slot, None)
        return slot
