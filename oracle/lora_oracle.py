"""CPU oracle for the multi-LoRA hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
may import this module, and only as the checker; the product
(``multi_lora_b200``) never does.

It restates, in numpy, the algorithm of the reference project's pure-PyTorch
path (Rick0037/multi_lora; citations are file:line within that project):

* routing tables: batch_info.py:45-179
* shrink / expand per segment: backend/torch_backend.py:17-90
* row-wise delta: layers.py:23-39
* RMSNorm arithmetic: kernels/rmsnorm.py:38-52
* slot pool + eviction: pool.py:382-473, eviction.py:12-50
* bank layout + scatter: pool.py:23-94, 186-299; kernels/scatter_bank.py:18-65

Parity of this oracle is PINNED against vectors produced by running the
reference's own code in the build container (``tests/golden/make_golden.py``
writes ``tests/golden/*.npz|json``; ``tests/test_oracle_golden.py`` checks the
oracle against them). bf16 is emulated on float32 arrays with
round-to-nearest-even, which is what torch does for bf16 tensors on the CPU.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Set, Tuple

import numpy as np

# ----------------------------------------------------------------------------
# element types
# ----------------------------------------------------------------------------


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    # NaN stays NaN
    return np.where(np.isnan(a), a, out)


def f16_round(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "f16":
        return f16_round(a)
    return np.asarray(a, dtype=np.float32)


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """uint16 storage of float32 values that are already bf16-exact."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------
# routing tables (batch_info.py)
# ----------------------------------------------------------------------------


def segment_lens(bs: int, seq_lens: Sequence[int]) -> Tuple[List[int], List[int]]:
    """batch_info.py:45-67: decode (empty seq_lens) is one token per segment."""
    lens = [int(v) for v in seq_lens] if seq_lens else [1] * bs
    assert len(lens) == bs
    indptr = [0]
    for n in lens:
        indptr.append(indptr[-1] + n)
    return lens, indptr


def group_rows(names: list, seq_lens: Sequence[int]) -> Tuple[list, List[int]]:
    """batch_info.py:70-97: merge only ADJACENT equal names."""
    row_lens = [int(v) for v in seq_lens] if seq_lens else [1] * len(names)
    if len(row_lens) != len(names):
        raise ValueError("seq_lens must match names")
    gn: list = []
    gl: List[int] = []
    for name, n in zip(names, row_lens):
        if gn and gn[-1] == name:
            gl[-1] += n
        else:
            gn.append(name)
            gl.append(n)
    return gn, gl


def metadata_columns(weight_indices: List[int], lora_ranks: List[int], scalings: List[float],
                     seq_lens: Sequence[int], capacity: int) -> dict:
    """Column contents after write_kernel_input_metadata (batch_info.py:128-179).

    ``capacity`` is the column length the tables had (they grow to the batch
    size when it does not fit). Padding: indices/ranks/lens 0, indptr the
    total row count, scalings 0.0.
    """
    rows = len(weight_indices)
    lens, indptr = segment_lens(rows, seq_lens)
    cap = max(capacity, rows)
    pad = lambda v, n, p: list(v) + [p] * (n - len(v))  # noqa: E731
    return {
        "bs": rows,
        "max_len": max(lens) if lens else 0,
        "seg_lens": pad(lens, cap, 0),
        "seg_indptr": pad(indptr, cap + 1, indptr[-1]),
        "weight_indices": pad(weight_indices, cap, 0),
        "lora_ranks": list(lora_ranks),
        "scalings": list(scalings),
    }


# ----------------------------------------------------------------------------
# shrink / expand (backend/torch_backend.py)
# ----------------------------------------------------------------------------


def _segments(indptr, widx, bs):
    for seg in range(bs):
        start, end = int(indptr[seg]), int(indptr[seg + 1])
        if start >= end:
            continue
        yield start, end, int(widx[seg])


def shrink(x: np.ndarray, A: np.ndarray, indptr, widx, ranks, bs: int, dtype: str = "f32",
           out: Optional[np.ndarray] = None) -> np.ndarray:
    """torch_backend.py:17-49: mid[start:end, :r] = dtype(x[start:end] @ A[slot, :r].T).

    x [S, in], A [K, R, in] hold dtype-exact float32 values; accumulation is
    float32 (torch's CPU bf16 matmul also accumulates in float32 and rounds
    once). Untouched entries keep ``out``'s values (zeros by default, like
    the Torch backend's buffer).
    """
    S = x.shape[0]
    R = A.shape[1]
    mid = np.zeros((S, R), np.float32) if out is None else out.copy()
    for start, end, slot in _segments(indptr, widx, bs):
        r = int(ranks[slot])
        if r == 0:
            continue
        acc = x[start:end].astype(np.float32) @ A[slot, :r, :].astype(np.float32).T
        mid[start:end, :r] = round_to(acc, dtype)
    return mid


def expand(mid: np.ndarray, B: np.ndarray, indptr, widx, ranks, scalings, bs: int, y: np.ndarray,
           dtype: str = "f32") -> np.ndarray:
    """torch_backend.py:51-90 with base_output given:
    delta = dtype(dtype(mid[:, :r] @ B[slot, :, :r].T) * dtype(scaling)); y = dtype(y + delta)."""
    y = y.astype(np.float32).copy()
    for start, end, slot in _segments(indptr, widx, bs):
        r = int(ranks[slot])
        if r == 0:
            continue
        prod = round_to(mid[start:end, :r].astype(np.float32) @ B[slot, :, :r].astype(np.float32).T, dtype)
        scale = round_to(np.float32(scalings[slot]), dtype)
        delta = round_to(prod * scale, dtype)
        y[start:end] = round_to(y[start:end] + delta, dtype)
    return y


def apply_lora_fp32(x, A, B, indptr, widx, ranks, scalings, bs, y) -> np.ndarray:
    """The parity target: the same per-segment math entirely in float32
    (inputs upcast; no intermediate rounding)."""
    y = y.astype(np.float32).copy()
    for start, end, slot in _segments(indptr, widx, bs):
        r = int(ranks[slot])
        if r == 0:
            continue
        mid = x[start:end].astype(np.float32) @ A[slot, :r].astype(np.float32).T
        y[start:end] += np.float32(scalings[slot]) * (mid @ B[slot, :, :r].astype(np.float32).T)
    return y


def lora_delta(x, a, b, scaling, rank) -> np.ndarray:
    """layers.py:23-39: scaling * x @ A[:rank].T @ B[:, :rank].T."""
    flat = x.reshape(-1, x.shape[-1]).astype(np.float32)
    d = (flat @ a[:rank].astype(np.float32).T @ b[:, :rank].astype(np.float32).T) * np.float32(scaling)
    return d.reshape(*x.shape[:-1], b.shape[0])


# ----------------------------------------------------------------------------
# RMSNorm (kernels/rmsnorm.py:38-52)
# ----------------------------------------------------------------------------


def rmsnorm_f32(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """(x_f32 * rsqrt(sum(x^2)/H + eps)) * w_f32 before the final cast (rmsnorm.py:38-44)."""
    xf = x.astype(np.float32)
    h = xf.shape[-1]
    var = (xf * xf).sum(axis=-1, keepdims=True, dtype=np.float32) / np.float32(h)
    rstd = (1.0 / np.sqrt(var.astype(np.float64) + eps)).astype(np.float32)
    return (xf * rstd) * w.astype(np.float32)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, dtype: str = "bf16") -> np.ndarray:
    """y = dtype((x_f32 * rsqrt(sum(x^2)/H + eps)) * w_f32), per row of the last dim
    (round-to-nearest-even cast, as the kernel does on the GPU)."""
    return round_to(rmsnorm_f32(x, w, eps), dtype)


def bf16_truncate(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 by dropping the low 16 bits (the Triton CPU interpreter's cast)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    return ((a.view(np.uint32) >> 16) << 16).view(np.float32)


# ----------------------------------------------------------------------------
# slot pool + eviction (pool.py, eviction.py)
# ----------------------------------------------------------------------------


class EvictionOracle:
    """eviction.py:12-50."""

    def __init__(self, kind: str = "lru"):
        assert kind in ("lru", "fifo")
        self.kind = kind
        self.order: "OrderedDict[str, None]" = OrderedDict()
        self.eviction_count = 0

    def mark_used(self, name):
        if name is None:
            return
        if self.kind == "lru":
            self.order.pop(name, None)
        self.order[name] = None

    def select_victim(self, candidates):
        for name in self.order:
            if name in candidates:
                self.eviction_count += 1
                return name
        if None in candidates:
            self.eviction_count += 1
            return None
        raise RuntimeError("no evictable adapter")

    def remove(self, name):
        if name is not None:
            self.order.pop(name, None)


class SlotPoolOracle:
    """Residency / victim choice of LoRAMemoryPool (pool.py:382-473), no weights.

    ``ranks`` maps adapter name -> (rank, scaling); None is the base model.
    """

    def __init__(self, num_slots: int, max_rank: int, ranks: Dict[Optional[str], Tuple[int, float]],
                 policy: str = "lru"):
        self.k, self.max_rank, self.ranks = num_slots, max_rank, ranks
        self.ev = EvictionOracle(policy)
        self.name_to_slot: Dict[Optional[str], int] = {}
        self.slot_names: Dict[int, Optional[str]] = {}
        self.rank_scaling: Dict[int, Tuple[int, float]] = {}
        self.loads: List[Tuple[int, Optional[str]]] = []  # (slot, name) in load order

    def prepare(self, names: Set[Optional[str]]) -> None:
        for n in names:
            self.ev.mark_used(n)
        for n in names:
            if n in self.name_to_slot:
                continue
            slot = self._alloc(names)
            self.name_to_slot[n] = slot
            self.slot_names[slot] = n
            if n is None:
                self.rank_scaling[slot] = (0, 0.0)
                continue
            r, s = self.ranks[n]
            if r > self.max_rank:
                raise ValueError("rank > max_lora_rank")
            self.rank_scaling[slot] = (r, s)
            self.loads.append((slot, n))

    def _alloc(self, keep) -> int:
        for s in range(self.k):
            if s not in self.slot_names:
                return s
        cands = {n for n in self.slot_names.values() if n not in keep and n is not None}
        base = any(n is None and n not in keep for n in self.slot_names.values())
        if not cands:
            if not base:
                raise ValueError("no evictable slot")
            cands = {None}
        victim = self.ev.select_victim(cands)
        slot = self.name_to_slot.pop(victim)
        self.ev.remove(victim)
        self.slot_names.pop(slot)
        self.rank_scaling.pop(slot, None)
        return slot

    def batch_info(self, names: List[Optional[str]]):
        widx = [self.name_to_slot[n] for n in names]
        ranks = [0] * self.k
        scal = [0.0] * self.k
        for s, (r, sc) in self.rank_scaling.items():
            ranks[s], scal[s] = r, sc
        return widx, ranks, scal


# ----------------------------------------------------------------------------
# bank layout + scatter (pool.py:23-94, kernels/scatter_bank.py:18-65)
# ----------------------------------------------------------------------------


def rank_plan(rank: int, keys: List[str], dims: Dict[str, Tuple[int, int]]) -> dict:
    """Offsets of the flat bank: A blocks of all keys, then B blocks (dims = (in, out))."""
    a_off, b_off, pos = {}, {}, 0
    for k in keys:
        a_off[k] = pos
        pos += rank * dims[k][0]
    for k in keys:
        b_off[k] = pos
        pos += dims[k][1] * rank
    return {"a_off": a_off, "b_off": b_off, "total": pos}


def build_bank(rank: int, keys: List[str], dims, modules: Dict[str, Tuple[np.ndarray, np.ndarray]]) -> np.ndarray:
    """pool.py:260-299: missing modules are zero in the bank."""
    plan = rank_plan(rank, keys, dims)
    flat = np.zeros(plan["total"], np.float32)
    for k in keys:
        if k not in modules:
            continue
        a, b = modules[k]
        flat[plan["a_off"][k]: plan["a_off"][k] + a.size] = a.reshape(-1)
        flat[plan["b_off"][k]: plan["b_off"][k] + b.size] = b.reshape(-1)
    return flat


def scatter_bank(bank: np.ndarray, rank: int, keys: List[str], dims, A: Dict[str, np.ndarray],
                 B: Dict[str, np.ndarray], slot: int) -> None:
    """kernels/scatter_bank.py:18-65 semantics: A[k][slot, :r, :] and B[k][slot, :, :r]
    take the bank blocks; entries past the rank are left as they were."""
    plan = rank_plan(rank, keys, dims)
    for k in keys:
        n_in, n_out = dims[k]
        A[k][slot, :rank, :] = bank[plan["a_off"][k]: plan["a_off"][k] + rank * n_in].reshape(rank, n_in)
        B[k][slot, :, :rank] = bank[plan["b_off"][k]: plan["b_off"][k] + n_out * rank].reshape(n_out, rank)
