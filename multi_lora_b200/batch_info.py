"""Segment routing metadata: CPU lists and the resident device tensors.

Drop-in for ``multi_lora/batch_info.py`` (same names, fields, padding and
in-place semantics). The device side differs in one respect: the five
columns of :class:`KernelInputMetaData` are views into ONE device buffer that
is refreshed by ONE pinned host->device copy per step, instead of one pageable
copy per column (batch_info.py:100-110 of the reference).

Column contents and padding follow write_kernel_input_metadata
(batch_info.py:128-179): weight_indices / lora_ranks / seg_lens are padded
with 0, seg_indptr with the total row count (so it stays non-decreasing),
scalings with 0.0. Columns keep their addresses while the batch fits the
capacity, so CUDA graphs captured against them stay valid.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np
import torch


@dataclass
class BatchLoRAInfo:
    """Slot routing of one batch on the host (batch_info.py:16-22)."""

    weight_indices: List[int]  # one entry per segment: its slot
    lora_ranks: List[int]      # one entry per slot: its rank (0 = base model)
    scalings: List[float]      # one entry per slot: its scaling


@dataclass
class KernelInputMetaData:
    """Device routing tables read by the kernels (batch_info.py:25-42).

    Segment i covers token rows [seg_indptr[i], seg_indptr[i+1]) and uses slot
    weight_indices[i]; slot s has rank lora_ranks[s] and scaling scalings[s].
    ``bs`` and ``max_len`` are host ints.
    """

    bs: int
    seg_lens: torch.Tensor
    seg_indptr: torch.Tensor
    weight_indices: torch.Tensor
    lora_ranks: torch.Tensor
    scalings: torch.Tensor
    max_len: int
    # packed storage behind the five columns (None for user-built metadata)
    _packed: Optional["_PackedColumns"] = field(default=None, repr=False, compare=False)


def segment_lens(bs: int, seq_lens: List[int]) -> Tuple[List[int], List[int]]:
    """Tokens per segment and their exclusive prefix (batch_info.py:45-67).

    ``seq_lens == []`` means decode: every segment is one token.
    """
    lens, indptr = _segment_arrays(bs, seq_lens)
    return lens.tolist(), indptr.tolist()


def _segment_arrays(bs: int, seq_lens: List[int]) -> Tuple[np.ndarray, np.ndarray]:
    """``segment_lens`` as int64 arrays (the per-step write path)."""
    if len(seq_lens):
        if len(seq_lens) != bs:
            raise AssertionError(f"seq_lens needs one entry per segment: {len(seq_lens)} vs {bs}")
        lens = np.asarray(seq_lens, dtype=np.int64)
    else:
        lens = np.ones(bs, dtype=np.int64)
    indptr = np.zeros(bs + 1, dtype=np.int64)
    np.cumsum(lens, out=indptr[1:])
    return lens, indptr


def group_rows(names: list, seq_lens: List[int]) -> Tuple[list, List[int]]:
    """Run-length merge of ADJACENT rows with the same adapter name.

    Mirrors batch_info.py:70-97: row order is never changed (KV-cache rows
    stay aligned); only neighbours merge. Decode rows (``seq_lens == []``)
    count one token each; prefill rows add their token counts.
    """
    row_lens = [int(n) for n in seq_lens] if seq_lens else [1] * len(names)
    if len(row_lens) != len(names):
        raise ValueError(f"seq_lens({len(row_lens)}) must match names({len(names)})")
    out_names: list = []
    out_lens: List[int] = []
    for name, n in zip(names, row_lens):
        if out_names and out_names[-1] == name:
            out_lens[-1] += n
        else:
            out_names.append(name)
            out_lens.append(n)
    return out_names, out_lens


def fill_column(column: torch.Tensor, values: list, pad: float) -> None:
    """Overwrite a whole column in place: values, then ``pad`` (batch_info.py:100-110)."""
    size = column.shape[0]
    if len(values) > size:
        raise AssertionError(f"{len(values)} values do not fit {size} entries")
    host = torch.full((size,), pad, dtype=column.dtype)
    if values:
        host[: len(values)] = torch.tensor(values, dtype=column.dtype)
    column.copy_(host)


def empty_kernel_input_metadata(*, device: torch.device, dtype: torch.dtype) -> KernelInputMetaData:
    """Zero-capacity metadata; the first write allocates (batch_info.py:113-125)."""
    i32 = dict(dtype=torch.int32, device=device)
    return KernelInputMetaData(
        bs=0,
        seg_lens=torch.empty(0, **i32),
        seg_indptr=torch.empty(0, **i32),
        weight_indices=torch.empty(0, **i32),
        lora_ranks=torch.empty(0, **i32),
        scalings=torch.empty(0, dtype=dtype, device=device),
        max_len=0,
    )


class _PackedColumns:
    """One device int32 buffer holding all five columns, plus its pinned twin.

    Layout (int32 words): seg_lens[cap] | seg_indptr[cap+1] | weight_indices[cap]
    | lora_ranks[K] | scalings (K elements of the model dtype, padded to words).
    """

    def __init__(self, cap: int, num_slots: int, device: torch.device, dtype: torch.dtype):
        self.cap, self.k, self.dtype = cap, num_slots, dtype
        es = torch.empty(0, dtype=dtype).element_size()
        self.scal_words = (num_slots * es + 3) // 4
        self.o_lens, self.o_indptr = 0, cap
        self.o_widx = 2 * cap + 1
        self.o_ranks = 3 * cap + 1
        self.o_scal = self.o_ranks + num_slots
        self.words = self.o_scal + self.scal_words
        self.device = torch.device(device)
        self.dev = torch.zeros(self.words, dtype=torch.int32, device=self.device)
        pin = self.device.type == "cuda"
        self.host = torch.zeros(self.words, dtype=torch.int32, pin_memory=pin)
        self.copy_done: Optional[torch.cuda.Event] = None
        self._scal_src: Optional[list] = None  # scalings last converted, and their words
        self._scal_words: Optional[np.ndarray] = None

    def views(self):
        d = self.dev
        scal = d[self.o_scal: self.o_scal + self.scal_words].view(self.dtype)[: self.k]
        return (d[self.o_lens: self.o_lens + self.cap], d[self.o_indptr: self.o_indptr + self.cap + 1],
                d[self.o_widx: self.o_widx + self.cap], d[self.o_ranks: self.o_ranks + self.k], scal)

    def write(self, lens, indptr, widx, ranks, scalings) -> None:
        if self.copy_done is not None:
            # the previous step's async copy still reads the pinned buffer
            self.copy_done.synchronize()
        h = self.host.numpy()
        total = indptr[-1]
        cap, k = self.cap, self.k
        h[self.o_lens: self.o_lens + cap] = 0
        h[self.o_lens: self.o_lens + len(lens)] = lens
        h[self.o_indptr: self.o_indptr + cap + 1] = total
        h[self.o_indptr: self.o_indptr + len(indptr)] = indptr
        h[self.o_widx: self.o_widx + cap] = 0
        h[self.o_widx: self.o_widx + len(widx)] = widx
        h[self.o_ranks: self.o_ranks + k] = 0
        h[self.o_ranks: self.o_ranks + len(ranks)] = ranks
        scalings = list(scalings)
        if scalings != self._scal_src:  # converted again only when they change
            es = torch.empty(0, dtype=self.dtype).element_size()
            scal = torch.zeros(self.scal_words * 4 // es, dtype=self.dtype)
            if scalings:
                scal[: len(scalings)] = torch.tensor(scalings, dtype=torch.float64).to(self.dtype)
            self._scal_src, self._scal_words = scalings, scal.view(torch.int32).numpy().copy()
        h[self.o_scal: self.o_scal + self.scal_words] = self._scal_words
        if self.device.type == "cuda":
            self.dev.copy_(self.host, non_blocking=True)
            if self.copy_done is None:
                self.copy_done = torch.cuda.Event()
            self.copy_done.record()
        else:
            self.dev.copy_(self.host)


def _validate(pool_batch: BatchLoRAInfo, lens: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Host-side routing checks, done before the lists leave the host; returns
    weight_indices and lora_ranks as int64 arrays."""
    k = len(pool_batch.lora_ranks)
    if len(pool_batch.scalings) != k:
        raise ValueError(f"scalings has {len(pool_batch.scalings)} entries, lora_ranks {k}")
    widx = np.asarray(pool_batch.weight_indices, dtype=np.int64).reshape(-1)
    if widx.size and (widx.min() < 0 or widx.max() >= k):  # the first offender is named
        i = int(np.flatnonzero((widx < 0) | (widx >= k))[0])
        raise ValueError(f"weight_indices[{i}] = {pool_batch.weight_indices[i]} outside [0, {k})")
    ranks = np.asarray(pool_batch.lora_ranks, dtype=np.int64).reshape(-1)
    if ranks.size and ranks.min() < 0:
        s = int(np.flatnonzero(ranks < 0)[0])
        raise ValueError(f"lora_ranks[{s}] = {pool_batch.lora_ranks[s]} is negative")
    if lens.size and lens.min() < 0:
        i = int(np.flatnonzero(lens < 0)[0])
        raise ValueError(f"segment {i} has negative length {int(lens[i])}")
    return widx, ranks


def write_kernel_input_metadata(
    meta: KernelInputMetaData,
    pool_batch: BatchLoRAInfo,
    *,
    device: torch.device,
    dtype: torch.dtype,
    seq_lens: List[int],
) -> KernelInputMetaData:
    """Write this batch's routing into ``meta`` (batch_info.py:128-179).

    In place when the batch fits the current capacity (same object, same
    addresses); otherwise new tables sized for this batch. lora_ranks and
    scalings always have one entry per pool slot.
    """
    rows = len(pool_batch.weight_indices)
    lens, indptr = _segment_arrays(rows, seq_lens)
    widx, ranks = _validate(pool_batch, lens)
    max_len = int(lens.max()) if rows else 0
    if rows > meta.weight_indices.shape[0]:
        # does not fit: new tables sized for this batch
        packed = _PackedColumns(rows, len(pool_batch.lora_ranks), device, dtype)
        cols = packed.views()
        meta = KernelInputMetaData(bs=rows, seg_lens=cols[0], seg_indptr=cols[1], weight_indices=cols[2],
                                   lora_ranks=cols[3], scalings=cols[4], max_len=max_len, _packed=packed)
    elif meta._packed is None:
        # user-built metadata with room: column-by-column refresh, as the reference does
        fill_column(meta.weight_indices, widx.tolist(), 0)
        fill_column(meta.lora_ranks, ranks.tolist(), 0)
        fill_column(meta.seg_lens, lens.tolist(), 0)
        fill_column(meta.seg_indptr, indptr.tolist(), int(indptr[-1]))
        fill_column(meta.scalings, pool_batch.scalings, 0.0)
        meta.bs, meta.max_len = rows, max_len
        return meta
    packed = meta._packed
    if len(pool_batch.lora_ranks) > packed.k:
        raise AssertionError(f"{len(pool_batch.lora_ranks)} slots do not fit {packed.k} entries")
    packed.write(lens, indptr, widx, ranks, pool_batch.scalings)
    meta.bs = rows
    meta.max_len = max_len
    return meta
