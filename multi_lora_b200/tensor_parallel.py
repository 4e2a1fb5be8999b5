"""Tensor-parallel LoRA: how the slot stacks shard and what each TP rank runs.

The reference has no tensor parallelism; this module extends its
``LoRABackend.apply_lora`` (backend/base.py:60-89) to a TP group the way the
path shards naturally (Megatron-style column / row parallel projections):

* column-parallel projections (q, k, v, gate, up): x is replicated, the A stack
  ``[K, R, in]`` is replicated, the B stack is column-sharded
  ``B[:, lo:hi, :]`` with ``[lo, hi)`` the rank's slice of ``out``. Each rank
  computes the full ``mid`` and the delta of its own output slice. No
  collective.
* row-parallel projections (o, down): x is sharded on ``in``, A is row-sharded
  ``A[:, :, lo:hi]``. Each rank computes the fp32 partial
  ``mid_p = x_p @ A_p[slot, :r].T``; one all-reduce (sum) over the TP group of
  the ``[S, R]`` fp32 partials gives the fp32 ``mid`` (rounded to the
  activation dtype before the expand, as the unsharded path rounds it). The B
  stack is column-sharded as for column layers and each rank adds the delta
  of ITS output columns into its pre-all-reduce partial output
  ``y_partial[S, out]``, so the model's own row-parallel output all-reduce
  completes the sum exactly once.

Only the ``[S, R]`` partials cross NVLink (64 KiB at S=1024, R=16). Two
ways to sum them: an NCCL all-reduce (the baseline), or a
:class:`PeerExchange`, where the shrink kernel stores each finished tile of
partial value into every rank's buffer over NVLink as an 8-byte word tagged
with the call, and the expand kernel polls the words until they carry the
call's tag and sums the ranks' values itself (no separate collective, memset
or launch; ``mlora_row_parallel_apply_p2p``).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

COLUMN = "column"
ROW = "row"

# projection -> how a Llama-style block shards it
LLAMA_TP_KIND = {
    "q_proj": COLUMN, "k_proj": COLUMN, "v_proj": COLUMN, "gate_proj": COLUMN, "up_proj": COLUMN,
    "o_proj": ROW, "down_proj": ROW,
}


def shard_bounds(n: int, tp_rank: int, tp_size: int) -> Tuple[int, int]:
    """[lo, hi) of rank ``tp_rank``'s equal slice of ``n`` (``n % tp_size == 0``)."""
    if tp_size < 1 or not 0 <= tp_rank < tp_size:
        raise ValueError(f"tp_rank {tp_rank} outside [0, {tp_size})")
    if n % tp_size != 0:
        raise ValueError(f"dimension {n} does not split evenly over {tp_size} ranks")
    part = n // tp_size
    return tp_rank * part, (tp_rank + 1) * part


def shard_lora_stacks(a_stack: torch.Tensor, b_stack: torch.Tensor, kind: str, tp_rank: int,
                      tp_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """This rank's (A, B) stacks for a ``kind`` ("column" | "row") projection.

    a_stack ``[K, R, in]``, b_stack ``[K, out, R]`` (the pool layout). B is
    column-sharded for both kinds; A is replicated (column) or row-sharded on
    ``in`` (row). Returned shards are contiguous copies.
    """
    if a_stack.dim() != 3 or b_stack.dim() != 3 or a_stack.shape[0] != b_stack.shape[0]:
        raise ValueError("expected A [K, R, in] and B [K, out, R] with the same K")
    lo, hi = shard_bounds(b_stack.shape[1], tp_rank, tp_size)
    b = b_stack[:, lo:hi, :].contiguous()
    if kind == COLUMN:
        return a_stack, b
    if kind == ROW:
        ilo, ihi = shard_bounds(a_stack.shape[2], tp_rank, tp_size)
        return a_stack[:, :, ilo:ihi].contiguous(), b
    raise ValueError(f"unknown tensor-parallel kind {kind!r}")


def column_parallel_apply(backend, x: torch.Tensor, a_stack: torch.Tensor, b_shard: torch.Tensor,
                          y_local: torch.Tensor) -> torch.Tensor:
    """Column-parallel projection: ``y_local [S, out/tp]`` (the rank's output
    shard) += delta of its columns. Same call as the unsharded apply_lora."""
    return backend.apply_lora(x, a_stack, b_shard, y_local)


class PeerExchange:
    """One rank's end of the row-parallel partial exchange over peer memory.

    Every rank owns one zeroed device buffer (tagged partial words, the call
    counter) made by ``mlora_peer_buffer_create``; the ranks trade CUDA IPC
    handles and map each other's buffers (:meth:`create`). Every rank must
    then run the same row-parallel calls in the same order. ``max_rows``
    bounds the rows of a call.
    """

    def __init__(self, tp: int, rank: int, max_rows: int, max_rank: int, buffers: List[int], owned: bool,
                 opened: List[int]):
        self.tp, self.rank = tp, rank
        self.max_rows, self.max_rank = max_rows, max_rank
        self.buffers = list(buffers)
        self._owned = owned
        self._opened = list(opened)
        self._struct = None

    @staticmethod
    def _create_buffer(nbytes: int):
        from multi_lora_b200 import _native

        lib = _native.capi()
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _native.check(lib.mlora_peer_buffer_create(nbytes, ctypes.byref(ptr), handle))
        return ptr.value, bytes(handle)

    @classmethod
    def create(cls, *, device: torch.device, max_rows: int, max_rank: int,
               group: Optional[dist.ProcessGroup] = None) -> "PeerExchange":
        """Collective over ``group``: make this rank's buffer and map every peer's."""
        from multi_lora_b200 import _native

        tp, rank = dist.get_world_size(group), dist.get_rank(group)
        lib = _native.capi()
        nbytes = lib.mlora_peer_exchange_bytes(tp, max_rows, max_rank)
        if nbytes == 0:
            raise ValueError(f"exchange sizes out of range (tp={tp}, rows={max_rows}, rank={max_rank})")
        with torch.cuda.device(device):
            own, handle = cls._create_buffer(nbytes)
            handles: list = [None] * tp
            dist.all_gather_object(handles, handle, group=group)
            bufs, opened = [], []
            for q, h in enumerate(handles):
                if q == rank:
                    bufs.append(own)
                    continue
                ptr = ctypes.c_void_p()
                hb = (ctypes.c_char * 64).from_buffer_copy(h)
                _native.check(lib.mlora_peer_buffer_open(hb, ctypes.byref(ptr)))
                bufs.append(ptr.value)
                opened.append(ptr.value)
        return cls(tp, rank, max_rows, max_rank, bufs, True, opened)

    @classmethod
    def local_group(cls, tp: int, *, device: torch.device, max_rows: int, max_rank: int) -> List["PeerExchange"]:
        """``tp`` ranks' exchanges in one process on one GPU (every buffer local).
        Drive them with phase 1 for every rank, then phase 2 for every rank,
        so that no kernel waits for one queued after it."""
        from multi_lora_b200 import _native

        nbytes = _native.capi().mlora_peer_exchange_bytes(tp, max_rows, max_rank)
        with torch.cuda.device(device):
            bufs = [cls._create_buffer(nbytes)[0] for _ in range(tp)]
        out = [cls(tp, r, max_rows, max_rank, bufs, False, []) for r in range(tp)]
        out[0]._owned_all = bufs  # rank 0's object frees every buffer
        return out

    def struct(self):
        from multi_lora_b200 import _native

        if self._struct is None:
            st = _native.PeerExchangeT()
            st.tp, st.rank, st.max_rows, st.max_rank = self.tp, self.rank, self.max_rows, self.max_rank
            for q, b in enumerate(self.buffers):
                st.buffers[q] = b
            self._struct = st
        return self._struct

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after all use has completed)."""
        from multi_lora_b200 import _native

        lib = _native.capi()
        for p in self._opened:
            _native.check(lib.mlora_peer_buffer_close(ctypes.c_void_p(p)))
        self._opened = []
        if self._owned:
            _native.check(lib.mlora_peer_buffer_destroy(ctypes.c_void_p(self.buffers[self.rank])))
            self._owned = False
        for b in getattr(self, "_owned_all", []):
            _native.check(lib.mlora_peer_buffer_destroy(ctypes.c_void_p(b)))
        self._owned_all = []


def row_parallel_apply_p2p(backend, x_shard: torch.Tensor, a_shard: torch.Tensor, b_shard: torch.Tensor,
                           y_cols: torch.Tensor, exchange: PeerExchange, phase: int = 0) -> torch.Tensor:
    """The row-parallel projection with the partials exchanged over peer memory
    (``mlora_row_parallel_apply_p2p``): ``y_cols`` (this rank's output columns of
    the pre-all-reduce partial output) is updated in place."""
    from multi_lora_b200 import _native

    meta = backend._meta()
    if x_shard.stride(1) != 1 or y_cols.stride(1) != 1:
        raise ValueError("x_shard and y_cols need unit column stride")
    ms = _native.meta_struct(meta)
    rc = _native.capi().mlora_row_parallel_apply_p2p(
        x_shard.data_ptr(), x_shard.shape[0], x_shard.shape[1], x_shard.stride(0), a_shard.data_ptr(),
        b_shard.data_ptr(), b_shard.shape[1], a_shard.shape[1], ctypes.byref(ms), y_cols.data_ptr(),
        y_cols.stride(0), ctypes.byref(exchange.struct()), phase, _native.dtype_code(x_shard.dtype),
        backend.status_word(x_shard.device).data_ptr(), torch.cuda.current_stream(x_shard.device).cuda_stream)
    _native.check(rc)
    return y_cols


def row_parallel_apply(backend, x_shard: torch.Tensor, a_shard: torch.Tensor, b_shard: torch.Tensor,
                       y_partial: torch.Tensor, tp_rank: int, tp_size: int,
                       group: Optional[dist.ProcessGroup] = None,
                       exchange: Optional[PeerExchange] = None) -> torch.Tensor:
    """Row-parallel projection on one TP rank.

    x_shard ``[S, in/tp]``; a_shard ``[K, R, in/tp]``; b_shard ``[K, out/tp, R]``;
    y_partial ``[S, out]`` is the rank's base partial output before the
    model's all-reduce. Updated in place: columns ``shard_bounds(out)`` get
    this rank's delta. Every rank of the group must call this in the same
    order (one all-reduce per call).
    """
    if y_partial.dim() != 2 or y_partial.stride(1) != 1:
        raise ValueError("y_partial must be [S, out] with unit column stride")
    lo, hi = shard_bounds(y_partial.shape[1], tp_rank, tp_size)
    if b_shard.shape[1] != hi - lo:
        raise ValueError(f"b_shard has {b_shard.shape[1]} output rows, the rank's slice has {hi - lo}")
    if exchange is not None:  # partials summed by the expand kernel from the peers' stores
        row_parallel_apply_p2p(backend, x_shard.contiguous(), a_shard, b_shard, y_partial[:, lo:hi], exchange)
        return y_partial
    partial = backend.shrink_partial(x_shard, a_shard)
    if tp_size > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    backend.expand_partial(partial, b_shard, y_partial[:, lo:hi])
    return y_partial
