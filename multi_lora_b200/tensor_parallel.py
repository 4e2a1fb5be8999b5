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

Only the ``[S, R]`` partials cross NVLink (64 KiB at S=1024, R=16).
"""

from __future__ import annotations

from typing import Optional, Tuple

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


def row_parallel_apply(backend, x_shard: torch.Tensor, a_shard: torch.Tensor, b_shard: torch.Tensor,
                       y_partial: torch.Tensor, tp_rank: int, tp_size: int,
                       group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
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
    partial = backend.shrink_partial(x_shard, a_shard)
    if tp_size > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    backend.expand_partial(partial, b_shard, y_partial[:, lo:hi])
    return y_partial
