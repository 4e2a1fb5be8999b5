"""LoRA backend interface (drop-in for ``multi_lora/backend/base.py:13-89``)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Optional

import torch

from multi_lora_b200.batch_info import KernelInputMetaData


class LoRABackend(ABC):
    """Segment-routed LoRA: each segment picks its adapter slot's weights."""

    name: str = "abstract"

    def __init__(self) -> None:
        self.kernel_input_metadata: Optional[KernelInputMetaData] = None
        # resident (rows, max_rank) shrink output, reused while it fits (base.py:24-38)
        self._mid = torch.empty((0, 0))
        self._partial = torch.empty((0, 0))

    def mid_buffer(self, rows: int, max_rank: int, like: torch.Tensor) -> torch.Tensor:
        """A (rows, max_rank) buffer; the same storage is reused while it fits.

        The width is fixed at max_rank, so the leading-rows slice stays contiguous.
        """
        m = self._mid
        if m.shape[0] < rows or m.shape[1] != max_rank or m.device != like.device or m.dtype != like.dtype:
            self._mid = torch.empty((rows, max_rank), dtype=like.dtype, device=like.device)
        return self._mid[:rows]

    def partial_buffer(self, rows: int, max_rank: int, like: torch.Tensor) -> torch.Tensor:
        """A resident fp32 (rows, max_rank) buffer for tensor-parallel shrink
        partials (same reuse rule as ``mid_buffer``)."""
        m = self._partial
        if m.shape[0] < rows or m.shape[1] != max_rank or m.device != like.device:
            self._partial = torch.empty((rows, max_rank), dtype=torch.float32, device=like.device)
        return self._partial[:rows]

    def shrink_partial(self, x: torch.Tensor, a_shard: torch.Tensor) -> torch.Tensor:
        """Tensor-parallel shrink: the unrounded fp32 ``x @ A[slot, :rank].T``
        of this rank's input slice, zero where no adapter column is written."""
        raise NotImplementedError(f"{type(self).__name__} has no tensor-parallel shrink")

    def expand_partial(self, partial: torch.Tensor, b_shard: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Tensor-parallel expand from the all-reduced fp32 ``partial`` (rounded
        to y's dtype first, as the unsharded mid is) into ``y`` in place."""
        raise NotImplementedError(f"{type(self).__name__} has no tensor-parallel expand")

    def set_kernel_input_metadata(self, metadata: KernelInputMetaData) -> None:
        """Bind this step's segment/slot routing."""
        self.kernel_input_metadata = metadata

    @abstractmethod
    def run_lora_a_sgemm(self, x: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """Shrink: x [S, in] with A[slot, :rank, :] -> mid [S, max_rank]; weights [K, max_rank, in]."""

    @abstractmethod
    def run_lora_b_sgemm(
        self,
        x: torch.Tensor,
        weights: torch.Tensor,
        base_output: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        """Expand: mid [S, r] with B[slot, :, :rank] * scaling, added into base_output."""

    def apply_lora(
        self,
        x: torch.Tensor,
        a_stack: torch.Tensor,
        b_stack: torch.Tensor,
        base_output: torch.Tensor,
    ) -> torch.Tensor:
        """Shrink then expand; the delta is added into base_output in place.

        x [S, in]; a_stack [K, max_rank, in]; b_stack [K, out, max_rank];
        base_output [S, out] (may be a row-strided slice). Returns base_output.
        """
        mid = self.run_lora_a_sgemm(x, a_stack)
        return self.run_lora_b_sgemm(mid, b_stack, base_output=base_output)
