"""The one backend: hand-written sm_100a kernels behind ``torch.ops.mlora``.

Takes the place of ``TritonLoRABackend`` (multi_lora/backend/triton_backend.py:19-78)
with the same methods. There is no CPU or Torch fallback: a non-CUDA input or
a missing extension raises.

The kernels behind these methods allocate nothing; this layer allocates only
in two cases the normal path never meets: an output whose column stride is
not 1 goes through a contiguous temporary (copied back), and routing tables
that are not int32 are converted per call (``write_kernel_input_metadata``
writes int32).
"""

from __future__ import annotations

from typing import Optional

import torch

from multi_lora_b200 import _native
from multi_lora_b200.backend.base import LoRABackend
from multi_lora_b200.batch_info import KernelInputMetaData


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 and t.is_contiguous() else t.to(torch.int32).contiguous()


class CudaLoRABackend(LoRABackend):
    """Slot-grouped segment shrink/expand on B200 (one launch each per call)."""

    name = "cuda"

    def __init__(self, stack_num: int = 1) -> None:
        super().__init__()
        self.stack_num = stack_num
        self._ops = _native.ops()
        self._status: Optional[torch.Tensor] = None
        self._gmid = torch.empty((0, 0))

    # -- routing-error status word ------------------------------------------
    def status_word(self, device: torch.device) -> torch.Tensor:
        """Device int32 word the kernels OR error bits into (see include/mlora_b200.h)."""
        if self._status is None or self._status.device != device:
            self._status = torch.zeros(1, dtype=torch.int32, device=device)
        return self._status

    def check_routing(self) -> None:
        """Raise if any launch so far met out-of-range routing (synchronises)."""
        if self._status is None:
            return
        bits = int(self._status.item())
        if bits:
            self._status.zero_()
            names = []
            if bits & 1:
                names.append("weight_indices outside [0, num_slots)")
            if bits & 2:
                names.append("lora_ranks outside [0, max_rank]")
            if bits & 4:
                names.append("seg_indptr decreasing or past the row count")
            if bits & 8:
                names.append("scatter descriptor out of range")
            if bits & 16:
                names.append("an asynchronous copy did not complete in time")
            raise RuntimeError("mlora: invalid routing metadata: " + "; ".join(names))

    def group_mid_buffer(self, rows: int, max_rank: int, like: torch.Tensor) -> torch.Tensor:
        """Resident (rows, 4 * max_rank) intermediate for ``apply_lora_group``:
        projection m's shrink output sits in columns [m*max_rank, (m+1)*max_rank).
        Reused while it fits (CUDA-graph safe once sized)."""
        m = self._gmid
        if (m.shape[0] < rows or m.shape[1] != 4 * max_rank or m.device != like.device
                or m.dtype != like.dtype):
            self._gmid = torch.empty((rows, 4 * max_rank), dtype=like.dtype, device=like.device)
        return self._gmid[:rows]

    def _meta(self) -> KernelInputMetaData:
        meta = self.kernel_input_metadata
        if meta is None:
            raise RuntimeError("kernel_input_metadata not set; call set_kernel_input_metadata first")
        return meta

    def _check_x(self, x: torch.Tensor, what: str) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError(f"mlora: {what} must be a CUDA tensor (no CPU path)")
        if x.dim() != 2:
            raise ValueError(f"CudaLoRABackend expects {what} [S, n]")
        return x if x.stride(1) == 1 else x.contiguous()

    def run_lora_a_sgemm(self, x: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        meta = self._meta()
        x = self._check_x(x, "x")
        out = self.mid_buffer(x.shape[0], weights.shape[-2], x)
        return self._ops.sgemm_lora_a(
            x, weights.contiguous(), _i32(meta.seg_lens), _i32(meta.seg_indptr), _i32(meta.weight_indices),
            _i32(meta.lora_ranks), int(meta.bs), int(meta.max_len), out, self.stack_num,
            self.status_word(x.device))

    def apply_lora(
        self,
        x: torch.Tensor,
        a_stack: torch.Tensor,
        b_stack: torch.Tensor,
        base_output: torch.Tensor,
    ) -> torch.Tensor:
        """Shrink + expand into base_output in place; one fused launch for short segments.

        ``mid_buffer`` still receives the shrink output, as with two launches.
        """
        meta = self._meta()
        x = self._check_x(x, "x")
        mid = self.mid_buffer(x.shape[0], a_stack.shape[-2], x)
        out = base_output
        target = out if (out.dim() == 2 and out.stride(1) == 1) else out.contiguous()
        self._ops.apply_lora(
            x, a_stack.contiguous(), b_stack.contiguous(), _i32(meta.seg_lens), _i32(meta.seg_indptr),
            _i32(meta.weight_indices), _i32(meta.lora_ranks), meta.scalings, int(meta.bs), int(meta.max_len),
            mid, target, self.status_word(x.device))
        if target is not out:
            out.copy_(target)
        return out

    def apply_lora_group(self, x: torch.Tensor, a_stacks, b_stacks, base_outputs) -> list:
        """apply_lora for up to 4 projections that share ``x`` and the routing
        (q/k/v, gate/up): one launch for short segments. Each base output is
        updated in place and returned."""
        meta = self._meta()
        x = self._check_x(x, "x")
        outs = list(base_outputs)
        targets = [o if (o.dim() == 2 and o.stride(1) == 1) else o.contiguous() for o in outs]
        mid = self.group_mid_buffer(x.shape[0], a_stacks[0].shape[-2], x)
        self._ops.apply_lora_group(
            x, [a.contiguous() for a in a_stacks], [b.contiguous() for b in b_stacks], _i32(meta.seg_lens),
            _i32(meta.seg_indptr), _i32(meta.weight_indices), _i32(meta.lora_ranks), meta.scalings, int(meta.bs),
            int(meta.max_len), targets, mid, self.status_word(x.device))
        for o, t in zip(outs, targets):
            if t is not o:
                o.copy_(t)
        return outs

    def shrink_partial(self, x: torch.Tensor, a_shard: torch.Tensor) -> torch.Tensor:
        """fp32 shrink partials of this rank's input slice into the resident
        partial buffer (zeroed first, so the all-reduce sums only real terms)."""
        meta = self._meta()
        x = self._check_x(x, "x")
        part = self.partial_buffer(x.shape[0], a_shard.shape[-2], x)
        part.zero_()
        return self._ops.sgemm_lora_a(
            x, a_shard.contiguous(), _i32(meta.seg_lens), _i32(meta.seg_indptr), _i32(meta.weight_indices),
            _i32(meta.lora_ranks), int(meta.bs), int(meta.max_len), part, self.stack_num,
            self.status_word(x.device))

    def expand_partial(self, partial: torch.Tensor, b_shard: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Expand from the all-reduced fp32 partials (the kernel rounds them to
        y's dtype before the product) into ``y`` (a column slice) in place."""
        if partial.dtype != torch.float32:
            raise TypeError("mlora: expand_partial expects the fp32 partial buffer")
        return self.run_lora_b_sgemm(partial, b_shard, base_output=y)

    def run_lora_b_sgemm(
        self,
        x: torch.Tensor,
        weights: torch.Tensor,
        base_output: Optional[torch.Tensor] = None,
    ) -> torch.Tensor:
        meta = self._meta()
        x = self._check_x(x, "mid")
        if base_output is None:
            out = torch.zeros((x.shape[0], weights.shape[-2]), dtype=weights.dtype, device=x.device)
        else:
            out = base_output
        target = out if (out.dim() == 2 and out.stride(1) == 1) else out.contiguous()
        self._ops.sgemm_lora_b(
            x, weights.contiguous(), _i32(meta.seg_lens), _i32(meta.seg_indptr), _i32(meta.weight_indices),
            _i32(meta.lora_ranks), meta.scalings, int(meta.bs), int(meta.max_len), target,
            self.status_word(x.device))
        if target is not out:
            out.copy_(target)
        return out
