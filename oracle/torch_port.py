"""CPU port of the reference's pure-PyTorch LoRA path — TEST/BASELINE INFRASTRUCTURE ONLY.

A restatement, in torch on the host, of ``TorchLoRABackend``
(multi_lora/backend/torch_backend.py:12-90 of Rick0037/multi_lora): a Python
loop over segments that reads each segment's bounds, slot and rank with
``.item()`` and does ``x_seg @ A[slot, :r].T`` then
``(mid_seg @ B[slot, :, :r].T) * scaling`` in the activation dtype. RMSNorm is
the eager fp32 formula of kernels/rmsnorm.py:38-45 in torch ops (on the CPU
the reference model runs the transformers RMSNorm, whose arithmetic this is).

bench.py times it on the host cores as the reference arm / CPU baseline; the
CUDA product never calls it.
"""

from __future__ import annotations

import torch


class TorchPortBackend:
    """Per-segment CPU LoRA, same call shape as the reference backend."""

    def __init__(self, seg_indptr: torch.Tensor, weight_indices: torch.Tensor, lora_ranks: torch.Tensor,
                 scalings: torch.Tensor, bs: int):
        self.seg_indptr, self.weight_indices = seg_indptr, weight_indices
        self.lora_ranks, self.scalings, self.bs = lora_ranks, scalings, bs

    def run_lora_a_sgemm(self, x: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """torch_backend.py:17-49."""
        y = torch.zeros(x.shape[0], weights.shape[1], dtype=x.dtype)
        for seg in range(self.bs):
            start = int(self.seg_indptr[seg].item())
            end = int(self.seg_indptr[seg + 1].item())
            if start >= end:
                continue
            slot = int(self.weight_indices[seg].item())
            r = int(self.lora_ranks[slot].item())
            if r == 0:
                continue
            y[start:end, :r] = x[start:end] @ weights[slot, :r, :].to(x.dtype).T
        return y

    def run_lora_b_sgemm(self, x: torch.Tensor, weights: torch.Tensor, base_output: torch.Tensor) -> torch.Tensor:
        """torch_backend.py:51-90 with base_output given."""
        y = base_output
        for seg in range(self.bs):
            start = int(self.seg_indptr[seg].item())
            end = int(self.seg_indptr[seg + 1].item())
            if start >= end:
                continue
            slot = int(self.weight_indices[seg].item())
            r = int(self.lora_ranks[slot].item())
            if r == 0:
                continue
            b = weights[slot, :, :r].to(x.dtype)
            scale = self.scalings[slot].to(x.dtype)
            y[start:end] = y[start:end] + (x[start:end, :r] @ b.T) * scale
        return y

    def apply_lora(self, x, a_stack, b_stack, base_output):
        return self.run_lora_b_sgemm(self.run_lora_a_sgemm(x, a_stack), b_stack, base_output)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    return ((h * torch.rsqrt(var + eps)) * w.to(torch.float32)).to(x.dtype)
