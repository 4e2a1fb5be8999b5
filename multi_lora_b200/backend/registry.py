"""Backend factory (drop-in for ``multi_lora/backend/registry.py:10-17``).

There is a single implementation. "triton" is accepted as an alias so code
written against the reference keeps working; it selects the CUDA kernels.
"""

from __future__ import annotations

from multi_lora_b200.backend.base import LoRABackend
from multi_lora_b200.backend.cuda_backend import CudaLoRABackend

_NAMES = ("cuda", "b200", "triton")


def get_lora_backend(name: str = "cuda") -> LoRABackend:
    key = name.lower().strip()
    if key in _NAMES:
        return CudaLoRABackend()
    if key == "torch":
        raise ValueError(
            "the per-segment torch backend is the reference's CPU path; this package "
            "ships only the CUDA backend (get_lora_backend('cuda'))")
    raise ValueError(f"unknown lora backend: {name}; try cuda")
