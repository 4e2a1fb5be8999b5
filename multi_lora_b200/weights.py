"""Per-adapter host weights (drop-in for the dataclass of ``multi_lora/weights.py:17-33``).

Extraction from a PEFT model (weights.py:36-68) is not part of this package:
``AdapterWeights`` is filled by the caller (e.g. from safetensors).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

import torch

# module key -> (A [rank, in], B [out, rank])
ModuleWeights = Dict[str, Tuple[torch.Tensor, torch.Tensor]]


@dataclass
class AdapterWeights:
    """All LoRA weights of one adapter, on the host."""

    rank: int
    scaling: float
    modules: ModuleWeights
    # set once the modules were packed into a pinned bank and released
    flattened: bool = False


def normalize_module_key(module_name: str) -> str:
    """Strip the PEFT prefixes so module names match the pool's keys."""
    for prefix in ("base_model.model.", "model."):
        if module_name.startswith(prefix):
            return module_name[len(prefix):]
    return module_name
