"""Per-step orchestration of the LoRA hot path.

Covers the parts of ``multi_lora/manager.py`` that sit on the hot path:
``prepare_lora_batch`` (:172-187), ``build_kernel_input_metadata`` (:189-212),
``_setup_forward_batch`` (:214-233) and ``forward_with_lora`` (:237-279).
Adapters are registered as :class:`AdapterWeights`, or read from PEFT adapter
directories with :meth:`MultiLoRAManager.load_adapter` (no ``peft`` install
needed); the target ``nn.Linear`` modules are wrapped with
:func:`wrap_linear_modules`.
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Dict, Iterable, List, Optional

import torch
import torch.nn as nn

from multi_lora_b200.admission import Admission, AdmissionPolicy
from multi_lora_b200.backend.base import LoRABackend
from multi_lora_b200.backend.registry import get_lora_backend
from multi_lora_b200.batch_info import (
    BatchLoRAInfo,
    KernelInputMetaData,
    empty_kernel_input_metadata,
    group_rows,
    write_kernel_input_metadata,
)
from multi_lora_b200.layers import LinearWithLoRA
from multi_lora_b200.pool import LoRAMemoryPool, LoraName
from multi_lora_b200.weights import AdapterWeights


def validate_lora_batch(lora_names: List[LoraName], *, max_loras_per_batch: int) -> bool:
    """Distinct adapters (``None`` counts as one) fit the slots (batching.py:33-39)."""
    return len(set(lora_names)) <= max_loras_per_batch


def wrap_linear_modules(model: nn.Module, keys: Iterable[str]) -> Dict[str, LinearWithLoRA]:
    """Replace each ``nn.Linear`` named in ``keys`` by a :class:`LinearWithLoRA` around it."""
    wanted = set(keys)
    wrappers: Dict[str, LinearWithLoRA] = {}
    for name, module in list(model.named_modules()):
        if name not in wanted or not isinstance(module, nn.Linear):
            continue
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        wrapper = LinearWithLoRA(module)
        setattr(parent, child, wrapper)
        wrappers[name] = wrapper
    missing = wanted - set(wrappers)
    if missing:
        raise KeyError(f"no nn.Linear named {sorted(missing)}")
    return wrappers


class MultiLoRAManager:
    """Slot pool + CUDA backend + wrapped linears, driven once per forward step."""

    def __init__(
        self,
        lora_wrappers: Dict[str, LinearWithLoRA],
        *,
        device: torch.device,
        dtype: torch.dtype,
        max_loras_per_batch: int = 4,
        max_lora_rank: int = 64,
        eviction_policy: str = "lru",
        lora_backend: str = "cuda",
        model: Optional[nn.Module] = None,
    ) -> None:
        self.model = model  # the model whose linears the wrappers sit in (optional)
        self.lora_wrappers = lora_wrappers
        self.max_loras_per_batch = max_loras_per_batch
        self.pool = LoRAMemoryPool(max_loras_per_batch, max_lora_rank, device, dtype, eviction_policy)
        self._weight_store: Dict[LoraName, AdapterWeights] = {}
        self._lora_backend: LoRABackend = get_lora_backend(lora_backend)
        self._resident_meta: KernelInputMetaData = empty_kernel_input_metadata(
            device=self.pool.device, dtype=self.pool.dtype)

    @classmethod
    def from_model(cls, model: nn.Module, *, target_suffixes: Iterable[str], device: torch.device,
                   dtype: torch.dtype, **kwargs) -> "MultiLoRAManager":
        """Wrap every ``nn.Linear`` of ``model`` whose name ends with one of
        ``target_suffixes`` (the reference's ``lora_target_suffixes``,
        manager.py:94-125) and build a manager that owns ``model``. Keys are the
        module names normalised like PEFT's (``normalize_module_key``)."""
        from multi_lora_b200.weights import normalize_module_key

        suffixes = tuple(target_suffixes)
        names = [n for n, m in model.named_modules() if isinstance(m, nn.Linear) and n.endswith(suffixes)]
        wrappers = wrap_linear_modules(model, names)
        keyed = {normalize_module_key(n): w for n, w in wrappers.items()}
        return cls(keyed, device=device, dtype=dtype, model=model, **kwargs)

    @property
    def inference_model(self) -> nn.Module:
        """The model a decode step runs (graph_decode.DecodeStep.run)."""
        if self.model is None:
            raise RuntimeError("this manager was built without a model")
        return self.model

    def register_adapter(self, name: str, weights: AdapterWeights) -> None:
        if not name:
            raise ValueError("lora_name cannot be empty")
        if name in self._weight_store:
            raise ValueError(f"LoRA name already registered: {name}")
        self._weight_store[name] = weights
        self.pool.ensure_buffers(weights)

    def load_adapter(self, name: str, path, *, dtype: Optional[torch.dtype] = None) -> AdapterWeights:
        """Register the PEFT adapter saved in directory ``path`` (``adapter_config.json`` +
        ``adapter_model.safetensors``) under ``name``; no ``peft`` install needed
        (:func:`multi_lora_b200.peft_io.load_adapter_dir`)."""
        from multi_lora_b200.peft_io import load_adapter_dir

        weights = load_adapter_dir(path, dtype=dtype)
        self.register_adapter(name, weights)
        return weights

    def prepare_lora_batch(self, lora_names: List[LoraName]) -> BatchLoRAInfo:
        if not validate_lora_batch(lora_names, max_loras_per_batch=self.max_loras_per_batch):
            raise ValueError(f"invalid lora batch: distinct={len(set(lora_names))} max={self.max_loras_per_batch}")
        self.pool.prepare_lora_batch(set(lora_names), weight_store=self._weight_store)
        return self.pool.build_batch_info(list(lora_names))

    def admit_tokens(self, lora_names: List[LoraName], *, n_deferred: int = 0, max_tokens: Optional[int] = None,
                     resident_first: bool = True) -> Admission:
        """Choose which queued tokens run this step so that they name at most
        ``max_loras_per_batch`` adapters (the reference raises instead,
        manager.py:172-180). ``lora_names[i]`` is token i's adapter; the first
        ``n_deferred`` are tokens deferred by earlier steps (admitted first),
        then tokens whose adapter is resident in the pool, then the rest
        (rule in :mod:`multi_lora_b200.admission`)."""
        policy = AdmissionPolicy(self.max_loras_per_batch, resident_first=resident_first)
        return policy.admit(lora_names, resident=self.pool.name_to_slot.keys(), n_deferred=n_deferred,
                            max_tokens=max_tokens)

    def prefetch_lora_batch(self, lora_names: Iterable[LoraName]) -> None:
        """Start the loads of a coming step's adapters now, before its metadata is built.

        The loads run on the pool's copy stream; a load into a slot that
        already-enqueued work reads waits only for that work (per-slot events),
        so the H2D overlaps the step in flight. The compute stream waits for the
        loads before anything enqueued after this call. The coming step's
        ``build_kernel_input_metadata`` then finds the adapters resident."""
        names = set(lora_names)
        if not validate_lora_batch(list(names), max_loras_per_batch=self.max_loras_per_batch):
            raise ValueError(f"invalid lora batch: distinct={len(names)} max={self.max_loras_per_batch}")
        self.pool.prepare_lora_batch(names, weight_store=self._weight_store)

    @torch.inference_mode()
    def build_kernel_input_metadata(self, lora_names: List[LoraName], *, seq_lens: List[int]) -> KernelInputMetaData:
        """Group adjacent rows, make their adapters resident, write the resident tables."""
        names, lens = group_rows(lora_names, seq_lens)
        info = self.prepare_lora_batch(names)
        self._resident_meta = write_kernel_input_metadata(
            self._resident_meta, info, device=self.pool.device, dtype=self.pool.dtype, seq_lens=lens)
        return self._resident_meta

    def _setup_forward_batch(self, lora_names: List[LoraName], *, seq_lens: List[int]) -> None:
        meta = self.build_kernel_input_metadata(lora_names, seq_lens=seq_lens)
        self._lora_backend.set_kernel_input_metadata(meta)
        for key, wrapper in self.lora_wrappers.items():
            a, b = self.pool.get_module_buffers(key)
            wrapper.set_lora_info(self._lora_backend, a, b)

    @torch.inference_mode()
    def forward_with_lora(self, model: Optional[nn.Module] = None, *, lora_names: List[LoraName],
                          seq_lens: List[int], x: Optional[torch.Tensor] = None, **kwargs):
        """Prepare the step, then run ``model(x, **kwargs)`` (or ``model(**kwargs)``);
        ``model`` defaults to the manager's own."""
        model = self.inference_model if model is None else model
        self._setup_forward_batch(lora_names, seq_lens=seq_lens)
        with nullcontext():
            if x is not None:
                return model(x, **kwargs)
            return model(**kwargs)
