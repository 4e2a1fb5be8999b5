"""PEFT adapter directories on disk <-> :class:`AdapterWeights`, without the ``peft`` package.

The reference builds ``AdapterWeights`` from a loaded ``PeftModel``
(``extract_adapter_weights``, multi_lora/weights.py:36-68): for every LoRA
layer it takes A ``[rank, in]`` and B ``[out, rank]``, keys the pair by the
layer's module name with the PEFT prefixes stripped (``normalize_module_key``,
weights.py:28-33), requires one rank across the adapter and sets
``scaling = lora_alpha / rank``. Its examples read the same information from
the files a PEFT ``save_pretrained`` writes (examples/make_rank_variants.py:
51-55): ``adapter_config.json`` (``r``, ``lora_alpha``, ``use_rslora``,
``rank_pattern``, ``alpha_pattern``) and ``adapter_model.safetensors``, whose
tensors are named ``<module>.lora_A.weight`` / ``<module>.lora_B.weight``.

This module reads those two files directly, so adapters can be registered
where ``peft`` is not installed. Only nn.Linear LoRA layers are supported
(``fan_in_fan_out`` false): A is ``[r, in]`` and B ``[out, r]`` as stored.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Dict, Optional, Tuple, Union

import torch

from multi_lora_b200.weights import AdapterWeights, normalize_module_key

CONFIG_NAME = "adapter_config.json"
SAFETENSORS_NAME = "adapter_model.safetensors"
BIN_NAME = "adapter_model.bin"
_A_SUFFIX = ".lora_A.weight"
_B_SUFFIX = ".lora_B.weight"


def _module_key(tensor_name: str, suffix: str) -> str:
    return normalize_module_key(tensor_name[: -len(suffix)])


def _read_tensors(directory: Path) -> Dict[str, torch.Tensor]:
    st = directory / SAFETENSORS_NAME
    if st.exists():
        from safetensors.torch import load_file

        return load_file(str(st))
    bin_path = directory / BIN_NAME
    if bin_path.exists():
        return torch.load(str(bin_path), map_location="cpu", weights_only=True)
    raise FileNotFoundError(f"no {SAFETENSORS_NAME} or {BIN_NAME} in {directory}")


def load_adapter_dir(path: Union[str, Path], *, dtype: Optional[torch.dtype] = None) -> AdapterWeights:
    """Read a PEFT adapter directory into host :class:`AdapterWeights`.

    Scaling is ``lora_alpha / r`` (``lora_alpha / sqrt(r)`` with
    ``use_rslora``), as PEFT applies it. Like the reference, every module must
    have the adapter's one rank: a ``rank_pattern`` or ``alpha_pattern`` that
    gives a module another rank or alpha raises ``ValueError``, as do an A
    without its B and tensors whose shapes disagree with the rank.
    """
    d = Path(path)
    cfg_path = d / CONFIG_NAME
    if not cfg_path.exists():
        raise FileNotFoundError(f"no {CONFIG_NAME} in {d}")
    cfg = json.loads(cfg_path.read_text())
    if cfg.get("fan_in_fan_out", False):
        raise ValueError("fan_in_fan_out adapters (Conv1D layers) are not supported")
    rank = int(cfg["r"])
    alpha = float(cfg.get("lora_alpha", rank))
    tensors = _read_tensors(d)

    modules: Dict[str, Tuple[torch.Tensor, torch.Tensor]] = {}
    for name, a in tensors.items():
        if not name.endswith(_A_SUFFIX):
            continue
        b_name = name[: -len(_A_SUFFIX)] + _B_SUFFIX
        if b_name not in tensors:
            raise ValueError(f"{name} has no matching {b_name}")
        b = tensors[b_name]
        key = _module_key(name, _A_SUFFIX)
        if a.dim() != 2 or b.dim() != 2 or a.shape[0] != b.shape[1]:
            raise ValueError(f"{key}: A {tuple(a.shape)} and B {tuple(b.shape)} are not [r, in] / [out, r]")
        if a.shape[0] != rank:
            raise ValueError(f"rank mismatch in {d.name}: module {key} has rank {a.shape[0]}, adapter r = {rank}")
        if dtype is not None:
            a, b = a.to(dtype), b.to(dtype)
        modules[key] = (a.contiguous(), b.contiguous())
    orphans = [n for n in tensors if n.endswith(_B_SUFFIX) and n[: -len(_B_SUFFIX)] + _A_SUFFIX not in tensors]
    if orphans:
        raise ValueError(f"{orphans[0]} has no matching lora_A")
    if not modules:
        raise ValueError(f"no LoRA weights found in {d}")
    for pattern, what in ((cfg.get("rank_pattern") or {}, "rank"), (cfg.get("alpha_pattern") or {}, "alpha")):
        for pat, value in pattern.items():
            if (what == "rank" and int(value) != rank) or (what == "alpha" and float(value) != alpha):
                raise ValueError(f"{what}_pattern gives {pat!r} {what} {value}; one {what} per adapter is supported")
    scaling = alpha / math.sqrt(rank) if cfg.get("use_rslora", False) else alpha / rank
    return AdapterWeights(rank=rank, scaling=scaling, modules=modules)


def save_adapter_dir(weights: AdapterWeights, path: Union[str, Path], *, lora_alpha: Optional[float] = None,
                     prefix: str = "base_model.model.") -> Path:
    """Write ``weights`` as a PEFT-format directory (config + safetensors).

    ``lora_alpha`` defaults to ``scaling * rank`` (no rslora), so that
    :func:`load_adapter_dir` returns the same scaling. Module keys get
    ``prefix`` in front, as PEFT names layers inside its wrapper model.
    """
    from safetensors.torch import save_file

    d = Path(path)
    d.mkdir(parents=True, exist_ok=True)
    if weights.flattened:
        raise RuntimeError("adapter module tensors were released after packing; nothing to save")
    alpha = weights.scaling * weights.rank if lora_alpha is None else float(lora_alpha)
    state = {}
    for key, (a, b) in weights.modules.items():
        state[f"{prefix}{key}{_A_SUFFIX}"] = a.detach().contiguous().cpu()
        state[f"{prefix}{key}{_B_SUFFIX}"] = b.detach().contiguous().cpu()
    save_file(state, str(d / SAFETENSORS_NAME))
    targets = sorted({k.rsplit(".", 1)[-1] for k in weights.modules})
    cfg = {"peft_type": "LORA", "r": weights.rank, "lora_alpha": alpha, "target_modules": targets,
           "use_rslora": False, "fan_in_fan_out": False, "bias": "none", "rank_pattern": {}, "alpha_pattern": {}}
    (d / CONFIG_NAME).write_text(json.dumps(cfg, indent=2))
    return d
