"""LoRA-wrapped linear layers (drop-in for ``multi_lora/layers.py``).

``LinearWithLoRA.forward`` = base projection + the backend's LoRA delta,
added in place into the base output (layers.py:42-88 of the reference).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from multi_lora_b200.backend.base import LoRABackend

# process-wide switch: when False, LinearWithLoRA returns the base output only
LORA_ENABLED = True


def set_lora_enabled(enabled: bool) -> None:
    """Turn the LoRA delta on or off for every wrapper (layers.py:17-20)."""
    global LORA_ENABLED
    LORA_ENABLED = bool(enabled)


def lora_delta(
    x: torch.Tensor,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scaling: float,
    *,
    rank: int,
) -> torch.Tensor:
    """Plain row-wise delta ``scaling * x @ A[:rank]^T @ B[:, :rank]^T`` (layers.py:23-39).

    Test reference only; runs in x's dtype on x's device.
    """
    a = lora_a[:rank]
    b = lora_b[:, :rank]
    rows = x.reshape(-1, x.shape[-1])
    out = (rows @ a.T @ b.T) * scaling
    return out.reshape(*x.shape[:-1], b.shape[0])


class LinearWithLoRA(nn.Module):
    """Replaces a PEFT LoraLayer: base GEMM plus the backend's per-slot delta."""

    def __init__(self, base_layer: nn.Module) -> None:
        super().__init__()
        self.base_layer = base_layer
        self.backend: Optional[LoRABackend] = None
        self.A_buffer: Optional[torch.Tensor] = None   # [K, max_rank, in]
        self.B_buffer: Optional[torch.Tensor] = None   # [K, out, max_rank]
        self.qkv_group: Optional["QKVProjGroup"] = None
        self.qkv_slice: Optional[tuple] = None

    def set_lora_info(self, backend: LoRABackend, a_buffer: torch.Tensor, b_buffer: torch.Tensor) -> None:
        """Attach the backend and the slot-major weight stacks for this step."""
        self.backend = backend
        self.A_buffer = a_buffer
        self.B_buffer = b_buffer

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.qkv_group is not None:
            return self.qkv_group.forward(self, x)
        return self.add_delta(x, self.base_layer(x))

    def add_delta(self, x: torch.Tensor, y_base: torch.Tensor) -> torch.Tensor:
        """Add the LoRA delta into an already computed base output (in place).

        y_base may be a column slice of a wider fused output; its row stride is
        passed to the expand kernel instead of copying (layers.py:82-83).
        """
        if not LORA_ENABLED or self.backend is None or self.A_buffer is None or self.B_buffer is None:
            return y_base
        x_rows = x.reshape(-1, x.shape[-1])
        y_rows = y_base.reshape(-1, y_base.shape[-1])
        y_rows = self.backend.apply_lora(x_rows, self.A_buffer, self.B_buffer, y_rows)
        return y_rows.reshape(y_base.shape)


class QKVProjGroup:
    """One concatenated base GEMM for the q/k/v projections of an attention block.

    At decode (one token per row) the first of q/k/v computes the whole qkv
    output; the other two reuse column slices of it (layers.py:91-125). The
    three base weights become slices of one shared storage.
    """

    def __init__(self, wrappers: list) -> None:
        if any(w.base_layer.bias is not None for w in wrappers):
            raise RuntimeError("QKV fusion requires bias=None")
        dims = [int(w.base_layer.weight.shape[0]) for w in wrappers]
        self.wrappers = list(wrappers)
        self.weight = torch.cat([w.base_layer.weight for w in wrappers], dim=0)
        lo = 0
        for w, d in zip(wrappers, dims):
            w.base_layer.weight = nn.Parameter(self.weight[lo: lo + d], requires_grad=False)
            w.qkv_slice = (lo, lo + d)
            w.qkv_group = self
            lo += d
        self._cached_x: Optional[torch.Tensor] = None
        self._cached_out: Optional[torch.Tensor] = None

    def forward(self, wrapper: LinearWithLoRA, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-2] != 1:  # prefill: separate GEMMs
            return wrapper.add_delta(x, wrapper.base_layer(x))
        if self._cached_x is not x:
            self._cached_x = x
            self._cached_out = F.linear(x, self.weight)
            self._deltas_added = self._add_group_delta(x)
        lo, hi = wrapper.qkv_slice
        out = self._cached_out[..., lo:hi]
        return out if self._deltas_added else wrapper.add_delta(x, out)

    def _add_group_delta(self, x: torch.Tensor) -> bool:
        """Add all three LoRA deltas into the fused output with one grouped call.

        Same numbers as three add_delta calls; used when every wrapper is bound
        to one backend that offers ``apply_lora_group``. Returns whether it ran.
        """
        ws = self.wrappers
        be = ws[0].backend
        if not LORA_ENABLED or be is None or not hasattr(be, "apply_lora_group"):
            return False
        if any(w.backend is not be or w.A_buffer is None or w.B_buffer is None for w in ws):
            return False
        x_rows = x.reshape(-1, x.shape[-1])
        y_rows = self._cached_out.reshape(-1, self._cached_out.shape[-1])
        be.apply_lora_group(x_rows, [w.A_buffer for w in ws], [w.B_buffer for w in ws],
                            [y_rows[:, w.qkv_slice[0]:w.qkv_slice[1]] for w in ws])
        return True


def fuse_qkv_projections(wrappers: dict) -> int:
    """Group the q/k/v wrappers of each attention block; returns the group count."""
    blocks: dict = {}
    for key, w in wrappers.items():
        for suffix in ("q_proj", "k_proj", "v_proj"):
            if key.endswith("." + suffix):
                blocks.setdefault(key[: -len(suffix)], {})[suffix] = w
                break
    n = 0
    for parts in blocks.values():
        if len(parts) == 3:
            QKVProjGroup([parts["q_proj"], parts["k_proj"], parts["v_proj"]])
            n += 1
    return n
