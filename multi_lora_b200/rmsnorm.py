"""Fused RMSNorm (drop-in for ``multi_lora/kernels/rmsnorm.py:48-115``)."""

from __future__ import annotations

import torch

from multi_lora_b200 import _native


def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``cast(x_f32 * rsqrt(mean(x_f32^2) + eps) * w_f32)``; new contiguous output of x's shape.

    Non-contiguous x whose first-dim blocks are dense (e.g. q/k column slices
    of a fused qkv output) is read in place with a two-level row stride.
    """
    if not x.is_cuda:
        raise RuntimeError("mlora: rmsnorm_fwd needs a CUDA tensor (no CPU path)")
    return _native.ops().rmsnorm(x, weight, float(eps))


def rmsnorm_out(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    """Same as :func:`rmsnorm_fwd` into a caller-owned contiguous ``out`` (no allocation)."""
    if not x.is_cuda:
        raise RuntimeError("mlora: rmsnorm_out needs a CUDA tensor (no CPU path)")
    return _native.ops().rmsnorm_out(x, weight, float(eps), out)


def fused_add_rmsnorm(residual: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, eps: float,
                      out: torch.Tensor | None = None):
    """``residual = residual + x`` (in place, rounded to the dtype), then RMSNorm of it.

    The residual add in front of a decoder layer's norm fused with the norm
    (the reference's planned T22, OPTIMIZATION_TODO.md:125-142). Returns
    ``(out, residual)``; ``out`` is allocated unless given. Bit-identical to
    ``residual += x; rmsnorm_fwd(residual, weight, eps)``.
    """
    if not (x.is_cuda and residual.is_cuda):
        raise RuntimeError("mlora: fused_add_rmsnorm needs CUDA tensors (no CPU path)")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    _native.ops().fused_add_rmsnorm(x, residual, weight, float(eps), out)
    return out, residual


def fuse_rmsnorm(model) -> int:
    """Route every ``*RMSNorm`` module with ``variance_epsilon`` through the fused kernel.

    Only the instance's ``forward`` is replaced (module tree, parameters,
    state_dict untouched). Returns the number of modules patched.
    """
    n = 0
    for module in model.modules():
        if not type(module).__name__.endswith("RMSNorm"):
            continue
        eps = getattr(module, "variance_epsilon", None)
        weight = getattr(module, "weight", None)
        if eps is None or weight is None:
            continue

        def _forward(hidden_states, _w=weight, _eps=float(eps)):
            return rmsnorm_fwd(hidden_states, _w, _eps)

        module.forward = _forward
        n += 1
    return n
