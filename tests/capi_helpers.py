"""ctypes calls into include/mlora_b200.h with torch tensors as device memory (tests only)."""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np
import torch

from multi_lora_b200 import _native

DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


@dataclass
class DevMeta:
    """Device routing tables plus the ctypes struct pointing at them."""

    seg_lens: torch.Tensor
    seg_indptr: torch.Tensor
    weight_indices: torch.Tensor
    lora_ranks: torch.Tensor
    scalings: torch.Tensor
    bs: int
    max_len: int

    def struct(self) -> _native.MetadataT:
        m = _native.MetadataT()
        m.bs, m.max_len = self.bs, self.max_len
        m.num_slots = self.lora_ranks.numel()
        m.scalings_dtype = DT[self.scalings.dtype]
        m.seg_lens = self.seg_lens.data_ptr()
        m.seg_indptr = self.seg_indptr.data_ptr()
        m.weight_indices = self.weight_indices.data_ptr()
        m.lora_ranks = self.lora_ranks.data_ptr()
        m.scalings = self.scalings.data_ptr()
        return m


def make_meta(lens: Sequence[int], widx: Sequence[int], ranks: Sequence[int], scalings: Sequence[float],
              device, scal_dtype=torch.float32, indptr: Optional[List[int]] = None) -> DevMeta:
    if indptr is None:
        indptr = [0]
        for n in lens:
            indptr.append(indptr[-1] + int(n))
    i32 = dict(dtype=torch.int32, device=device)
    return DevMeta(torch.tensor(list(lens) or [0], **i32), torch.tensor(indptr, **i32),
                   torch.tensor(list(widx) or [0], **i32), torch.tensor(list(ranks), **i32),
                   torch.tensor(list(scalings), dtype=scal_dtype, device=device), len(lens),
                   max(lens) if len(lens) else 0)


def meta_from_npz(z: dict, device, prefix: str = "", scal_dtype=torch.float32) -> DevMeta:
    i32 = dict(dtype=torch.int32, device=device)
    return DevMeta(torch.tensor(z[prefix + "seg_lens"], **i32), torch.tensor(z[prefix + "seg_indptr"], **i32),
                   torch.tensor(z[prefix + "weight_indices"], **i32), torch.tensor(z[prefix + "lora_ranks"], **i32),
                   torch.tensor(z[prefix + "scalings"], dtype=scal_dtype, device=device),
                   int(z[prefix + "bs"]), int(z[prefix + "max_len"]))


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def shrink(x: torch.Tensor, A: torch.Tensor, meta: DevMeta, out: torch.Tensor, stack_num: int = 1,
           status: Optional[torch.Tensor] = None) -> int:
    lib = _native.capi()
    m = meta.struct()
    return lib.mlora_sgemm_lora_a_fwd(
        x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), A.data_ptr(), A.shape[1], ctypes.byref(m),
        out.data_ptr(), out.stride(0), DT[out.dtype], DT[x.dtype], stack_num,
        status.data_ptr() if status is not None else None, _stream())


def expand(mid: torch.Tensor, B: torch.Tensor, meta: DevMeta, y: torch.Tensor,
           status: Optional[torch.Tensor] = None) -> int:
    lib = _native.capi()
    m = meta.struct()
    return lib.mlora_sgemm_lora_b_fwd(
        mid.data_ptr(), mid.shape[0], mid.stride(0), DT[mid.dtype], B.data_ptr(), B.shape[1], B.shape[2],
        ctypes.byref(m), y.data_ptr(), y.stride(0), DT[y.dtype],
        status.data_ptr() if status is not None else None, _stream())


def apply_lora(x, A, B, meta: DevMeta, mid, y, status=None) -> int:
    lib = _native.capi()
    m = meta.struct()
    return lib.mlora_apply_lora(
        x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), A.data_ptr(), B.data_ptr(), B.shape[1], A.shape[1],
        ctypes.byref(m), mid.data_ptr(), mid.stride(0), y.data_ptr(), y.stride(0), DT[x.dtype],
        status.data_ptr() if status is not None else None, _stream())


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor, stride_outer=None,
            stride_inner=None, inner=None) -> int:
    lib = _native.capi()
    hidden = x.shape[-1]
    rows = x.numel() // hidden
    so = 0 if stride_outer is None else stride_outer
    si = hidden if stride_inner is None else stride_inner
    inn = rows if inner is None else inner
    return lib.mlora_rmsnorm_fwd(x.data_ptr(), rows, hidden, so, si, max(inn, 1), w.data_ptr(), DT[w.dtype],
                                 out.data_ptr(), hidden, eps, DT[x.dtype], _stream())


def check(rc: int) -> None:
    _native.check(rc)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()
