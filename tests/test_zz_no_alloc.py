"""The allocation-free apply_lora group entry point (mlora_apply_lora_group_noalloc).

Some callers cannot allocate device memory — a plugin host that passes this
library only its inputs and outputs, or a serving loop that must avoid
cudaMalloc's device synchronisation. For them the entry point keeps the
shrink-to-expand intermediate in a fixed 1 MiB device array owned by the
library. These tests call it through the C ABI twice in a row (the array
keeps the first call's contents when the second runs) and compare each
result with mlora_apply_lora_group, which uses a caller buffer, and with
the oracle's fp32 per-segment apply_lora, within the tolerance used for
bf16 results in the other GPU tests (max-abs 2e-2, relative 1e-2; 1e-4 for
fp32). Decode-shaped calls run the streaming shrink/expand kernels through
the array; prefill-shaped (rank 32, 128-row segments) and fp32 calls run the
general kernels; each test checks which ones ran. A call needing more than
1 MiB is refused with an error instead of running.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import capi_helpers as C
from multi_lora_b200 import _native
from oracle import lora_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
P = ctypes.c_void_p
I64 = ctypes.c_int64


def _problem(seed, dev, n_in=4096, outs=(4096, 1024, 1024), R=16, K=8, S=64, lens=None, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    ranks = [R if i % 4 else R // 2 for i in range(K)]
    lens = [1] * S if lens is None else lens
    S = sum(lens)
    widx = torch.randint(0, K, (len(lens),), generator=g).tolist()
    meta = C.make_meta(lens, widx, ranks, [0.5 + (i % 3) for i in range(K)], dev)
    x = torch.randn(S, n_in, generator=g).to(dtype).to(dev)
    a = [(torch.randn(K, R, n_in, generator=g) * n_in ** -0.5).to(dtype).to(dev) for _ in outs]
    b = [(torch.randn(K, o, R, generator=g) * 0.05).to(dtype).to(dev) for o in outs]
    y = [torch.randn(S, o, generator=g).to(dtype).to(dev) for o in outs]
    return x, a, b, y, meta, R, outs


def _oracle(x, a, b, y0, meta):
    """fp32 per-segment apply_lora of the reference's Torch backend (oracle restatement)."""
    ind = meta.seg_indptr.cpu().numpy()
    widx = meta.weight_indices.cpu().tolist()
    ranks = meta.lora_ranks.cpu().tolist()
    scal = meta.scalings.float().cpu().tolist()
    return O.apply_lora_fp32(C.f32(x), C.f32(a), C.f32(b), ind, widx, ranks, scal, len(widx), C.f32(y0))


DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _arrays(a, b, outs, ys):
    n = len(outs)
    return ((P * n)(*[t.data_ptr() for t in a]), (P * n)(*[t.data_ptr() for t in b]), (I64 * n)(*outs),
            (P * n)(*[t.data_ptr() for t in ys]), (I64 * n)(*[t.stride(0) for t in ys]))


def _run_noalloc(x, a, b, ys, meta, R, outs):
    aa, bb, oo, yy, ss = _arrays(a, b, outs, ys)
    m = meta.struct()
    return _native.capi().mlora_apply_lora_group_noalloc(
        x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), len(outs), aa, bb, oo, yy, ss, R, ctypes.byref(m),
        DTYPE_CODE[x.dtype], None, torch.cuda.current_stream().cuda_stream)


def _run_with_buffer(x, a, b, ys, meta, R, outs):
    aa, bb, oo, yy, ss = _arrays(a, b, outs, ys)
    m = meta.struct()
    mid = torch.empty(x.shape[0], R, dtype=x.dtype, device=x.device)
    return _native.capi().mlora_apply_lora_group(
        x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), len(outs), aa, bb, oo, yy, ss, R, ctypes.byref(m),
        mid.data_ptr(), R, DTYPE_CODE[x.dtype], None, torch.cuda.current_stream().cuda_stream)


CASES = {
    # name: (problem arguments, kernels the scratch passes through: 3 streaming pair, 2 general pair)
    "decode_bf16": (dict(), 3),
    "prefill_r32": (dict(n_in=1024, outs=(768, 256), R=32, K=4, lens=[128, 128, 128, 128]), 2),
    "decode_f32": (dict(n_in=512, outs=(256, 384), R=16, K=4, S=48, dtype=torch.float32), 2),
}


@pytest.mark.parametrize("case", list(CASES))
def test_noalloc_matches_buffered_entry_point_twice(cuda_dev, case):
    kwargs, path = CASES[case]
    tol = (1e-4, 1e-4) if kwargs.get("dtype") == torch.float32 else (RTOL, ATOL)
    for seed in (1, 2):  # two calls in a row: the scratch holds the previous call's mid
        x, a, b, y0, meta, R, outs = _problem(seed, cuda_dev, **kwargs)
        y_ref = [t.clone() for t in y0]
        y_new = [t.clone() for t in y0]
        C.check(_run_with_buffer(x, a, b, y_ref, meta, R, outs))
        C.check(_run_noalloc(x, a, b, y_new, meta, R, outs))
        assert _native.capi().mlora_last_apply_path() == path
        torch.cuda.synchronize()
        for i, (r, n, before) in enumerate(zip(y_ref, y_new, y0)):
            np.testing.assert_allclose(C.f32(n), C.f32(r), rtol=tol[0], atol=tol[1])
            np.testing.assert_allclose(C.f32(n), _oracle(x, a[i], b[i], before, meta), rtol=tol[0], atol=tol[1])
            assert not torch.equal(n, before)  # the delta was applied


def test_noalloc_refuses_calls_beyond_its_scratch(cuda_dev):
    # 40000 rows x max_rank 16 x 2 bytes = 1.28 MB > 1 MiB: refused before any launch
    x, a, b, y, meta, R, outs = _problem(3, cuda_dev, n_in=64, outs=(64,), S=40000, K=2)
    rc = _run_noalloc(x, a, b, y, meta, R, outs)
    assert rc == -1
    assert b"1 MiB" in _native.capi().mlora_last_error()
