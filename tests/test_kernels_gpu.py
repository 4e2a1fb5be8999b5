"""Parity of the CUDA shrink/expand kernels, called through the C ABI, against the
oracle and the reference's golden vectors.

Tolerances: fp32 paths 1e-5 (accumulation order only); bf16/fp16 outputs within
max-abs 2e-2 and relative 1e-2 of the fp32-accumulated per-segment reference
(the bound stated for this path), and within 2 ulp of the reference's own
bf16 Torch backend where golden vectors exist.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import capi_helpers as C
from conftest import load_npz
from multi_lora_b200 import _native
from oracle import lora_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _to(a, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)


@pytest.mark.parametrize("name, key", [("toy_f32.npz", "torch"), ("toy_f32.npz", "triton"),
                                       ("decode_f32.npz", "torch"), ("decode_f32.npz", "triton")])
def test_fp32_matches_reference_golden(cuda_dev, name, key):
    z = load_npz(name)
    x, A, B, y = (_to(z[k], cuda_dev) for k in ("x", "A", "B", "y"))
    meta = C.meta_from_npz(z, cuda_dev)
    mid = torch.zeros(x.shape[0], A.shape[1], device=cuda_dev)
    C.check(C.shrink(x, A, meta, mid))
    C.check(C.expand(mid, B, meta, y))
    torch.cuda.synchronize()
    np.testing.assert_allclose(C.f32(mid), z[f"mid_{key}"][:, :A.shape[1]], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(C.f32(y), z[f"y_{key}"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ["prefill", "decode"])
def test_bf16_matches_reference_torch_backend(cuda_dev, case):
    z = load_npz("torch_bf16.npz")
    bf = lambda k: _to(O.bf16_from_bits(z[k]), cuda_dev, torch.bfloat16)  # noqa: E731
    A, B, x, y = bf("A"), bf("B"), bf(f"{case}_x"), bf(f"{case}_y")
    meta = C.meta_from_npz(z, cuda_dev, f"{case}_", scal_dtype=torch.bfloat16)
    mid = torch.zeros(x.shape[0], A.shape[1], device=cuda_dev, dtype=torch.bfloat16)
    C.check(C.shrink(x, A, meta, mid))
    C.check(C.expand(mid, B, meta, y))
    torch.cuda.synchronize()
    ref_mid = O.bf16_from_bits(z[f"{case}_mid"])
    ref_out = O.bf16_from_bits(z[f"{case}_out"])
    np.testing.assert_allclose(C.f32(mid), ref_mid, rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(C.f32(y), ref_out, rtol=2 ** -6, atol=2 ** -7)
    ind, widx, ranks, scal, bs = (z[f"{case}_seg_indptr"], z[f"{case}_weight_indices"], z[f"{case}_lora_ranks"],
                                  z[f"{case}_scalings"], int(z[f"{case}_bs"]))
    want = O.apply_lora_fp32(O.bf16_from_bits(z[f"{case}_x"]), O.bf16_from_bits(z["A"]), O.bf16_from_bits(z["B"]),
                             ind, widx, ranks, scal, bs, O.bf16_from_bits(z[f"{case}_y"]))
    np.testing.assert_allclose(C.f32(y), want, rtol=RTOL, atol=ATOL)


def _case(seed, dtype, n_in, n_out, R, ranks, lens, dev, nan_tails=True, y_pad=(1, 8)):
    g = torch.Generator().manual_seed(seed)
    K = len(ranks)
    S = sum(lens)
    widx = torch.randint(0, K, (len(lens),), generator=g).tolist()
    scal = [float(0.5 + (i % 4) * 0.5) for i in range(K)]
    x = torch.randn(S, n_in, generator=g).to(dtype)
    A = (torch.randn(K, R, n_in, generator=g) * n_in ** -0.5).to(dtype)
    B = (torch.randn(K, n_out, R, generator=g) * 0.05).to(dtype)
    if nan_tails:  # weights past each slot's rank are stale in the pool; must never be read
        for s, r in enumerate(ranks):
            A[s, r:] = float("nan")
            B[s, :, r:] = float("nan")
    ybase = torch.randn(S, n_out, generator=g).to(dtype)
    # y lives inside a larger buffer with a sentinel border (guard band)
    big = torch.full((S + 2 * y_pad[0], n_out + 2 * y_pad[1]), 7.0, dtype=dtype)
    big[y_pad[0]:y_pad[0] + S, y_pad[1]:y_pad[1] + n_out] = ybase
    return dict(x=x.to(dev), A=A.to(dev), B=B.to(dev), ybase=ybase, big=big.to(dev), widx=widx, scal=scal,
                lens=lens, ranks=ranks, pad=y_pad)


def _check_case(c, dev, dtype, scal_dtype=torch.float32):
    S = c["x"].shape[0]
    R = c["A"].shape[1]
    n_out = c["B"].shape[1]
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], dev, scal_dtype)
    mid_big = torch.full((S, R + 4), -3.0, dtype=dtype, device=dev)  # columns past rank keep the sentinel
    mid = mid_big[:, :R]
    p0, p1 = c["pad"]
    y = c["big"][p0:p0 + S, p1:p1 + n_out]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    C.check(C.shrink(c["x"], c["A"], meta, mid, status=status))
    C.check(C.expand(mid, c["B"], meta, y, status=status))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ind = meta.seg_indptr.cpu().numpy()
    want = O.apply_lora_fp32(C.f32(c["x"]), np.nan_to_num(C.f32(c["A"])), np.nan_to_num(C.f32(c["B"])), ind,
                             c["widx"], c["ranks"], [float(torch.tensor(s, dtype=scal_dtype)) for s in c["scal"]],
                             len(c["lens"]), C.f32(c["ybase"]))
    got = C.f32(y)
    assert np.isfinite(got).all()
    tol = (1e-4, 1e-4) if dtype == torch.float32 else (RTOL, ATOL)
    np.testing.assert_allclose(got, want, rtol=tol[0], atol=tol[1])
    # guard band untouched
    big = C.f32(c["big"])
    inner = np.zeros(big.shape, bool)
    inner[p0:p0 + S, p1:p1 + n_out] = True
    assert (big[~inner] == 7.0).all()
    # mid: columns >= rank (and whole rank-0 / empty segments) untouched
    m = C.f32(mid_big)
    assert (m[:, R:] == -3.0).all()
    x32, a32 = C.f32(c["x"]), np.nan_to_num(C.f32(c["A"]))
    for seg, slot in enumerate(c["widx"]):
        r = c["ranks"][slot]
        rows = slice(ind[seg], ind[seg + 1])
        assert (m[rows, r:R] == -3.0).all()
        mid_want = O.shrink(x32[rows], a32[[slot]], [0, rows.stop - rows.start], [0], [r], 1, "f32")
        tol_m = 1e-4 if dtype == torch.float32 else 1e-2
        np.testing.assert_allclose(m[rows, :r], mid_want[:, :r], rtol=tol_m, atol=tol_m)


STREAM_OP_SHAPES = [
    # n_in, n_out, R, ranks, lens: 256 rows or more of short segments
    (4096, 1024, 16, [16] * 8 + [0], [1] * 300),                # decode-sized, a base (rank-0) slot
    (1024, 768, 32, [32, 8, 17, 24], [1] * 200 + [3] * 30),     # ranks < max_rank (NaN tails), multi-token segments
]


@pytest.mark.parametrize("mid_dtype", [torch.bfloat16, torch.float32], ids=["mid_bf16", "mid_f32"])
@pytest.mark.parametrize("shape", STREAM_OP_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_standalone_shrink_and_expand_take_streaming_kernels(cuda_dev, shape, mid_dtype):
    """mlora_sgemm_lora_a_fwd / _b_fwd at 256+ rows run the streaming kernels
    alone. An fp32 mid is the tensor-parallel shrink partial: written unrounded
    by the shrink, rounded to bf16 by the expand as it loads it."""
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 5)) % 1000, torch.bfloat16, n_in, n_out, R, ranks, lens, cuda_dev)
    S = c["x"].shape[0]
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], cuda_dev)
    mid_big = torch.full((S, R + 8), -3.0, dtype=mid_dtype, device=cuda_dev)  # 16-byte rows, sentinel past R
    mid = mid_big[:, :R]
    p0, p1 = c["pad"]
    y = c["big"][p0:p0 + S, p1:p1 + n_out]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    C.check(C.shrink(c["x"], c["A"], meta, mid, status=status))
    assert _native.capi().mlora_last_apply_path() == 3
    C.check(C.expand(mid, c["B"], meta, y, status=status))
    assert _native.capi().mlora_last_apply_path() == 3
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ind = meta.seg_indptr.cpu().numpy()
    A32, B32 = np.nan_to_num(C.f32(c["A"])), np.nan_to_num(C.f32(c["B"]))
    want = O.apply_lora_fp32(C.f32(c["x"]), A32, B32, ind, c["widx"], c["ranks"], c["scal"], len(c["lens"]),
                             C.f32(c["ybase"]))
    got = C.f32(y)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    big = C.f32(c["big"])
    inner = np.zeros(big.shape, bool)
    inner[p0:p0 + S, p1:p1 + n_out] = True
    assert (big[~inner] == 7.0).all()
    m = C.f32(mid_big)
    assert (m[:, R:] == -3.0).all()
    tol_m = 1e-3 if mid_dtype == torch.float32 else 1e-2
    for seg, slot in enumerate(c["widx"]):
        r = c["ranks"][slot]
        rows = slice(ind[seg], ind[seg + 1])
        assert (m[rows, r:R] == -3.0).all()  # columns past the rank, and rank-0 segments, untouched
        mid_want = C.f32(c["x"])[rows] @ A32[slot, :r].T
        np.testing.assert_allclose(m[rows, :r], mid_want, rtol=tol_m, atol=tol_m)


SHAPES = [
    # n_in, n_out, R, ranks, lens
    (4096, 4096, 16, [16] * 6, [1] * 24),                       # decode, cfg2-like module
    (4096, 11008, 16, [16, 16, 0, 16], [1] * 16),               # gate/up width, base slot
    (11008, 4096, 16, [16, 16, 16], [1] * 12),                  # down in-dim
    (1024, 1000, 64, [0, 8, 64, 17, 32], [1] * 20),             # mixed ranks incl. odd rank, out % 256 != 0
    (512, 384, 64, [8, 64, 16], [5, 1, 7, 3, 2, 0, 9]),         # prefill segments incl. an empty one
    (100, 72, 20, [20, 4, 9], [3, 1, 4]),                       # unaligned in/out/R: scalar paths
    (256, 256, 8, [8, 8, 8, 8], [1, 3, 5, 2, 7, 4]),            # cfg1 shape
    (2048, 2048, 16, [16] * 3, [40, 25, 33]),                   # many tokens per slot (> tile)
    (28672 // 8, 8192 // 8, 16, [16] * 8, [1] * 32),            # cfg5 TP8 down shard
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_random_cases_match_oracle(cuda_dev, dtype, shape):
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R)) % 1000, dtype, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_case(c, cuda_dev, dtype)


class forced_path:
    """Force the apply path tried first (mlora_set_apply_path) inside a with-block."""

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        self.old = _native.get_apply_path()
        _native.set_apply_path(self.name)

    def __exit__(self, *exc):
        _native.set_apply_path(self.old)


def _check_apply(c, dev, dtype, expect_path=None, force="auto"):
    """apply_lora through the C ABI (path `force` tried first) against the oracle."""
    S = c["x"].shape[0]
    R = c["A"].shape[1]
    n_out = c["B"].shape[1]
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], dev)
    mid_big = torch.full((S, R + 8), -3.0, dtype=dtype, device=dev)
    mid = mid_big[:, :R]
    p0, p1 = c["pad"]
    y = c["big"][p0:p0 + S, p1:p1 + n_out]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    with forced_path(force):
        C.check(C.apply_lora(c["x"], c["A"], c["B"], meta, mid, y, status=status))
        path = _native.capi().mlora_last_apply_path()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    if expect_path is not None:
        assert path == expect_path
    ind = meta.seg_indptr.cpu().numpy()
    want = O.apply_lora_fp32(C.f32(c["x"]), np.nan_to_num(C.f32(c["A"])), np.nan_to_num(C.f32(c["B"])), ind,
                             c["widx"], c["ranks"], c["scal"], len(c["lens"]), C.f32(c["ybase"]))
    got = C.f32(y)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    big = C.f32(c["big"])
    inner = np.zeros(big.shape, bool)
    inner[p0:p0 + S, p1:p1 + n_out] = True
    assert (big[~inner] == 7.0).all()
    m = C.f32(mid_big)
    assert (m[:, R:] == -3.0).all()
    x32, a32 = C.f32(c["x"]), np.nan_to_num(C.f32(c["A"]))  # once: the stacks can be 100+ MB
    for seg, slot in enumerate(c["widx"]):
        r = c["ranks"][slot]
        rows = slice(ind[seg], ind[seg + 1])
        assert (m[rows, r:R] == -3.0).all()
        mid_want = x32[rows] @ a32[slot, :r].T
        np.testing.assert_allclose(m[rows, :r], mid_want, rtol=1e-2, atol=1e-2)
    return path


FUSED_SHAPES = [s for s in SHAPES if s[0] % 8 == 0 and s[2] % 8 == 0 and s[2] <= 64 and max(s[4]) <= 16]
STREAM_SHAPES = [s for s in SHAPES if s[0] % 16 == 0 and s[1] % 8 == 0 and s[2] % 8 == 0 and s[2] <= 64]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", FUSED_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_fused_apply_matches_oracle(cuda_dev, dtype, shape):
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 1)) % 1000, dtype, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_apply(c, cuda_dev, dtype, expect_path=1, force="fused")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", STREAM_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_stream_apply_matches_oracle(cuda_dev, dtype, shape):
    """The streaming shrink/expand pair (chosen automatically from 256 rows up)."""
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 3)) % 1000, dtype, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_apply(c, cuda_dev, dtype, expect_path=3, force="stream")


@pytest.mark.parametrize("shape", [s for s in SHAPES if s not in FUSED_SHAPES], ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_apply_falls_back_to_two_launches(cuda_dev, shape):
    """Below 256 rows, shapes the fused kernel cannot take run shrink + expand."""
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 2)) % 1000, torch.bfloat16, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=2)


@pytest.mark.parametrize("shape", SHAPES[:2] + SHAPES[7:8], ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}")
def test_forced_split_apply_matches_oracle(cuda_dev, shape):
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 4)) % 1000, torch.bfloat16, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=2, force="split")


def test_fused_apply_many_segments_and_cluster16(cuda_dev):
    """bs above one scan pass (256) and an in-dim that needs 16-CTA clusters."""
    c = _case(21, torch.bfloat16, 512, 640, 16, [16, 16, 8] * 4, [1] * 700, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=1, force="fused")
    c = _case(22, torch.bfloat16, 40960, 1024, 16, [16] * 4, [1] * 16, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=1, force="fused")


TC_SHAPES = [
    # n_in, n_out, R, ranks, lens
    (512, 384, 64, [64, 64, 64], [300, 129, 64]),              # ragged tiles (300 = 128 + 128 + 44), 1-row tile
    (1024, 1000, 64, [64, 8, 33, 0], [200, 150, 77, 90]),      # ranks < R (NaN-planted tails), base segment,
                                                               # out % 128 != 0 (partial column block)
    (4096, 1024, 64, [64] * 8, [469, 845, 454, 989, 348, 314, 495, 426]),  # cfg3 k/v projection, full size
    (512, 384, 16, [16, 16, 8], [300, 129, 64]),               # max_rank 16: 32-byte swizzled rank tiles
    (1024, 1000, 32, [32, 8, 17, 0], [200, 150, 77, 90]),      # max_rank 32: 64-byte swizzle, odd rank 17
    (4096, 4096, 16, [16] * 8, [469, 845, 454, 989, 348, 314, 495, 426]),  # cfg3 q shape at rank 16
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}r{s[2]}s{sum(s[4])}")
def test_tc_apply_matches_oracle(cuda_dev, dtype, shape):
    """tcgen05 shrink/expand pair (the automatic choice for segments of >= 64 rows)."""
    n_in, n_out, R, ranks, lens = shape
    c = _case(hash((n_in, n_out, R, 5)) % 1000, dtype, n_in, n_out, R, ranks, lens, cuda_dev)
    _check_apply(c, cuda_dev, dtype, expect_path=4)


@pytest.mark.parametrize("lens", [[128, 100] * 80, [200, 64] * 30], ids=["160_tiles_1_split", "90_tiles_2_splits"])
def test_tc_apply_many_tiles(cuda_dev, lens):
    """Many prefill tiles: the shrink's K split falls to 1 (a grid of more than one wave of
    two-per-SM CTAs) or 2, where the small cases above run 3-8 way splits."""
    c = _case(31, torch.bfloat16, 512, 384, 64, [64, 40, 16], lens, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=4)


@pytest.mark.parametrize("R, ranks", [(64, [64, 8, 33]), (16, [16, 8, 13]), (32, [32, 32, 24])])
def test_tc_group_matches_separate_projections(cuda_dev, R, ranks):
    """q/k/v-like group on the tensor-core pair: mid [S, 3R] holds one column block per projection."""
    import ctypes

    dev, dt = cuda_dev, torch.bfloat16
    g = torch.Generator().manual_seed(77 + R)
    outs, lens, n_in = (512, 256, 128), [150, 90, 70], 640
    K, S = len(ranks), sum(lens)
    widx = [0, 1, 2]
    scal = [0.5 + i for i in range(K)]
    x = torch.randn(S, n_in, generator=g).to(dt)
    meta = C.make_meta(lens, widx, ranks, scal, dev)
    As, Bs, ys, y0 = [], [], [], []
    for o in outs:
        a = (torch.randn(K, R, n_in, generator=g) * n_in ** -0.5).to(dt)
        b = (torch.randn(K, o, R, generator=g) * 0.05).to(dt)
        for s_, r in enumerate(ranks):
            a[s_, r:] = float("nan")
            b[s_, :, r:] = float("nan")
        yb = torch.randn(S, o, generator=g).to(dt)
        As.append(a.to(dev))
        Bs.append(b.to(dev))
        y0.append(yb)
        ys.append(yb.to(dev).clone())
    xd = x.to(dev)
    mid = torch.zeros(S, 3 * R, dtype=dt, device=dev)
    n = len(outs)
    P = ctypes.c_void_p
    arr = lambda vals, t: (t * n)(*vals)  # noqa: E731
    m = meta.struct()
    rc = _native.capi().mlora_apply_lora_group(
        xd.data_ptr(), S, n_in, n_in, n, arr([a.data_ptr() for a in As], P), arr([b.data_ptr() for b in Bs], P),
        arr(list(outs), ctypes.c_int64), arr([y.data_ptr() for y in ys], P),
        arr([y.stride(0) for y in ys], ctypes.c_int64), R, ctypes.byref(m), mid.data_ptr(), 3 * R, 0, None,
        torch.cuda.current_stream().cuda_stream)
    C.check(rc)
    assert _native.capi().mlora_last_apply_path() == 4
    torch.cuda.synchronize()
    ind = meta.seg_indptr.cpu().numpy()
    for a, b, yb, y in zip(As, Bs, y0, ys):
        want = O.apply_lora_fp32(C.f32(x), np.nan_to_num(C.f32(a)), np.nan_to_num(C.f32(b)), ind, widx, ranks, scal,
                                 len(lens), C.f32(yb))
        np.testing.assert_allclose(C.f32(y), want, rtol=RTOL, atol=ATOL)


def test_stream_apply_many_slots_and_long_segments(cuda_dev):
    """cfg5-like routing (128 slots, 512 one-token segments), one slot with 100
    tokens (13 tiles), and more segments than one slot's tile."""
    c = _case(31, torch.bfloat16, 1024, 512, 16, [16, 8, 0, 16] * 32, [1] * 512, cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=3)
    c = _case(32, torch.bfloat16, 512, 1024, 32, [32, 24], [100, 3, 1, 60], cuda_dev)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=3, force="stream")


@pytest.mark.parametrize("n_slots", [8, 32])
def test_stream_apply_many_one_token_segments_per_slot(cuda_dev, n_slots):
    """Hundreds of one-token segments over few slots: each slot spans several
    tiles, and every CTA must cut them identically (a single apply and a group)."""
    dev = cuda_dev
    c = _case(40 + n_slots, torch.bfloat16, 1024, 1024, 16, [16] * n_slots, [1] * 256, dev)
    _check_apply(c, dev, torch.bfloat16, expect_path=3)  # 256 rows: the automatic choice
    import ctypes

    g = torch.Generator().manual_seed(n_slots)
    outs = (1024, 256, 256)
    x = torch.randn(256, 1024, generator=g).bfloat16()
    widx = torch.randint(0, n_slots, (256,), generator=g).tolist()
    ranks, scal = [16] * n_slots, [2.0] * n_slots
    meta = C.make_meta([1] * 256, widx, ranks, scal, dev)
    As = [((torch.rand(n_slots, 16, 1024, generator=g) * 2 - 1) / 32).bfloat16() for _ in outs]
    Bs = [(torch.randn(n_slots, o, 16, generator=g) * 0.02).bfloat16() for o in outs]
    y0 = [torch.randn(256, o, generator=g).bfloat16() for o in outs]
    ys = [y.to(dev).clone() for y in y0]
    xd, Ad, Bd = x.to(dev), [a.to(dev) for a in As], [b.to(dev) for b in Bs]  # alive across the launch
    mid = torch.zeros(256, 64, dtype=torch.bfloat16, device=dev)
    P = ctypes.c_void_p
    arr = lambda vals, t: (t * 3)(*vals)  # noqa: E731
    m = meta.struct()
    rc = _native.capi().mlora_apply_lora_group(
        xd.data_ptr(), 256, 1024, 1024, 3, arr([a.data_ptr() for a in Ad], P),
        arr([b.data_ptr() for b in Bd], P), arr(list(outs), ctypes.c_int64), arr([y.data_ptr() for y in ys], P),
        arr([y.stride(0) for y in ys], ctypes.c_int64), 16, ctypes.byref(m), mid.data_ptr(), 64, 0, None,
        torch.cuda.current_stream().cuda_stream)
    C.check(rc)
    assert _native.capi().mlora_last_apply_path() == 3
    torch.cuda.synchronize()
    ind = meta.seg_indptr.cpu().numpy()
    for a, b, yb, y in zip(As, Bs, y0, ys):
        want = O.apply_lora_fp32(C.f32(x), C.f32(a), C.f32(b), ind, widx, ranks, scal, 256, C.f32(yb))
        np.testing.assert_allclose(C.f32(y), want, rtol=RTOL, atol=ATOL)


def test_stream_apply_is_deterministic(cuda_dev):
    """Two calls in a row on the same inputs give bit-identical y and mid."""
    c = _case(33, torch.bfloat16, 4096, 4096, 16, [16] * 32, [1] * 64, cuda_dev, nan_tails=False)
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], cuda_dev)
    outs = []
    with forced_path("stream"):
        for _ in range(2):
            mid = torch.zeros(64, 16, dtype=torch.bfloat16, device=cuda_dev)
            y = c["ybase"].to(cuda_dev).clone()
            C.check(C.apply_lora(c["x"], c["A"], c["B"], meta, mid, y))
            assert _native.capi().mlora_last_apply_path() == 3
            outs.append((mid, y))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_stream_apply_invalid_routing_sets_status(cuda_dev):
    """Slot out of range, overlapping segments (more rows than S) and a rank
    above max_rank are reported; the launch stays in bounds."""
    dev = cuda_dev
    x = torch.randn(4, 64, device=dev).bfloat16()
    A = torch.randn(2, 16, 64, device=dev).bfloat16()
    B = torch.randn(2, 128, 16, device=dev).bfloat16()
    cases = {
        1: C.make_meta([1, 1], [0, 5], [16, 16], [1.0, 1.0], dev),
        4: C.make_meta([4, 3, 3], [0, 1, 0], [16, 16], [1.0, 1.0], dev, indptr=[0, 4, 1, 4]),
        2: C.make_meta([1, 1], [0, 1], [16, 99], [1.0, 1.0], dev),
    }
    for bit, meta in cases.items():
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        mid = torch.zeros(4, 16, dtype=torch.bfloat16, device=dev)
        y = torch.zeros(4, 128, dtype=torch.bfloat16, device=dev)
        with forced_path("stream"):
            C.check(C.apply_lora(x, A, B, meta, mid, y, status=status))
            assert _native.capi().mlora_last_apply_path() == 3
        torch.cuda.synchronize()
        assert int(status.item()) & bit, (bit, int(status.item()))


@pytest.mark.parametrize("force", ["fused", "stream"])
def test_apply_rank0_and_unused_slots_leave_y(cuda_dev, force):
    """Only base-model (rank 0) segments: y is bit-identical afterwards."""
    c = _case(23, torch.bfloat16, 1024, 512, 16, [0, 16, 16], [1] * 8, cuda_dev, nan_tails=False)
    c["widx"] = [0] * 8
    before = c["big"].clone()
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], cuda_dev)
    mid = torch.zeros(8, 16, dtype=torch.bfloat16, device=cuda_dev)
    p0, p1 = c["pad"]
    with forced_path(force):
        C.check(C.apply_lora(c["x"], c["A"], c["B"], meta, mid, c["big"][p0:p0 + 8, p1:p1 + 512]))
    torch.cuda.synchronize()
    assert torch.equal(c["big"], before)


@pytest.mark.parametrize("outs, R, ranks, lens, path, wide_path", [
    ((4096, 1024, 1024), 16, [16] * 8, [1] * 32, 1, 3),        # q/k/v of a GQA block
    ((11008, 11008), 16, [16, 0, 16, 8], [1] * 24, 1, 3),      # gate/up
    ((384, 200, 72), 64, [64, 8, 17], [3, 1, 5, 2], 1, 3),     # mixed ranks
    ((96, 64), 20, [20, 4], [2, 1, 3], 2, 2),                  # R % 8 != 0: two launches per projection
])
@pytest.mark.parametrize("wide", [False, True], ids=["auto_mid_R", "stream_mid_4R"])
def test_group_matches_separate_projections(cuda_dev, outs, R, ranks, lens, path, wide_path, wide):
    """Automatic path with mid [S, R]; the streaming pair (forced) needs mid
    [S, >= n*R], one column block per projection."""
    """mlora_apply_lora_group == one oracle apply per projection (shared x and routing)."""
    import ctypes

    dev, dt = cuda_dev, torch.bfloat16
    g = torch.Generator().manual_seed(len(outs) * 7 + R)
    n_in = 256 if R != 20 else 96
    K = len(ranks)
    S = sum(lens)
    widx = torch.randint(0, K, (len(lens),), generator=g).tolist()
    scal = [0.5 + i for i in range(K)]
    x = torch.randn(S, n_in, generator=g).to(dt)
    meta = C.make_meta(lens, widx, ranks, scal, dev)
    As, Bs, ys, y0 = [], [], [], []
    for o in outs:
        a = (torch.randn(K, R, n_in, generator=g) * n_in ** -0.5).to(dt)
        b = (torch.randn(K, o, R, generator=g) * 0.05).to(dt)
        for s, r in enumerate(ranks):
            a[s, r:] = float("nan")
            b[s, :, r:] = float("nan")
        yb = torch.randn(S, o, generator=g).to(dt)
        As.append(a.to(dev))
        Bs.append(b.to(dev))
        y0.append(yb)
        ys.append(yb.to(dev).clone())
    xd = x.to(dev)
    mid_cols = 4 * R if wide else R
    mid = torch.zeros(S, mid_cols, dtype=dt, device=dev)
    n = len(outs)
    P = ctypes.c_void_p
    arr = lambda vals, t: (t * n)(*vals)  # noqa: E731
    m = meta.struct()
    with forced_path("stream" if wide else "auto"):
        rc = _native.capi().mlora_apply_lora_group(
            xd.data_ptr(), S, n_in, n_in, n, arr([a.data_ptr() for a in As], P), arr([b.data_ptr() for b in Bs], P),
            arr(list(outs), ctypes.c_int64), arr([y.data_ptr() for y in ys], P),
            arr([y.stride(0) for y in ys], ctypes.c_int64), R, ctypes.byref(m), mid.data_ptr(), mid_cols, 0, None,
            torch.cuda.current_stream().cuda_stream)
        C.check(rc)
        assert _native.capi().mlora_last_apply_path() == (wide_path if wide else path)
    torch.cuda.synchronize()
    ind = meta.seg_indptr.cpu().numpy()
    for a, b, yb, y in zip(As, Bs, y0, ys):
        want = O.apply_lora_fp32(C.f32(x), np.nan_to_num(C.f32(a)), np.nan_to_num(C.f32(b)), ind, widx, ranks, scal,
                                 len(lens), C.f32(yb))
        np.testing.assert_allclose(C.f32(y), want, rtol=RTOL, atol=ATOL)


def test_many_segments_more_than_one_pass(cuda_dev):
    """bs above the per-pass segment capacity (256) for one slot."""
    lens = [1] * 700
    c = _case(5, torch.bfloat16, 512, 640, 16, [16, 16], lens, cuda_dev)
    _check_case(c, cuda_dev, torch.bfloat16)


def test_bf16_scalings_dtype(cuda_dev):
    c = _case(7, torch.bfloat16, 1024, 512, 16, [16, 8, 16], [1] * 10, cuda_dev)
    _check_case(c, cuda_dev, torch.bfloat16, scal_dtype=torch.bfloat16)


def test_fp32_partial_mid_equals_rounded_path(cuda_dev):
    """Shrink into f32 partial sums + expand reading f32 mid == the bf16-mid path, bit for bit."""
    c = _case(11, torch.bfloat16, 2048, 1024, 16, [16, 16, 8], [1] * 12, cuda_dev, nan_tails=False)
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], cuda_dev)
    S = c["x"].shape[0]
    mid_b = torch.zeros(S, 16, dtype=torch.bfloat16, device=cuda_dev)
    mid_f = torch.zeros(S, 16, dtype=torch.float32, device=cuda_dev)
    y1 = c["ybase"].to(cuda_dev).clone()
    y2 = c["ybase"].to(cuda_dev).clone()
    C.check(C.shrink(c["x"], c["A"], meta, mid_b))
    C.check(C.shrink(c["x"], c["A"], meta, mid_f))
    C.check(C.expand(mid_b, c["B"], meta, y1))
    C.check(C.expand(mid_f, c["B"], meta, y2))
    torch.cuda.synchronize()
    assert torch.equal(mid_f.bfloat16(), mid_b)
    assert torch.equal(y1, y2)


def test_stack_num(cuda_dev):
    """stack_num widens the written rows to rank * stack_num (sgemm_lora_a.py:51)."""
    dev = cuda_dev
    g = torch.Generator().manual_seed(3)
    K, R, n_in, S = 3, 48, 256, 6
    ranks = [8, 16, 4]
    A = torch.randn(K, R, n_in, generator=g).bfloat16().to(dev)
    x = torch.randn(S, n_in, generator=g).bfloat16().to(dev)
    meta = C.make_meta([2, 1, 3], [0, 1, 2], ranks, [1.0] * K, dev)
    mid = torch.full((S, R), -5.0, dtype=torch.bfloat16, device=dev)
    C.check(C.shrink(x, A, meta, mid, stack_num=3))
    torch.cuda.synchronize()
    m = C.f32(mid)
    ind = [0, 2, 3, 6]
    for seg, slot in enumerate([0, 1, 2]):
        n = min(R, ranks[slot] * 3)
        want = C.f32(x)[ind[seg]:ind[seg + 1]] @ C.f32(A)[slot, :n].T
        np.testing.assert_allclose(m[ind[seg]:ind[seg + 1], :n], want, rtol=1e-2, atol=1e-2)
        assert (m[ind[seg]:ind[seg + 1], n:] == -5.0).all()


def test_invalid_routing_sets_status_and_skips(cuda_dev):
    """Out-of-range slot / indptr / rank are reported in the status word; nothing is written."""
    dev = cuda_dev
    x = torch.randn(4, 64, device=dev).bfloat16()
    A = torch.randn(2, 16, 64, device=dev).bfloat16()
    B = torch.randn(2, 128, 16, device=dev).bfloat16()
    cases = {
        1: C.make_meta([1, 1], [0, 5], [16, 16], [1.0, 1.0], dev),                     # slot 5 of 2
        4: C.make_meta([1, 1], [0, 1], [16, 16], [1.0, 1.0], dev, indptr=[0, 1, 9]),   # past S=4
        2: C.make_meta([1, 1], [0, 1], [16, 99], [1.0, 1.0], dev),                     # rank > max_rank (clamped)
    }
    for bit, meta in cases.items():
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        mid = torch.zeros(4, 16, dtype=torch.bfloat16, device=dev)
        y = torch.zeros(4, 128, dtype=torch.bfloat16, device=dev)
        C.check(C.shrink(x, A, meta, mid, status=status))
        C.check(C.expand(mid, B, meta, y, status=status))
        torch.cuda.synchronize()
        assert int(status.item()) & bit, (bit, int(status.item()))


@pytest.mark.parametrize("force", ["fused", "stream"])
def test_pdl_on_and_off_agree(cuda_dev, force):
    c = _case(13, torch.bfloat16, 4096, 4096, 16, [16] * 8, [1] * 32, cuda_dev, nan_tails=False)
    meta = C.make_meta(c["lens"], c["widx"], c["ranks"], c["scal"], cuda_dev)
    outs = []
    old = _native.get_pdl()
    with forced_path(force):
        for pdl in (True, False):
            _native.set_pdl(pdl)
            mid = torch.zeros(32, 16, dtype=torch.bfloat16, device=cuda_dev)
            y = c["ybase"].to(cuda_dev).clone()
            C.check(C.apply_lora(c["x"], c["A"], c["B"], meta, mid, y))
            torch.cuda.synchronize()
            outs.append(y)
    _native.set_pdl(old)
    assert torch.equal(outs[0], outs[1])


def test_empty_batch_is_noop(cuda_dev):
    x = torch.randn(0, 64, device=cuda_dev).bfloat16()
    A = torch.randn(2, 16, 64, device=cuda_dev).bfloat16()
    meta = C.make_meta([], [], [16, 16], [1.0, 1.0], cuda_dev)
    mid = torch.zeros(0, 16, dtype=torch.bfloat16, device=cuda_dev)
    C.check(C.shrink(x, A, meta, mid))
    torch.cuda.synchronize()
