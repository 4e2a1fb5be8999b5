"""RMSNorm kernel parity: reference golden (its Triton kernel), oracle, and the
reference's own test cases (test_fused_rmsnorm.py: 2e-2 against the HF formula)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn

import capi_helpers as C
from conftest import load_npz
from multi_lora_b200.rmsnorm import fuse_rmsnorm, rmsnorm_fwd, rmsnorm_out
from oracle import lora_oracle as O

pytestmark = pytest.mark.gpu


class RefRMSNorm(nn.Module):
    """The HF formula the reference tests compare against (test_fused_rmsnorm.py:18-32)."""

    def __init__(self, hidden, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(hidden))
        self.variance_epsilon = eps

    def forward(self, x):
        h = x.to(torch.float32)
        var = h.pow(2).mean(-1, keepdim=True)
        h = h * torch.rsqrt(var + self.variance_epsilon)
        return self.weight * h.to(x.dtype)


def test_matches_reference_kernel_golden(cuda_dev):
    z = load_npz("rmsnorm.npz")
    x = torch.from_numpy(z["f32_x"]).to(cuda_dev)
    w = torch.from_numpy(z["f32_w"]).to(cuda_dev)
    np.testing.assert_allclose(C.f32(rmsnorm_fwd(x, w, 1e-6)), z["f32_y"], rtol=1e-5, atol=1e-5)
    bf = lambda k: torch.from_numpy(O.bf16_from_bits(z[k])).to(cuda_dev).bfloat16()  # noqa: E731
    for case in ("bf16", "wide"):
        x, w = bf(f"{case}_x"), bf(f"{case}_w")
        got = C.f32(rmsnorm_fwd(x, w, 1e-6))
        pre = O.rmsnorm_f32(C.f32(x), C.f32(w), 1e-6)
        # the golden was cast by truncation (interpreter); the GPU rounds to nearest even
        np.testing.assert_allclose(got, O.bf16_from_bits(z[f"{case}_y"]), rtol=2 ** -7, atol=1e-6)
        np.testing.assert_allclose(got, O.bf16_round(pre), rtol=2 ** -7, atol=1e-6)
        assert np.mean(got == O.bf16_round(pre)) > 0.98
    qkv = bf("slice_qkv")
    sl = qkv[..., :256].view(2, 3, 2, 128)
    assert not sl.is_contiguous()
    got = rmsnorm_fwd(sl, bf("slice_w"), 1e-6)
    assert got.shape == sl.shape
    np.testing.assert_allclose(C.f32(got), O.bf16_from_bits(z["slice_y"]), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("hidden", [128, 2560, 4096, 8192, 100, 33000])
def test_matches_hf_formula(cuda_dev, hidden):
    torch.manual_seed(0)
    ref = RefRMSNorm(hidden).to(cuda_dev, torch.bfloat16)
    for shape in ((64, 1, hidden), (64, 7, hidden), (3, hidden)):
        x = torch.randn(*shape, device=cuda_dev, dtype=torch.bfloat16)
        want = ref(x)
        got = rmsnorm_fwd(x, ref.weight, 1e-6)
        assert got.shape == want.shape and got.dtype == want.dtype
        torch.testing.assert_close(got, want, rtol=2e-2, atol=2e-2)
        pre = O.rmsnorm_f32(C.f32(x), C.f32(ref.weight), 1e-6)
        np.testing.assert_allclose(C.f32(got), O.bf16_round(pre), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("batch,seq", [(64, 1), (64, 7)])
def test_non_contiguous_qkv_slice(cuda_dev, batch, seq):
    """q slice of a fused qkv [B,S,6144] output, read in place (two-level stride)."""
    torch.manual_seed(0)
    ref = RefRMSNorm(128).to(cuda_dev, torch.bfloat16)
    qkv = torch.randn(batch, seq, 6144, device=cuda_dev, dtype=torch.bfloat16)
    sl = qkv[..., :4096].view(batch, seq, 32, 128)
    assert not sl.is_contiguous()
    got = rmsnorm_fwd(sl, ref.weight, 1e-6)
    torch.testing.assert_close(got, ref(sl.contiguous()), rtol=2e-2, atol=2e-2)


def test_fp16_fp32_and_out_variant(cuda_dev):
    torch.manual_seed(1)
    for dt in (torch.float16, torch.float32):
        x = torch.randn(17, 1024, device=cuda_dev, dtype=dt)
        w = torch.randn(1024, device=cuda_dev, dtype=torch.float32)
        out = torch.empty_like(x)
        rmsnorm_out(x, w, 1e-5, out)
        pre = O.rmsnorm_f32(C.f32(x), C.f32(w), 1e-5)
        want = O.round_to(pre, "f16" if dt == torch.float16 else "f32")
        np.testing.assert_allclose(C.f32(out), want, rtol=2e-3 if dt == torch.float16 else 1e-5, atol=1e-5)


def test_fuse_patches_all_and_keeps_numerics(cuda_dev):
    torch.manual_seed(0)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.n1 = RefRMSNorm(2560)
            self.n2 = RefRMSNorm(128)
            self.lin = nn.Linear(8, 8)

    model = nn.Sequential(Block(), Block()).to(cuda_dev, torch.bfloat16)
    x1 = torch.randn(16, 1, 2560, device=cuda_dev, dtype=torch.bfloat16)
    x2 = torch.randn(16, 1, 128, device=cuda_dev, dtype=torch.bfloat16)
    want1, want2 = model[0].n1(x1), model[0].n2(x2)
    assert fuse_rmsnorm(model) == 4
    torch.testing.assert_close(model[0].n1(x1), want1, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(model[0].n2(x2), want2, rtol=2e-2, atol=2e-2)
    assert isinstance(model[0].n1.weight, nn.Parameter)


def test_cpu_input_raises():
    with pytest.raises(RuntimeError):
        rmsnorm_fwd(torch.randn(2, 8), torch.ones(8), 1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows, hidden", [(64, 4096), (7, 8192), (5, 1001), (3, 40960)])
def test_fused_add_rmsnorm_equals_add_then_norm(cuda_dev, dtype, rows, hidden):
    """residual = T(residual + x), out = rmsnorm(residual): bit-identical to the
    two-step sequence (a dtype add, then the RMSNorm kernel), and within the
    kernel's own tolerance of the oracle's RMSNorm of the rounded sum.
    Shapes: decode rows, rows longer than one register pass (40960), and a
    hidden size that is not a multiple of the 16-byte chunk (scalar path)."""
    from multi_lora_b200.rmsnorm import fused_add_rmsnorm

    g = torch.Generator().manual_seed(rows * 131 + hidden)
    res0 = torch.randn(rows, hidden, generator=g).to(dtype).to(cuda_dev)
    x = torch.randn(rows, hidden, generator=g).to(dtype).to(cuda_dev)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype).to(cuda_dev)
    res = res0.clone()
    out, res_ret = fused_add_rmsnorm(res, x, w, 1e-6)
    assert res_ret is res
    want_res = res0 + x  # torch adds in the dtype (fp32 arithmetic, one rounding)
    want_out = rmsnorm_fwd(want_res, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(res, want_res)
    assert torch.equal(out, want_out)
    name = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[dtype]
    oracle_res = O.round_to(C.f32(res0) + C.f32(x), name)
    np.testing.assert_array_equal(C.f32(res), oracle_res)
    np.testing.assert_allclose(C.f32(out), O.rmsnorm(oracle_res, C.f32(w), 1e-6, name),
                               rtol=2 ** -6 if dtype != torch.float32 else 1e-5, atol=1e-5)


def test_fused_add_rmsnorm_capi_strided_rows(cuda_dev):
    """Through the C ABI with row strides wider than hidden (rows inside larger buffers)."""
    import ctypes

    from multi_lora_b200 import _native

    g = torch.Generator().manual_seed(5)
    rows, hidden = 6, 512
    x_big = torch.randn(rows, hidden + 64, generator=g).bfloat16().to(cuda_dev)
    r_big = torch.randn(rows, hidden + 32, generator=g).bfloat16().to(cuda_dev)
    y_big = torch.full((rows, hidden + 16), 3.0, dtype=torch.bfloat16, device=cuda_dev)
    w = torch.randn(hidden, generator=g).bfloat16().to(cuda_dev)
    x, r, y = x_big[:, :hidden], r_big[:, :hidden], y_big[:, :hidden]
    want_r = r + x
    want_y = rmsnorm_fwd(want_r, w, 1e-5)
    rc = _native.capi().mlora_fused_add_rmsnorm_fwd(
        x.data_ptr(), x.stride(0), r.data_ptr(), r.stride(0), rows, hidden, w.data_ptr(), 0, y.data_ptr(),
        y.stride(0), ctypes.c_float(1e-5), 0, torch.cuda.current_stream().cuda_stream)
    C.check(rc)
    torch.cuda.synchronize()
    assert torch.equal(r, want_r) and torch.equal(y, want_y)
    assert (y_big[:, hidden:] == 3.0).all()  # the row tails are not written
