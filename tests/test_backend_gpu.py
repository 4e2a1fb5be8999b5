"""Drop-in API on the GPU: backend, LinearWithLoRA, QKV fusion, manager, CUDA graphs.

Mirrors the reference's integration tests (test_phase4_backend.py,
test_triton_sgemm.py, test_fused_qkv.py, test_grouped_rows.py,
test_graph_decode.py) with the CUDA backend in place of Triton and the
oracle / a torch fp32 computation as the comparator.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn

from multi_lora_b200.backend import CudaLoRABackend, get_lora_backend
from multi_lora_b200.batch_info import KernelInputMetaData
from multi_lora_b200.layers import LinearWithLoRA, fuse_qkv_projections, lora_delta, set_lora_enabled
from multi_lora_b200.manager import MultiLoRAManager, wrap_linear_modules
from multi_lora_b200.weights import AdapterWeights

pytestmark = pytest.mark.gpu


def make_meta(lens, widx, ranks, scalings, dev, scal_dtype=torch.float32):
    indptr = [0]
    for n in lens:
        indptr.append(indptr[-1] + n)
    return KernelInputMetaData(
        bs=len(lens), seg_lens=torch.tensor(lens, dtype=torch.int32, device=dev),
        seg_indptr=torch.tensor(indptr, dtype=torch.int32, device=dev),
        weight_indices=torch.tensor(widx, dtype=torch.int32, device=dev),
        lora_ranks=torch.tensor(ranks, dtype=torch.int32, device=dev),
        scalings=torch.tensor(scalings, dtype=scal_dtype, device=dev), max_len=max(lens))


def naive_delta(x, a_stack, b_stack, widx_rows, ranks, scalings):
    """Row-wise reference: delta[r] = scaling * x[r] @ A[:r]^T @ B[:, :r]^T (fp32)."""
    out = []
    for row, slot in enumerate(widx_rows):
        r = ranks[slot]
        if r == 0:
            out.append(torch.zeros(b_stack.shape[1], dtype=torch.float32, device=x.device))
            continue
        out.append(lora_delta(x[row:row + 1].float(), a_stack[slot].float(), b_stack[slot].float(),
                              scalings[slot], rank=r)[0])
    return torch.stack(out)


@pytest.mark.parametrize("rows_per_adapter", [2, 8])
def test_grouped_matches_rowwise_decode(cuda_dev, rows_per_adapter):
    """test_grouped_rows.py:94-134 with our kernels: grouped vs per-row metadata vs naive."""
    dev, dt = cuda_dev, torch.bfloat16
    torch.manual_seed(0)
    in_dim, out_dim, max_rank = 96, 256, 64
    ranks, scalings = [8, 16], [1.0, 2.0]
    a = torch.randn(2, max_rank, in_dim, device=dev, dtype=dt) * 0.1
    b = torch.randn(2, out_dim, max_rank, device=dev, dtype=dt) * 0.1
    rows = rows_per_adapter * 2
    x = torch.randn(rows, in_dim, device=dev, dtype=dt)
    widx_rows = [0] * rows_per_adapter + [1] * rows_per_adapter
    base = torch.randn(rows, out_dim, device=dev, dtype=dt)
    outs = {}
    for tag, meta in (("group", make_meta([rows_per_adapter] * 2, [0, 1], ranks, scalings, dev)),
                      ("row", make_meta([1] * rows, widx_rows, ranks, scalings, dev))):
        be = CudaLoRABackend()
        be.set_kernel_input_metadata(meta)
        mid = torch.zeros(rows, max_rank, device=dev, dtype=dt)
        be._mid = mid
        mid = be.run_lora_a_sgemm(x, a)
        y = be.run_lora_b_sgemm(mid, b, base_output=base.clone())
        outs[tag] = (mid, y)
        be.check_routing()
    for tag in ("group", "row"):
        for row, slot in enumerate(widx_rows):
            assert (outs[tag][0][row, ranks[slot]:] == 0).all()
    ref = base.float() + naive_delta(x, a, b, widx_rows, ranks, scalings)
    torch.testing.assert_close(outs["group"][1], outs["row"][1], rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(outs["group"][1].float(), ref, rtol=2e-2, atol=2e-2)


def test_grouped_matches_rowwise_prefill(cuda_dev):
    dev, dt = cuda_dev, torch.bfloat16
    torch.manual_seed(1)
    in_dim, out_dim, max_rank = 96, 256, 64
    ranks, scalings = [8, 16], [1.0, 2.0]
    a = torch.randn(2, max_rank, in_dim, device=dev, dtype=dt) * 0.1
    b = torch.randn(2, out_dim, max_rank, device=dev, dtype=dt) * 0.1
    x = torch.randn(16, in_dim, device=dev, dtype=dt)
    base = torch.randn(16, out_dim, device=dev, dtype=dt)
    outs = []
    for meta in (make_meta([10, 6], [0, 1], ranks, scalings, dev),
                 make_meta([5, 5, 3, 3], [0, 0, 1, 1], ranks, scalings, dev)):
        be = get_lora_backend("cuda")
        be.set_kernel_input_metadata(meta)
        outs.append(be.apply_lora(x, a, b, base.clone()))
    torch.testing.assert_close(outs[0], outs[1], rtol=2e-2, atol=2e-2)


def test_strided_base_output_slice(cuda_dev):
    """y is a column slice of a fused qkv output (row stride 6144 != out)."""
    dev, dt = cuda_dev, torch.bfloat16
    torch.manual_seed(2)
    qkv = torch.randn(8, 6144, device=dev, dtype=dt)
    before = qkv.clone()
    y = qkv[:, 4096:5120]
    a = torch.randn(3, 16, 512, device=dev, dtype=dt) * 0.05
    b = torch.randn(3, 1024, 16, device=dev, dtype=dt) * 0.05
    x = torch.randn(8, 512, device=dev, dtype=dt)
    widx = [0, 1, 2, 0, 1, 2, 0, 1]
    be = CudaLoRABackend()
    be.set_kernel_input_metadata(make_meta([1] * 8, widx, [16, 16, 16], [1.0, 2.0, 0.5], dev))
    out = be.apply_lora(x, a, b, y)
    assert out.data_ptr() == y.data_ptr()
    ref = before[:, 4096:5120].float() + naive_delta(x, a, b, widx, [16] * 3, [1.0, 2.0, 0.5])
    torch.testing.assert_close(qkv[:, 4096:5120].float(), ref, rtol=2e-2, atol=2e-2)
    assert torch.equal(qkv[:, :4096], before[:, :4096]) and torch.equal(qkv[:, 5120:], before[:, 5120:])


def test_backend_errors(cuda_dev):
    be = CudaLoRABackend()
    with pytest.raises(RuntimeError):
        be.run_lora_a_sgemm(torch.randn(2, 8, device=cuda_dev), torch.randn(1, 4, 8, device=cuda_dev))
    be.set_kernel_input_metadata(make_meta([1], [0], [4], [1.0], cuda_dev))
    with pytest.raises(RuntimeError):
        be.run_lora_a_sgemm(torch.randn(2, 8), torch.randn(1, 4, 8))
    with pytest.raises(ValueError):
        be.run_lora_a_sgemm(torch.randn(2, 2, 8, device=cuda_dev), torch.randn(1, 4, 8, device=cuda_dev))
    with pytest.raises(ValueError):
        get_lora_backend("torch")
    # out-of-range slot is reported by check_routing
    be.set_kernel_input_metadata(make_meta([1], [3], [4], [1.0], cuda_dev))
    be.run_lora_a_sgemm(torch.randn(1, 8, device=cuda_dev), torch.randn(1, 4, 8, device=cuda_dev))
    with pytest.raises(RuntimeError, match="weight_indices"):
        be.check_routing()


class ToyLM(nn.Module):
    def __init__(self, n_in=16, n_out=32):
        super().__init__()
        self.lin = nn.Linear(n_in, n_out, bias=True)

    def forward(self, x):
        return self.lin(x)


def _adapters(n_in, n_out, rank, names, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return {n: AdapterWeights(rank=rank, scaling=2.0 / (i + 1),
                              modules={"lin": (torch.randn(rank, n_in, generator=g).to(dtype),
                                               (torch.randn(n_out, rank, generator=g) * 0.1).to(dtype))})
            for i, n in enumerate(names)}


@pytest.mark.parametrize("dtype, tol", [(torch.float32, (1e-4, 1e-5)), (torch.bfloat16, (1e-2, 2e-2))])
def test_manager_forward_matches_row_reference(cuda_dev, dtype, tol):
    """test_phase4_backend.py:71-82: forward_with_lora vs base + per-row lora_delta."""
    model = ToyLM().to(cuda_dev, dtype)
    wrappers = wrap_linear_modules(model, ["lin"])
    mgr = MultiLoRAManager(wrappers, device=cuda_dev, dtype=dtype, max_loras_per_batch=3, max_lora_rank=8)
    ads = _adapters(16, 32, 4, ["a", "b"], dtype=dtype)
    ref_ads = _adapters(16, 32, 4, ["a", "b"], dtype=dtype)  # the pool releases the host tensors
    for n, w in ads.items():
        mgr.register_adapter(n, w)
    x = torch.randn(3, 16, device=cuda_dev, dtype=dtype)
    names = ["a", None, "b"]
    y = mgr.forward_with_lora(model, x=x, lora_names=names, seq_lens=[1, 1, 1])
    base = wrappers["lin"].base_layer(x)
    ref = base.clone().float()
    for i, n in enumerate(names):
        if n is None:
            continue
        a, b = ref_ads[n].modules["lin"]
        ref[i] += lora_delta(x[i:i + 1].float(), a.to(cuda_dev).float(), b.to(cuda_dev).float(),
                             ref_ads[n].scaling, rank=4)[0]
    torch.testing.assert_close(y.float(), ref, rtol=tol[0], atol=tol[1])
    y2 = mgr.forward_with_lora(model, x=x, lora_names=names, seq_lens=[1, 1, 1])
    torch.testing.assert_close(y, y2)
    meta = mgr._resident_meta
    assert meta.bs == 3 and meta.lora_ranks.shape[0] == 3 and meta.seg_indptr[:4].tolist() == [0, 1, 2, 3]
    set_lora_enabled(False)
    try:
        torch.testing.assert_close(model(x), base)
    finally:
        set_lora_enabled(True)


def test_manager_grouped_rows_metadata(cuda_dev):
    model = ToyLM(64, 128).to(cuda_dev)
    wrappers = wrap_linear_modules(model, ["lin"])
    mgr = MultiLoRAManager(wrappers, device=cuda_dev, dtype=torch.float32, max_loras_per_batch=3, max_lora_rank=16)
    for n, w in _adapters(64, 128, 8, ["a", "b"], seed=3).items():
        mgr.register_adapter(n, w)
    x = torch.randn(4, 5, 64, device=cuda_dev)
    mgr.forward_with_lora(model, x=x, lora_names=["a", "a", "b", "b"], seq_lens=[5] * 4)
    assert mgr._resident_meta.bs == 2 and mgr._resident_meta.max_len == 10
    mgr.forward_with_lora(model, x=x, lora_names=["a", "b", "a", "b"], seq_lens=[5] * 4)
    assert mgr._resident_meta.bs == 4 and mgr._resident_meta.max_len == 5


def test_fused_qkv_with_lora(cuda_dev):
    """test_fused_qkv.py:84-103 on the GPU: fused base GEMM + per-slice deltas == separate."""
    torch.manual_seed(0)
    prefix = "model.layers.0.self_attn."
    dims = {"q_proj": 32, "k_proj": 8, "v_proj": 8}
    wr = {prefix + n: LinearWithLoRA(nn.Linear(16, d, bias=False).to(cuda_dev)) for n, d in dims.items()}
    be = CudaLoRABackend()
    be.set_kernel_input_metadata(make_meta([1, 1], [0, 1], [4, 4], [1.0, 1.0], cuda_dev))
    for n, d in dims.items():
        wr[prefix + n].set_lora_info(be, torch.randn(2, 4, 16, device=cuda_dev),
                                     torch.randn(2, d, 4, device=cuda_dev) * 0.1)
    x = torch.randn(2, 1, 16, device=cuda_dev)
    order = [prefix + n for n in dims]
    ref = [wr[k](x).clone() for k in order]
    assert fuse_qkv_projections(wr) == 1
    got = [wr[k](x) for k in order]
    for g, r in zip(got, ref):
        assert (g - r).abs().max().item() < 1e-5


def test_cuda_graph_capture_and_replay(cuda_dev):
    """Captured apply_lora replays the same numbers; resident tensors keep their addresses."""
    dev, dt = cuda_dev, torch.bfloat16
    torch.manual_seed(4)
    a = torch.randn(4, 16, 1024, device=dev, dtype=dt) * 0.03
    b = torch.randn(4, 2048, 16, device=dev, dtype=dt) * 0.05
    x = torch.randn(16, 1024, device=dev, dtype=dt)
    y0 = torch.randn(16, 2048, device=dev, dtype=dt)
    be = CudaLoRABackend()
    widx = [i % 4 for i in range(16)]
    be.set_kernel_input_metadata(make_meta([1] * 16, widx, [16, 8, 0, 16], [1.0, 2.0, 0.0, 0.5], dev))
    y = y0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            y.copy_(y0)
            be.apply_lora(x, a, b, y)
    torch.cuda.current_stream().wait_stream(s)
    direct = y.clone()
    mid_ptr = be._mid.data_ptr()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y.copy_(y0)
        be.apply_lora(x, a, b, y)
    assert be._mid.data_ptr() == mid_ptr
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, direct)
    # new routing written in place is picked up by the same graph
    meta = be.kernel_input_metadata
    meta.weight_indices.copy_(torch.tensor([3 - w for w in widx], dtype=torch.int32, device=dev))
    g.replay()
    torch.cuda.synchronize()
    ref = y0.float() + naive_delta(x, a, b, [3 - w for w in widx], [16, 8, 0, 16], [1.0, 2.0, 0.0, 0.5])
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
