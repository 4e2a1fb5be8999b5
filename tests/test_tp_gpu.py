"""Tensor-parallel LoRA on the GPU through the CUDA backend.

* one GPU: TP ranks emulated in one process (the all-reduce is a sum of the
  ranks' fp32 partials), checked against the oracle's fp32 delta and, for
  column-parallel projections, against the unsharded kernel;
* two or more GPUs: one process per GPU over NCCL through
  ``row_parallel_apply`` (skipped when the box has one GPU).

Tolerance: bf16 within atol 2e-2 / rtol 1e-2 of the fp32-accumulated
reference (the parity bar for bf16 outputs).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from multi_lora_b200.backend import CudaLoRABackend
from multi_lora_b200.batch_info import KernelInputMetaData
from multi_lora_b200.tensor_parallel import COLUMN, ROW, row_parallel_apply, shard_bounds, shard_lora_stacks
from oracle import lora_oracle as orc

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-2, rtol=1e-2)


def _case(seed=0, S=64, IN=1024, OUT=768, K=8, R=16):
    """Decode-like routing (1-3 tokens per segment, one rank-0 slot, one rank-8 slot)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 4, (S,), generator=g).tolist()
    lens = lens[: next(i for i in range(len(lens) + 1) if sum(lens[:i]) >= S)]
    lens[-1] -= sum(lens) - S
    lens = [n for n in lens if n > 0]
    widx = torch.randint(0, K, (len(lens),), generator=g).tolist()
    ranks = [R] * K
    ranks[1], ranks[2] = 0, 8
    scalings = [2.0] * K
    x = torch.randn(S, IN, generator=g).bfloat16()
    A = ((torch.rand(K, R, IN, generator=g) * 2 - 1) / IN ** 0.5).bfloat16()
    B = (torch.randn(K, OUT, R, generator=g) * 0.02).bfloat16()
    y = torch.randn(S, OUT, generator=g).bfloat16()
    return dict(lens=lens, widx=widx, ranks=ranks, scalings=scalings, x=x, A=A, B=B, y=y)


def _meta(c, dev):
    indptr = np.concatenate([[0], np.cumsum(c["lens"])]).astype(np.int32)
    return KernelInputMetaData(
        bs=len(c["lens"]), seg_lens=torch.tensor(c["lens"], dtype=torch.int32, device=dev),
        seg_indptr=torch.from_numpy(indptr).to(dev), weight_indices=torch.tensor(c["widx"], dtype=torch.int32,
                                                                                 device=dev),
        lora_ranks=torch.tensor(c["ranks"], dtype=torch.int32, device=dev),
        scalings=torch.tensor(c["scalings"], dtype=torch.bfloat16, device=dev), max_len=max(c["lens"]))


def _ref_delta(c):
    indptr = np.concatenate([[0], np.cumsum(c["lens"])])
    f = lambda t: t.float().numpy()
    return orc.apply_lora_fp32(f(c["x"]), f(c["A"]), f(c["B"]), indptr, c["widx"], c["ranks"],
                               np.array(c["scalings"], np.float32), len(c["lens"]), np.zeros(tuple(c["y"].shape),
                                                                                            np.float32))


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_emulated_one_gpu(cuda_dev, tp):
    dev = cuda_dev
    c = _case()
    be = CudaLoRABackend()
    be.set_kernel_input_metadata(_meta(c, dev))
    x, A, B = c["x"].to(dev), c["A"].to(dev), c["B"].to(dev)
    ref = torch.from_numpy(_ref_delta(c))
    # row-parallel: partials per rank, summed as the all-reduce would
    partials, shards = [], []
    for p in range(tp):
        a_s, b_s = shard_lora_stacks(A, B, ROW, p, tp)
        ilo, ihi = shard_bounds(x.shape[1], p, tp)
        partials.append(be.shrink_partial(x[:, ilo:ihi].contiguous(), a_s).clone())
        shards.append(b_s)
    total = torch.stack(partials).sum(0)
    delta = torch.zeros(c["y"].shape, dtype=torch.float32)
    for p in range(tp):
        y_part = torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev)
        lo, hi = shard_bounds(y_part.shape[1], p, tp)
        be.expand_partial(total, shards[p], y_part[:, lo:hi])
        assert (y_part[:, :lo] == 0).all() and (y_part[:, hi:] == 0).all()
        delta += y_part.float().cpu()
    be.check_routing()
    torch.testing.assert_close(delta, ref, **TOL)
    # column-parallel: slices of the unsharded result
    y_full = c["y"].to(dev).clone()
    be.apply_lora(x, A, B, y_full)
    for p in range(tp):
        a_c, b_c = shard_lora_stacks(A, B, COLUMN, p, tp)
        lo, hi = shard_bounds(B.shape[1], p, tp)
        y_loc = c["y"][:, lo:hi].to(dev).contiguous()
        be.apply_lora(x, a_c, b_c, y_loc)
        torch.testing.assert_close(y_loc.float(), y_full[:, lo:hi].float(), **TOL)
        torch.testing.assert_close(y_loc.float().cpu(), (c["y"][:, lo:hi].float() + ref[:, lo:hi]), **TOL)
    be.check_routing()


def test_shrink_partial_zero_outside_adapter_columns(cuda_dev):
    """fp32 partials are zero past each slot's rank and on base (rank-0) rows,
    so the all-reduce adds nothing stale."""
    dev = cuda_dev
    c = _case(seed=3)
    be = CudaLoRABackend()
    be.set_kernel_input_metadata(_meta(c, dev))
    be.partial_buffer(64, 16, c["x"].to(dev)).fill_(7.0)  # stale contents
    part = be.shrink_partial(c["x"].to(dev), c["A"].to(dev)).cpu()
    row = 0
    for n, w in zip(c["lens"], c["widx"]):
        r = c["ranks"][w]
        assert (part[row:row + n, r:] == 0).all()
        row += n


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        c = _case()
        be = CudaLoRABackend()
        be.set_kernel_input_metadata(_meta(c, dev))
        x, A, B = c["x"].to(dev), c["A"].to(dev), c["B"].to(dev)
        a_s, b_s = shard_lora_stacks(A, B, ROW, rank, world)
        ilo, ihi = shard_bounds(x.shape[1], rank, world)
        y_part = torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev)
        for _ in range(2):  # twice: the resident partial buffer is reused
            y_part.zero_()
            row_parallel_apply(be, x[:, ilo:ihi].contiguous(), a_s, b_s, y_part, rank, world)
        be.check_routing()
        d = y_part.float()
        dist.all_reduce(d)
        torch.cuda.synchronize()
        if rank == 0:
            q.put(d.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_nccl_row_parallel():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    np.testing.assert_allclose(got, _ref_delta(_case()), **TOL)
