"""Tensor-parallel LoRA on the GPU through the CUDA backend.

* one GPU: TP ranks emulated in one process (the all-reduce is a sum of the
  ranks' fp32 partials), checked against the oracle's fp32 delta and, for
  column-parallel projections, against the unsharded kernel;
* two or more GPUs: one process per GPU over NCCL through
  ``row_parallel_apply`` (skipped when the box has one GPU), with the
  partials summed by an NCCL all-reduce and by the peer-memory exchange;
* the peer-memory exchange with 2, 4 and 8 ranks emulated on one GPU (every
  rank's shrink-and-publish phase, then every rank's wait-and-expand phase, so
  no kernel waits for one queued after it), repeated calls, inside a CUDA
  graph, one rank's single-launch call between the others' two phases, and
  the bounded wait running out on partials that no rank writes; each on the
  fused decode kernel and on the streaming pair.

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

from multi_lora_b200 import _native
from multi_lora_b200.backend import CudaLoRABackend
from multi_lora_b200.batch_info import KernelInputMetaData
from multi_lora_b200.tensor_parallel import (COLUMN, ROW, PeerExchange, row_parallel_apply, row_parallel_apply_p2p,
                                             shard_bounds, shard_lora_stacks)
from oracle import lora_oracle as orc

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-2, rtol=1e-2)
PATHS = {"fused": 1, "stream": 3}  # mlora_last_apply_path codes of the exchange's two kernels


class forced_path:
    """Force the apply path tried first (mlora_set_apply_path) inside a with-block."""

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        self.old = _native.get_apply_path()
        _native.set_apply_path(self.name)

    def __exit__(self, *exc):
        _native.set_apply_path(self.old)


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


def _p2p_setup(dev, tp, c):
    meta = _meta(c, dev)
    bes = []
    for _ in range(tp):
        be = CudaLoRABackend()
        be.set_kernel_input_metadata(meta)
        bes.append(be)
    x, A, B = c["x"].to(dev), c["A"].to(dev), c["B"].to(dev)
    ranks = []
    for p in range(tp):
        a_s, b_s = shard_lora_stacks(A, B, ROW, p, tp)
        ilo, ihi = shard_bounds(x.shape[1], p, tp)
        lo, hi = shard_bounds(B.shape[1], p, tp)
        ranks.append((x[:, ilo:ihi].contiguous(), a_s, b_s, lo, hi))
    return bes, ranks


def _p2p_call(bes, ranks, xs, y_parts, path=None):
    """All ranks' shrink-and-publish phase, then all ranks' wait-and-expand phase."""
    for phase in (1, 2):
        for p, (xp, a_s, b_s, lo, hi) in enumerate(ranks):
            row_parallel_apply_p2p(bes[p], xp, a_s, b_s, y_parts[p][:, lo:hi], xs[p], phase=phase)
            if path is not None:
                assert _native.capi().mlora_last_apply_path() == PATHS[path]


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_p2p_exchange_emulated_one_gpu(cuda_dev, tp, path):
    """Sum over ranks of the pre-all-reduce outputs = the unsharded delta; three
    calls in a row (epochs 1..3, both halves of the double-buffered partials)."""
    dev = cuda_dev
    c = _case(seed=5)
    bes, ranks = _p2p_setup(dev, tp, c)
    xs = PeerExchange.local_group(tp, device=dev, max_rows=64, max_rank=16)
    ref = torch.from_numpy(_ref_delta(c))
    try:
        for _ in range(3):
            y_parts = [torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev) for _ in range(tp)]
            with forced_path(path):
                _p2p_call(bes, ranks, xs, y_parts, path)
            torch.cuda.synchronize()
            for p, (_, _, _, lo, hi) in enumerate(ranks):  # each rank wrote only its columns
                assert (y_parts[p][:, :lo] == 0).all() and (y_parts[p][:, hi:] == 0).all()
            delta = torch.stack([y.float() for y in y_parts]).sum(0).cpu()
            torch.testing.assert_close(delta, ref, **TOL)
        for be in bes:
            be.check_routing()
    finally:
        xs[0].close()


@pytest.mark.parametrize("path", sorted(PATHS))
def test_p2p_exchange_in_cuda_graph(cuda_dev, path):
    """The exchange captured once and replayed: the epoch advances on the device."""
    dev = cuda_dev
    c = _case(seed=6)
    tp = 2
    bes, ranks = _p2p_setup(dev, tp, c)
    xs = PeerExchange.local_group(tp, device=dev, max_rows=64, max_rank=16)
    ref = torch.from_numpy(_ref_delta(c))
    y_parts = [torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev) for _ in range(tp)]
    try:
        with forced_path(path):
            _p2p_call(bes, ranks, xs, y_parts, path)  # eager once (epoch 1)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for y in y_parts:
                    y.zero_()
                _p2p_call(bes, ranks, xs, y_parts)
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            delta = torch.stack([y.float() for y in y_parts]).sum(0).cpu()
            torch.testing.assert_close(delta, ref, **TOL)
        for be in bes:
            be.check_routing()
        del g
    finally:
        xs[0].close()


@pytest.mark.parametrize("path", sorted(PATHS))
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_p2p_single_launch_between_phases(cuda_dev, tp, path):
    """Rank 0 runs the whole call in one go (phase 0: publish, wait, expand)
    after every other rank published and before they expand, so its waits
    find every partial already there; two calls in a row."""
    dev = cuda_dev
    c = _case(seed=8)
    bes, ranks = _p2p_setup(dev, tp, c)
    xs = PeerExchange.local_group(tp, device=dev, max_rows=64, max_rank=16)
    ref = torch.from_numpy(_ref_delta(c))
    try:
        for _ in range(2):
            y_parts = [torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev) for _ in range(tp)]
            with forced_path(path):
                for phase, who in ((1, range(1, tp)), (0, [0]), (2, range(1, tp))):
                    for p in who:
                        xp, a_s, b_s, lo, hi = ranks[p]
                        row_parallel_apply_p2p(bes[p], xp, a_s, b_s, y_parts[p][:, lo:hi], xs[p], phase=phase)
                        assert _native.capi().mlora_last_apply_path() == PATHS[path]
            torch.cuda.synchronize()
            delta = torch.stack([y.float() for y in y_parts]).sum(0).cpu()
            torch.testing.assert_close(delta, ref, **TOL)
        for be in bes:
            be.check_routing()
    finally:
        xs[0].close()


def test_p2p_fused_declines_grids_over_one_wave(cuda_dev):
    """The fused exchange kernel's CTAs wait on other ranks' CTAs, so it runs
    only when its whole grid is resident at once. With 512 slots (at least
    1024 CTAs, while the exchange instance's register cap leaves at most 4
    CTAs on each of 148 SMs) it declines and the streaming pair runs the
    call, even when the fused path is forced."""
    dev = cuda_dev
    c = _case(seed=9, K=512)
    tp = 2
    bes, ranks = _p2p_setup(dev, tp, c)
    xs = PeerExchange.local_group(tp, device=dev, max_rows=64, max_rank=16)
    ref = torch.from_numpy(_ref_delta(c))
    try:
        y_parts = [torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev) for _ in range(tp)]
        with forced_path("fused"):
            _p2p_call(bes, ranks, xs, y_parts, "stream")
        torch.cuda.synchronize()
        delta = torch.stack([y.float() for y in y_parts]).sum(0).cpu()
        torch.testing.assert_close(delta, ref, **TOL)
        for be in bes:
            be.check_routing()
    finally:
        xs[0].close()


@pytest.mark.parametrize("path", sorted(PATHS))
def test_p2p_exchange_wait_times_out_and_reports(cuda_dev, path):
    """A rank whose peer never publishes: its bounded polls run out (about 2 s),
    the status word carries the timeout bit, the tile is skipped, the context
    stays usable."""
    dev = cuda_dev
    c = _case(seed=7)
    bes, ranks = _p2p_setup(dev, 2, c)
    xs = PeerExchange.local_group(2, device=dev, max_rows=64, max_rank=16)
    try:
        y = torch.zeros(c["y"].shape, dtype=torch.bfloat16, device=dev)
        xp, a_s, b_s, lo, hi = ranks[0]
        with forced_path(path):
            row_parallel_apply_p2p(bes[0], xp, a_s, b_s, y[:, lo:hi], xs[0], phase=1)
            row_parallel_apply_p2p(bes[0], xp, a_s, b_s, y[:, lo:hi], xs[0], phase=2)  # rank 1 never published
            assert _native.capi().mlora_last_apply_path() == PATHS[path]
        torch.cuda.synchronize()
        assert int(bes[0].status_word(dev).item()) & 0x10
        assert (y == 0).all()  # nothing expanded from a missing partial
        with pytest.raises(RuntimeError, match="did not complete in time"):
            bes[0].check_routing()
        z = torch.ones(4, device=dev) * 2  # the context still runs work
        assert float(z.sum()) == 8.0
    finally:
        xs[0].close()


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


def _nccl_worker(rank, world, port, q, exchange=None):
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
        xchg = PeerExchange.create(device=dev, max_rows=64, max_rank=16) if exchange else None
        if exchange:
            _native.set_apply_path(exchange)
        for _ in range(3):  # repeated: the resident partial buffer (or the exchange's halves) is reused
            y_part.zero_()
            row_parallel_apply(be, x[:, ilo:ihi].contiguous(), a_s, b_s, y_part, rank, world, exchange=xchg)
        torch.cuda.synchronize()
        be.check_routing()
        if xchg is not None:
            dist.barrier()
            xchg.close()
        d = y_part.float()
        dist.all_reduce(d)
        torch.cuda.synchronize()
        if rank == 0:
            q.put(d.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", [None, "fused", "stream"],
                         ids=["nccl_allreduce", "peer_exchange_fused", "peer_exchange_stream"])
def test_tp_nccl_row_parallel(exchange):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    np.testing.assert_allclose(got, _ref_delta(_case()), **TOL)
