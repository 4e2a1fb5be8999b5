"""Tensor-parallel host logic on CPU: sharding rules and the row-parallel
all-reduce, run as two gloo ranks with an oracle-backed stand-in backend.

The product's CUDA backend implements the same ``shrink_partial`` /
``expand_partial`` / ``apply_lora`` hooks with the kernels; its NCCL version is
in test_tp_gpu.py. The invariant checked is the one the sharding must keep:
the sum over ranks of the row-parallel partial outputs equals the unsharded
result, and the column-parallel output slices concatenate to it.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from multi_lora_b200.tensor_parallel import (COLUMN, LLAMA_TP_KIND, ROW, column_parallel_apply, row_parallel_apply,
                                             shard_bounds, shard_lora_stacks)
from oracle import lora_oracle as orc


class OracleTPBackend:
    """CPU stand-in with the tensor-parallel hooks of the CUDA backend,
    computed by the oracle (test infrastructure only)."""

    def __init__(self, indptr, widx, ranks, scalings, bs, dtype):
        self.indptr, self.widx, self.ranks, self.scalings, self.bs = indptr, widx, ranks, scalings, bs
        self.dtype = dtype

    def shrink_partial(self, x, a_shard):
        part = orc.shrink(x.numpy(), a_shard.numpy(), self.indptr, self.widx, self.ranks, self.bs, dtype="f32")
        return torch.from_numpy(part)

    def expand_partial(self, partial, b_shard, y):
        mid = orc.round_to(partial.numpy(), self.dtype)
        out = orc.expand(mid, b_shard.numpy(), self.indptr, self.widx, self.ranks, self.scalings, self.bs,
                         y.numpy(), dtype=self.dtype)
        y.copy_(torch.from_numpy(out))
        return y

    def apply_lora(self, x, a, b, y):
        mid = orc.shrink(x.numpy(), a.numpy(), self.indptr, self.widx, self.ranks, self.bs, dtype=self.dtype)
        out = orc.expand(mid, b.numpy(), self.indptr, self.widx, self.ranks, self.scalings, self.bs, y.numpy(),
                         dtype=self.dtype)
        y.copy_(torch.from_numpy(out))
        return y


def _case(dtype: str, seed: int = 0):
    """Seeded routing and weights: S rows over K slots (one rank-0 slot), R=8."""
    rng = np.random.default_rng(seed)
    S, IN, OUT, K, R = 30, 64, 48, 5, 8
    ranks = np.array([8, 4, 0, 8, 2], np.int32)
    scalings = np.array([2.0, 0.5, 0.0, 1.0, 4.0], np.float32)
    lens = [3, 1, 5, 2, 7, 4, 8]
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    widx = rng.integers(0, K, len(lens)).astype(np.int32)
    widx[2] = 2  # a base (rank-0) segment
    x = orc.round_to(rng.standard_normal((S, IN)).astype(np.float32), dtype)
    A = orc.round_to(rng.uniform(-0.125, 0.125, (K, R, IN)).astype(np.float32), dtype)
    B = orc.round_to((rng.standard_normal((K, OUT, R)) * 0.02).astype(np.float32), dtype)
    y = orc.round_to(rng.standard_normal((S, OUT)).astype(np.float32), dtype)
    return dict(x=x, A=A, B=B, y=y, indptr=indptr, widx=widx, ranks=ranks, scalings=scalings, bs=len(lens))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, dtype: str, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _case(dtype)
        be = OracleTPBackend(c["indptr"], c["widx"], c["ranks"], c["scalings"], c["bs"], dtype)
        x, A, B = torch.from_numpy(c["x"]), torch.from_numpy(c["A"]), torch.from_numpy(c["B"])
        # row-parallel: every rank holds its own base partial of y
        rng = np.random.default_rng(100 + rank)
        y_part = torch.from_numpy(orc.round_to(rng.standard_normal(c["y"].shape).astype(np.float32), dtype))
        base_part = y_part.clone()
        a_s, b_s = shard_lora_stacks(A, B, ROW, rank, world)
        ilo, ihi = shard_bounds(x.shape[1], rank, world)
        row_parallel_apply(be, x[:, ilo:ihi].contiguous(), a_s, b_s, y_part, rank, world)
        delta = y_part - base_part
        dist.all_reduce(delta)
        # column-parallel: the rank's output slice of y
        a_c, b_c = shard_lora_stacks(A, B, COLUMN, rank, world)
        lo, hi = shard_bounds(B.shape[1], rank, world)
        y_loc = torch.from_numpy(c["y"][:, lo:hi].copy())
        column_parallel_apply(be, x, a_c, b_c, y_loc)
        slices = [torch.empty_like(y_loc) for _ in range(world)]
        dist.all_gather(slices, y_loc)
        if rank == 0:
            q.put((delta.numpy(), torch.cat(slices, dim=1).numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_tp_two_gloo_ranks_match_unsharded(dtype):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, dtype, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        delta, col = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    c = _case(dtype)
    # row-parallel: the summed deltas equal the fp32 reference delta
    ref = orc.apply_lora_fp32(c["x"], c["A"], c["B"], c["indptr"], c["widx"], c["ranks"], c["scalings"], c["bs"],
                              np.zeros_like(c["y"]))
    tol = dict(atol=1e-5, rtol=1e-5) if dtype == "f32" else dict(atol=2e-2, rtol=1e-2)
    np.testing.assert_allclose(delta, ref, **tol)
    # column-parallel: slices concatenate to the unsharded result, bit for bit
    mid = orc.shrink(c["x"], c["A"], c["indptr"], c["widx"], c["ranks"], c["bs"], dtype=dtype)
    full = orc.expand(mid, c["B"], c["indptr"], c["widx"], c["ranks"], c["scalings"], c["bs"], c["y"], dtype=dtype)
    np.testing.assert_array_equal(col, full)


def test_shard_rules():
    A = torch.arange(2 * 4 * 8, dtype=torch.float32).reshape(2, 4, 8)
    B = torch.arange(2 * 6 * 4, dtype=torch.float32).reshape(2, 6, 4)
    a, b = shard_lora_stacks(A, B, COLUMN, 1, 2)
    assert a is A and torch.equal(b, B[:, 3:6])
    a, b = shard_lora_stacks(A, B, ROW, 1, 2)
    assert torch.equal(a, A[:, :, 4:8]) and torch.equal(b, B[:, 3:6]) and a.is_contiguous()
    assert shard_bounds(11008, 7, 8) == (9632, 11008)
    with pytest.raises(ValueError):
        shard_bounds(10, 0, 4)
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)
    with pytest.raises(ValueError):
        shard_lora_stacks(A, B, "diagonal", 0, 2)
    assert {k for k, v in LLAMA_TP_KIND.items() if v == ROW} == {"o_proj", "down_proj"}


def test_row_parallel_rejects_mismatched_shard():
    c = _case("f32")
    be = OracleTPBackend(c["indptr"], c["widx"], c["ranks"], c["scalings"], c["bs"], "f32")
    x, A, B = torch.from_numpy(c["x"]), torch.from_numpy(c["A"]), torch.from_numpy(c["B"])
    y = torch.zeros(30, 48)
    with pytest.raises(ValueError):
        row_parallel_apply(be, x, A, B[:, :10], y, 0, 2)  # B slice of the wrong width
