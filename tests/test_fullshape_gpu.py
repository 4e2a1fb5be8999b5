"""Parity at the full shapes the bench runs (BASELINE configs 3 and 5), against the oracle.

* cfg3 (Llama-3-8B prefill, tensor-core pair): gate/up 4096->14336 and down
  14336->4096 at rank 64, 8 adapters, the seed-0 request lengths
  [469, 845, 454, 989, 348, 314, 495, 426] (4340 rows);
* cfg5 (Llama-3-70B decode, streaming pair): q 8192->8192, gate/up
  8192->28672 and down 28672->8192, 128 adapters of rank 16, 512 one-token
  segments with seeded adapter ids.

Inputs are seeded synthetic tensors of those shapes (no checkpoints exist here).
Tolerance: bf16 outputs within max-abs 2e-2 / relative 1e-2 of the
fp32-accumulated per-segment reference, as for every bf16 case.
"""

from __future__ import annotations

import pytest
import torch

from test_kernels_gpu import _case, _check_apply

pytestmark = pytest.mark.gpu

CFG3_LENS = [469, 845, 454, 989, 348, 314, 495, 426]


@pytest.mark.parametrize("n_in, n_out", [(4096, 14336), (14336, 4096)], ids=["gate_up", "down"])
def test_cfg3_tensor_core_full_shapes(cuda_dev, n_in, n_out):
    c = _case(301 + n_in % 97, torch.bfloat16, n_in, n_out, 64, [64] * 8, CFG3_LENS, cuda_dev, nan_tails=False)
    c["widx"] = list(range(8))  # one adapter per request, as the cfg3 workload routes them
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=4)


@pytest.mark.parametrize("n_in, n_out", [(8192, 8192), (8192, 28672), (28672, 8192)], ids=["q", "gate_up", "down"])
def test_cfg5_streaming_full_shapes(cuda_dev, n_in, n_out):
    c = _case(501 + n_out % 89, torch.bfloat16, n_in, n_out, 16, [16] * 128, [1] * 512, cuda_dev, nan_tails=False)
    _check_apply(c, cuda_dev, torch.bfloat16, expect_path=3)
