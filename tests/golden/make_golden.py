"""Generate the golden fixtures in this directory by running the REFERENCE's own code.

Runs only where a checkout of the reference project is available; point
MLORA_REFERENCE at its root. The fixtures are committed; tests never import
the reference.

What produces each fixture (paths within the reference project):
* toy_f32.npz        — cfg1: backend/torch_backend.py
                       TorchLoRABackend.apply_lora, plus the Triton GEMM-path
                       kernels kernels/sgemm_lora_a.py / sgemm_lora_b.py run by
                       Triton's CPU interpreter, plus layers.lora_delta rows.
* decode_f32.npz     — the Triton GEMV path (max_len == 1), interpreter, fp32.
* torch_bf16.npz     — TorchLoRABackend in bf16 on the CPU (prefill and decode
                       routing, a rank-0 slot, mixed ranks). (The interpreter
                       does not execute the bf16 sgemm kernels correctly, so
                       bf16 goldens come from the Torch backend.)
* rmsnorm.npz        — kernels/rmsnorm.py rmsnorm_fwd under the interpreter
                       (fp32, bf16, a non-contiguous two-level-stride input).
* metadata.json      — batch_info.write_kernel_input_metadata over a sequence
                       of batches (in-place refresh and capacity growth).
* group_rows.json    — batch_info.group_rows.
* pool.json, pool_slots.npz — pool.LoRAMemoryPool on the CPU (LRU and FIFO):
                       residency, evictions, batch info and slot contents.

    MLORA_REFERENCE=<reference checkout> python tests/golden/make_golden.py
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("MLORA_REFERENCE"):
    sys.exit("set MLORA_REFERENCE to the root of a reference checkout")
REF = Path(os.environ["MLORA_REFERENCE"])

if os.environ.get("PYTHONHASHSEED") != "0" or os.environ.get("TRITON_INTERPRET") != "1":
    env = dict(os.environ, PYTHONHASHSEED="0", TRITON_INTERPRET="1")
    sys.exit(subprocess.call([sys.executable, __file__, *sys.argv[1:]], env=env))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# the reference's pool/weights import peft names only; a stub is enough
_peft = types.ModuleType("peft")
_peft.PeftModel = type("PeftModel", (), {})
_tuners = types.ModuleType("peft.tuners")
_lora = types.ModuleType("peft.tuners.lora")
_lora.LoraLayer = type("LoraLayer", (), {})
sys.modules.update({"peft": _peft, "peft.tuners": _tuners, "peft.tuners.lora": _lora})
sys.path.insert(0, str(REF))

from multi_lora.backend.torch_backend import TorchLoRABackend  # noqa: E402
from multi_lora.batch_info import (  # noqa: E402
    BatchLoRAInfo,
    KernelInputMetaData,
    empty_kernel_input_metadata,
    group_rows,
    write_kernel_input_metadata,
)
from multi_lora.kernels.rmsnorm import rmsnorm_fwd  # noqa: E402
from multi_lora.kernels.sgemm_lora_a import sgemm_lora_a_fwd  # noqa: E402
from multi_lora.kernels.sgemm_lora_b import sgemm_lora_b_fwd  # noqa: E402
from multi_lora.layers import lora_delta  # noqa: E402
from multi_lora.pool import LoRAMemoryPool  # noqa: E402
from multi_lora.weights import AdapterWeights  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 storage."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_meta(lens, widx, ranks, scalings, scal_dtype=torch.float32) -> KernelInputMetaData:
    indptr = [0]
    for n in lens:
        indptr.append(indptr[-1] + n)
    return KernelInputMetaData(
        bs=len(lens),
        seg_lens=torch.tensor(lens, dtype=torch.int32),
        seg_indptr=torch.tensor(indptr, dtype=torch.int32),
        weight_indices=torch.tensor(widx, dtype=torch.int32),
        lora_ranks=torch.tensor(ranks, dtype=torch.int32),
        scalings=torch.tensor(scalings, dtype=scal_dtype),
        max_len=max(lens),
    )


def meta_arrays(m: KernelInputMetaData) -> dict:
    return {
        "seg_lens": m.seg_lens.numpy(), "seg_indptr": m.seg_indptr.numpy(),
        "weight_indices": m.weight_indices.numpy(), "lora_ranks": m.lora_ranks.numpy(),
        "scalings": m.scalings.float().numpy(), "bs": np.int32(m.bs), "max_len": np.int32(m.max_len),
    }


def torch_apply(meta, x, A, B, y):
    be = TorchLoRABackend()
    be.set_kernel_input_metadata(meta)
    mid = be.run_lora_a_sgemm(x, A)
    out = be.run_lora_b_sgemm(mid, B, base_output=y.clone())
    return mid, out


def toy_f32() -> None:
    """cfg1: in=out=256 fp32, 4 adapters r=8 alpha=16, lens [1,3,5,2,7,4], ids ~ U{0..3}."""
    g = torch.Generator().manual_seed(0)
    lens = [1, 3, 5, 2, 7, 4]
    S, n_in, n_out, K, r = sum(lens), 256, 256, 4, 8
    widx = torch.randint(0, K, (len(lens),), generator=g).tolist()
    x = torch.randn(S, n_in, generator=g)
    A = (torch.rand(K, r, n_in, generator=g) * 2 - 1) / 16.0  # U(+-1/sqrt(256))
    B = torch.randn(K, n_out, r, generator=g) * 0.02
    y = torch.randn(S, n_out, generator=g)
    ranks, scal = [r] * K, [16 / r] * K
    meta = make_meta(lens, widx, ranks, scal)
    mid_t, y_t = torch_apply(meta, x, A, B, y)
    mid_k = sgemm_lora_a_fwd(x, A, meta, torch.zeros(S, r))
    y_k = sgemm_lora_b_fwd(mid_k.contiguous(), B, meta, base_output=y.clone())
    rows = []
    indptr = meta.seg_indptr.tolist()
    for seg, slot in enumerate(widx):
        for t in range(indptr[seg], indptr[seg + 1]):
            rows.append(lora_delta(x[t:t + 1], A[slot], B[slot], scal[slot], rank=r)[0])
    np.savez_compressed(
        HERE / "toy_f32.npz", x=x.numpy(), A=A.numpy(), B=B.numpy(), y=y.numpy(), **meta_arrays(meta),
        mid_torch=mid_t.numpy(), y_torch=y_t.numpy(), mid_triton=mid_k.numpy(), y_triton=y_k.numpy(),
        delta_rows=torch.stack(rows).numpy())


def decode_f32() -> None:
    """GEMV path (one token per segment), mixed ranks incl. a rank-0 slot, out % 256 != 0."""
    g = torch.Generator().manual_seed(1)
    S, n_in, n_out, K, R = 16, 192, 320, 5, 16
    ranks, scal = [16, 8, 0, 12, 4], [2.0, 0.5, 0.0, 1.0, 3.0]
    widx = torch.randint(0, K, (S,), generator=g).tolist()
    x = torch.randn(S, n_in, generator=g)
    A = torch.randn(K, R, n_in, generator=g) * 0.1
    B = torch.randn(K, n_out, R, generator=g) * 0.1
    y = torch.randn(S, n_out, generator=g)
    meta = make_meta([1] * S, widx, ranks, scal)
    mid_t, y_t = torch_apply(meta, x, A, B, y)
    mid_k = sgemm_lora_a_fwd(x, A, meta, torch.zeros(S, R))
    y_k = sgemm_lora_b_fwd(mid_k.contiguous(), B, meta, base_output=y.clone())
    np.savez_compressed(
        HERE / "decode_f32.npz", x=x.numpy(), A=A.numpy(), B=B.numpy(), y=y.numpy(), **meta_arrays(meta),
        mid_torch=mid_t.numpy(), y_torch=y_t.numpy(), mid_triton=mid_k.numpy(), y_triton=y_k.numpy())


def torch_bf16() -> None:
    """TorchLoRABackend in bf16: a prefill batch and a decode batch on one pool."""
    g = torch.Generator().manual_seed(2)
    n_in, n_out, K, R = 256, 384, 4, 16
    ranks, scal = [16, 8, 0, 12], [2.0, 1.5, 0.0, 0.75]
    A = (torch.randn(K, R, n_in, generator=g) * 0.05).bfloat16()
    B = (torch.randn(K, n_out, R, generator=g) * 0.05).bfloat16()
    out = {"A": bits(A), "B": bits(B)}
    cases = {"prefill": ([5, 1, 7, 3, 2], [0, 3, 1, 2, 0]),
             "decode": ([1] * 24, torch.randint(0, K, (24,), generator=g).tolist())}
    for name, (lens, widx) in cases.items():
        S = sum(lens)
        x = torch.randn(S, n_in, generator=g).bfloat16()
        y = torch.randn(S, n_out, generator=g).bfloat16()
        meta = make_meta(lens, widx, ranks, scal, scal_dtype=torch.bfloat16)
        mid_t, y_t = torch_apply(meta, x, A, B, y)
        out.update({f"{name}_x": bits(x), f"{name}_y": bits(y), f"{name}_mid": bits(mid_t),
                    f"{name}_out": bits(y_t)})
        out.update({f"{name}_{k}": v for k, v in meta_arrays(meta).items()})
    np.savez_compressed(HERE / "torch_bf16.npz", **out)


def rmsnorm_cases() -> None:
    g = torch.Generator().manual_seed(3)
    out = {}
    x = torch.randn(6, 256, generator=g)
    w = torch.randn(256, generator=g)
    out.update(f32_x=x.numpy(), f32_w=w.numpy(), f32_y=rmsnorm_fwd(x, w, 1e-6).numpy())
    x = torch.randn(8, 128, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(128, generator=g)).bfloat16()
    out.update(bf16_x=bits(x), bf16_w=bits(w), bf16_y=bits(rmsnorm_fwd(x, w, 1e-6)))
    x = torch.randn(3, 2560, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(2560, generator=g)).bfloat16()
    out.update(wide_x=bits(x), wide_w=bits(w), wide_y=bits(rmsnorm_fwd(x, w, 1e-6)))
    # q slice of a fused qkv output: [B, S, 384] -> [..., :256] viewed [B, S, 2, 128]
    qkv = torch.randn(2, 3, 384, generator=g).bfloat16()
    sl = qkv[..., :256].view(2, 3, 2, 128)
    w = (1 + 0.1 * torch.randn(128, generator=g)).bfloat16()
    out.update(slice_qkv=bits(qkv), slice_w=bits(w), slice_y=bits(rmsnorm_fwd(sl, w, 1e-6)))
    np.savez_compressed(HERE / "rmsnorm.npz", **out)


def metadata_seq() -> None:
    dev, dt = torch.device("cpu"), torch.bfloat16
    meta = empty_kernel_input_metadata(device=dev, dtype=dt)
    steps = [
        (BatchLoRAInfo([0, 1, 0], [8, 16, 0, 4], [2.0, 1.5, 0.0, 0.25]), []),
        (BatchLoRAInfo([2, 1], [8, 16, 0, 4], [2.0, 1.5, 0.0, 0.25]), [4, 2]),
        (BatchLoRAInfo([3, 3, 1, 0, 2], [8, 16, 0, 4], [2.0, 1.5, 0.0, 0.25]), [1, 2, 3, 4, 5]),
        (BatchLoRAInfo([1, 0], [8, 0, 0, 4], [2.0, 0.0, 0.0, 0.25]), []),
    ]
    rec = []
    for info, seq in steps:
        before = meta
        meta = write_kernel_input_metadata(meta, info, device=dev, dtype=dt, seq_lens=seq)
        rec.append({
            "weight_indices": info.weight_indices, "lora_ranks": info.lora_ranks, "scalings": info.scalings,
            "seq_lens": seq, "same_object": meta is before, "bs": meta.bs, "max_len": meta.max_len,
            "seg_lens": meta.seg_lens.tolist(), "seg_indptr": meta.seg_indptr.tolist(),
            "out_weight_indices": meta.weight_indices.tolist(), "out_lora_ranks": meta.lora_ranks.tolist(),
            "out_scalings": meta.scalings.float().tolist()})
    (HERE / "metadata.json").write_text(json.dumps(rec, indent=1))


def group_rows_cases() -> None:
    cases = [
        (["a", "b", "a", "b"], []), (["a", "a", "b", "b", "b", None, None], []),
        (["a", "a", "b"], [5, 7, 3]), ([None], []), ([], []),
        (["x", "x", "x", "y", "x", "x"], [1, 2, 3, 4, 5, 6]),
    ]
    rec = []
    for names, seq in cases:
        gn, gl = group_rows(names, seq)
        rec.append({"names": names, "seq_lens": seq, "group_names": gn, "group_lens": gl})
    (HERE / "group_rows.json").write_text(json.dumps(rec, indent=1))


MODULES = {"m1": (4, 3), "m2": (5, 3)}  # key: (out, in)


def make_weights(rank, keys, seed):
    g = torch.Generator().manual_seed(seed)
    mods = {}
    for key in keys:
        n_out, n_in = MODULES[key]
        mods[key] = (torch.randn(rank, n_in, generator=g), torch.randn(n_out, rank, generator=g))
    return AdapterWeights(rank=rank, scaling=1.0 / rank, modules=mods)


def pool_traces() -> None:
    specs = {"a": (8, ["m1", "m2"], 1), "b": (4, ["m1"], 2), "c": (8, ["m1", "m2"], 3), "d": (2, ["m2"], 4),
             "e": (6, ["m1", "m2"], 5), "f": (8, ["m2"], 6)}
    rounds = [["a", "b"], ["c", None], ["a", "d", None], ["e", "f", "a"], ["b", "c"], ["d", "e", "f"],
              ["a", None], ["c", "b", "f"]]
    traces, slots = {}, {}
    for policy in ("lru", "fifo"):
        pool = LoRAMemoryPool(max_loras_per_batch=3, max_lora_rank=8, device=torch.device("cpu"),
                              dtype=torch.float32, eviction_policy=policy)
        pool.buffers.scatter_impl = "python"
        store = {n: make_weights(r, k, s) for n, (r, k, s) in specs.items()}
        for w in store.values():
            pool.ensure_buffers(w)
        rec = []
        for i, names in enumerate(rounds):
            pool.prepare_lora_batch(set(names), weight_store=store)
            info = pool.build_batch_info(names)
            rec.append({"names": names, "name_to_slot": {str(k): v for k, v in pool.name_to_slot.items()},
                        "eviction_count": pool.eviction_policy.eviction_count,
                        "weight_indices": info.weight_indices, "lora_ranks": info.lora_ranks,
                        "scalings": info.scalings})
            for key in MODULES:
                a, b = pool.get_module_buffers(key)
                slots[f"{policy}_{i}_{key}_A"] = a.numpy().copy()
                slots[f"{policy}_{i}_{key}_B"] = b.numpy().copy()
        traces[policy] = rec
    (HERE / "pool.json").write_text(json.dumps({"specs": specs, "modules": MODULES, "rounds": rounds,
                                                "traces": traces}, indent=1))
    np.savez_compressed(HERE / "pool_slots.npz", **slots)


def main() -> None:
    torch.set_num_threads(1)
    toy_f32()
    decode_f32()
    torch_bf16()
    rmsnorm_cases()
    metadata_seq()
    group_rows_cases()
    pool_traces()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
