#!/usr/bin/env python
"""Throughput of the multi-LoRA hot path on B200.

Default workload (the metric's config): Llama-2-7B-shaped
decode — 32 layers x {q,k,v,o: 4096->4096; gate,up: 4096->11008; down:
11008->4096}, bf16, 32 resident adapters of rank 16 (alpha 32 -> scaling 2),
64 tokens (one per request) with adapter ids uniform over 32 (seed 0), fused
RMSNorm (eps 1e-6) in front of the attention and MLP projections.

One step = one forward of the hot path over the whole model: per layer two
RMSNorms and, for each of the 7 projections, shrink + expand (apply_lora)
with the fused scaling and residual add. Each layer has its own adapter
slots, so one step streams ~2.6 GB of adapter weights — far more than the
126 MB L2, so no L2 flush is needed between steps. The step is captured
once into a CUDA graph through the public API and replayed.

With N > 1 GPUs (one process per GPU under torchrun) the same workload runs
tensor-parallel over the N ranks (strong scaling: the job still processes
64 tokens per step): q/k/v/gate/up are column-parallel (A replicated, B
column-sharded, no collective); o/down are row-parallel (A row-sharded on the
input dim, fp32 [T, r] shrink partials all-reduced over NCCL, B
column-sharded into the rank's columns of the pre-all-reduce output).
``--workload cfg5`` selects the Llama-3-70B-shaped TP decode config (80
layers, hidden 8192, 128 adapters, 512 tokens) instead.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload cfg2|cfg5]

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "LoRA shrink+expand tokens/s and % HBM/TC roofline, 1/2/4/8 B200"
UNIT = "tokens/s"

EPS = 1e-6
COLUMN, ROW = "column", "row"
GROUPS = (("q", "k", "v"), ("o",), ("gate", "up"), ("down",))  # calls per layer, in dependency order


class Workload:
    """A Llama-shaped decode workload: per layer q/k/v/o/gate/up/down LoRA
    projections and two RMSNorms; ``tokens`` tokens with uniform adapter ids."""

    def __init__(self, name, desc, hidden, kv, inter, layers, tokens, adapters, rank, alpha, requests=None):
        self.name, self.desc = name, desc
        self.requests = requests  # prefill: number of requests, one adapter each, lengths drawn in routing()
        self.hidden, self.layers, self.tokens = hidden, layers, tokens
        self.adapters, self.rank, self.scaling = adapters, rank, alpha / rank
        # (name, in, out, tensor-parallel kind)
        self.projs = [("q", hidden, hidden, COLUMN), ("k", hidden, kv, COLUMN), ("v", hidden, kv, COLUMN),
                      ("o", hidden, hidden, ROW), ("gate", hidden, inter, COLUMN), ("up", hidden, inter, COLUMN),
                      ("down", inter, hidden, ROW)]
        self.inter = inter


WORKLOADS = {
    "cfg2": Workload("cfg2", "Llama-2-7B-shaped decode: 32 layers x 7 LoRA projections + 2 RMSNorm, 64 tokens, "
                             "32 adapters r16 (alpha 32), bf16", 4096, 4096, 11008, 32, 64, 32, 16, 32),
    "cfg3": Workload("cfg3", "Llama-3-8B-shaped prefill: 32 layers x 7 LoRA projections + 2 RMSNorm, 8 requests of "
                             "128..1024 tokens (seed 0: 4340 tokens), one adapter each, 8 adapters r64 (alpha 128), "
                             "bf16", 4096, 1024, 14336, 32, 4340, 8, 64, 128, requests=8),
    "cfg4": Workload("cfg4", "Heavy-tail decode with eviction: Llama-2-7B shapes, 32 layers, 256 adapters of rank "
                             "{8,16,32,64} (alpha 2r), 64-slot pool (max_rank 64, LRU), 256 tokens/step with Zipf(1.1) "
                             "adapter ids, admission (multi_lora_b200.admission): deferred tokens first, then tokens whose "
                             "adapter is resident, then the rest, while at most 64 adapters are named; the others "
                             "wait for the next step; pinned-host slot loads; RMSNorm on; bf16",
                     4096, 4096, 11008, 32, 256, 256, 64, 128),
    "cfg5": Workload("cfg5", "Llama-3-70B-shaped decode: 80 layers x 7 LoRA projections + 2 RMSNorm, 512 tokens, "
                             "128 adapters r16 (alpha 32), bf16", 8192, 1024, 28672, 80, 512, 128, 16, 32),
}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def routing(wl: Workload, seed: int = 0):
    """Adapter id per token (uniform) -> grouped segments (adjacent equal ids merge); adapter i in slot i."""
    from multi_lora_b200.batch_info import BatchLoRAInfo, group_rows

    g = torch.Generator().manual_seed(seed)
    if wl.requests:  # prefill: request i uses adapter i, lengths uniform in [128, 1024]
        req_lens = torch.randint(128, 1025, (wl.requests,), generator=g).tolist()
        ids = [i for i, n in enumerate(req_lens) for _ in range(n)]
        names, lens = list(range(wl.requests)), req_lens
        assert sum(lens) == wl.tokens, (sum(lens), wl.tokens)
    else:
        ids = torch.randint(0, wl.adapters, (wl.tokens,), generator=g).tolist()
        names, lens = group_rows(ids, [])
    info = BatchLoRAInfo(weight_indices=list(names), lora_ranks=[wl.rank] * wl.adapters,
                         scalings=[wl.scaling] * wl.adapters)
    return ids, info, lens


def shard_dims(wl: Workload, tp: int) -> dict:
    """Per projection on one TP rank: (input dim read, B rows held, y columns)."""
    dims = {}
    for name, n_in, n_out, kind in wl.projs:
        if tp == 1:
            dims[name] = (n_in, n_out, n_out)
        elif kind == COLUMN:
            dims[name] = (n_in, n_out // tp, n_out // tp)
        else:  # row-parallel: x and A sharded on in; B column-sharded into the full-width partial output
            dims[name] = (n_in // tp, n_out // tp, n_out)
    return dims


def algorithmic_bytes(wl: Workload, ids, tp: int) -> dict:
    """Bytes a perfect kernel moves per step on one rank: A rows up to the rank
    of each distinct adapter, B columns up to the rank, x once, y read and
    written once, mid written and read once (per projection)."""
    d = len(set(ids))
    T, es, r = wl.tokens, 2, wl.rank
    dims = shard_dims(wl, tp)
    lora = flops = 0
    for name, *_ in wl.projs:
        i, o, _ = dims[name]
        lora += d * r * i * es + d * r * o * es + T * i * es + 2 * T * o * es + 2 * T * r * es
        flops += 2 * T * r * (i + o)
    rms = 2 * (2 * T * wl.hidden * es + wl.hidden * es)
    return {"lora": lora * wl.layers, "rmsnorm": rms * wl.layers, "distinct_adapters": d,
            "lora_flops": flops * wl.layers}


class Layer:
    pass


def build_workload(wl: Workload, dev, tp_rank: int = 0, tp: int = 1):
    """Per-layer adapter slot stacks (this rank's shards) and activations, generated on the device."""
    g = torch.Generator(device=dev).manual_seed(1234 + 7919 * tp_rank)
    dt = torch.bfloat16
    T, K, R = wl.tokens, wl.adapters, wl.rank
    dims = shard_dims(wl, tp)
    layers = []
    for _ in range(wl.layers):
        L = Layer()
        L.A, L.B, L.y = {}, {}, {}
        for name, n_in, _, _ in wl.projs:
            i, o, ycols = dims[name]
            bound = 1.0 / math.sqrt(n_in)  # kaiming-uniform(a=sqrt(5)) of an [r, in] weight
            L.A[name] = ((torch.rand(K, R, i, generator=g, device=dev) * 2 - 1) * bound).to(dt)
            L.B[name] = (torch.randn(K, o, R, generator=g, device=dev) * 0.02).to(dt)
            L.y[name] = torch.randn(T, ycols, generator=g, device=dev).to(dt)
        H = wl.hidden
        L.h1 = torch.randn(T, H, generator=g, device=dev).to(dt)
        L.h2 = torch.randn(T, H, generator=g, device=dev).to(dt)
        L.w1 = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dt)
        L.w2 = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(dt)
        L.xn1 = torch.empty(T, H, device=dev, dtype=dt)
        L.xn2 = torch.empty(T, H, device=dev, dtype=dt)
        xo = torch.randn(T, dims["o"][0], generator=g, device=dev).to(dt)      # attention output (this rank's part)
        xd = torch.randn(T, dims["down"][0], generator=g, device=dev).to(dt)   # act(gate) * up (this rank's part)
        L.x = {"q": L.xn1, "k": L.xn1, "v": L.xn1, "o": xo, "gate": L.xn2, "up": L.xn2, "down": xd}
        layers.append(L)
    return layers


def run_step(wl: Workload, layers, be, parts=("rmsnorm", "lora"), grouped=True, tp=1, tp_rank=0, exchange=None):
    """One forward of the LoRA hot path over all layers, in the model's
    dependency order: rmsnorm -> {q,k,v} -> o -> rmsnorm -> {gate,up} -> down.

    grouped: q/k/v and gate/up (shared input) each go through one
    ``apply_lora_group`` call; otherwise one ``apply_lora`` per projection.
    tp > 1: o and down are row-parallel (``row_parallel_apply``: shrink
    partials summed over the ranks through ``exchange`` (peer memory) or an
    NCCL all-reduce, then the expand), the rest column-parallel.
    """
    from multi_lora_b200.rmsnorm import rmsnorm_out
    from multi_lora_b200.tensor_parallel import row_parallel_apply

    kinds = {name: kind for name, _, _, kind in wl.projs}
    for L in layers:
        for grp in GROUPS:
            if "rmsnorm" in parts and grp[0] in ("q", "gate"):
                rmsnorm_out(L.h1 if grp[0] == "q" else L.h2, L.w1 if grp[0] == "q" else L.w2, EPS,
                            L.xn1 if grp[0] == "q" else L.xn2)
            if "lora" not in parts:
                continue
            if tp > 1 and kinds[grp[0]] == ROW:
                for n in grp:
                    row_parallel_apply(be, L.x[n], L.A[n], L.B[n], L.y[n], tp_rank, tp, exchange=exchange)
            elif grouped and len(grp) > 1:
                be.apply_lora_group(L.x[grp[0]], [L.A[n] for n in grp], [L.B[n] for n in grp],
                                    [L.y[n] for n in grp])
            else:
                for n in grp:
                    be.apply_lora(L.x[n], L.A[n], L.B[n], L.y[n])


def tp_parity_check(wl: Workload, dev, be, tp_rank: int, tp: int, seed: int = 4242, exchange=None) -> dict:
    """One checked layer at N > 1: the tensor-parallel result equals the unsharded one.

    Every rank builds the same full-size layer (one seed), computes the
    unsharded apply_lora of each projection on its own GPU (the 1-GPU path),
    then runs the tensor-parallel path on its shards: column-parallel
    projections write their output columns (all-gathered), row-parallel ones
    add their columns of the delta into a partial output that is ybase on
    rank 0 and zero elsewhere (all-reduced, as the model's own row-parallel
    all-reduce would). Bound: max-abs 2e-2 / relative 1e-2, the bf16 bound of
    this path. Returns {"parity": "ok" | "mismatch", "max_abs_err": ...}.
    """
    import torch.distributed as dist

    from multi_lora_b200.tensor_parallel import row_parallel_apply, shard_bounds, shard_lora_stacks

    g = torch.Generator(device=dev).manual_seed(seed)
    dt = torch.bfloat16
    T, K, R = wl.tokens, wl.adapters, wl.rank
    worst, ok = 0.0, True
    for name, n_in, n_out, kind in wl.projs:
        if name not in ("q", "o", "gate", "down"):  # one projection of each shape class
            continue
        A = ((torch.rand(K, R, n_in, generator=g, device=dev) * 2 - 1) / math.sqrt(n_in)).to(dt)
        B = (torch.randn(K, n_out, R, generator=g, device=dev) * 0.02).to(dt)
        x = torch.randn(T, n_in, generator=g, device=dev).to(dt)
        ybase = torch.randn(T, n_out, generator=g, device=dev).to(dt)
        want = ybase.clone()
        be.apply_lora(x, A, B, want)
        a_sh, b_sh = shard_lora_stacks(A, B, kind, tp_rank, tp)
        lo, hi = shard_bounds(n_out, tp_rank, tp)
        if kind == COLUMN:
            y_loc = ybase[:, lo:hi].contiguous()
            be.apply_lora(x, a_sh, b_sh, y_loc)
            parts = [torch.empty_like(y_loc) for _ in range(tp)]
            dist.all_gather(parts, y_loc)
            got = torch.cat(parts, dim=1)
        else:
            ilo, ihi = shard_bounds(n_in, tp_rank, tp)
            y_part = ybase.clone() if tp_rank == 0 else torch.zeros_like(ybase)
            row_parallel_apply(be, x[:, ilo:ihi].contiguous(), a_sh, b_sh, y_part, tp_rank, tp, exchange=exchange)
            dist.all_reduce(y_part)
            got = y_part
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs()
        worst = max(worst, float(err.max()))
        ok = ok and bool((err <= 2e-2 + 1e-2 * want.float().abs()).all())
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return {"parity": "ok" if int(flag.item()) == 1 else "mismatch", "max_abs_err": round(worst, 6),
            "checked": "q, gate (column-parallel) and o, down (row-parallel), one full-size layer, vs unsharded"}


APPLY_PATH_NAMES = {1: "fused", 2: "split", 3: "stream", 4: "tc"}
APPLY_KERNELS = {1: "apply_fused_kernel", 2: "shrink_kernel+expand_kernel",
                 3: "lora_shrink_stream_kernel+lora_expand_stream_kernel",
                 4: "lora_shrink_tc_kernel+lora_expand_tc_kernel"}


def launches_per_layer(wl: Workload, grouped: bool, path: int, tp: int) -> dict:
    """Our kernel launches per layer (torch's memsets and NCCL's kernels not counted).
    path: 1 = one fused launch per call, 3 = streaming shrink + expand pair per
    call, 2 = shrink + expand per projection."""
    kinds = {name: kind for name, _, _, kind in wl.projs}
    lora = 0
    for grp in GROUPS:
        if tp > 1 and kinds[grp[0]] == ROW:
            lora += 2 * len(grp)  # shrink (fp32 partials) + expand
        elif path == 2:
            lora += 2 * len(grp)
        else:
            calls = 1 if grouped else len(grp)
            lora += calls * (1 if path == 1 else 2)
    return {"lora": lora, "rmsnorm": 2}


def capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, iters: int) -> float:
    """Mean ms per replay, CUDA events on the replaying stream."""
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(iters):
        g.replay()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="mlora_clocks_", suffix=".csv")[1])

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def read_traffic() -> dict:
    p = ROOT / "profiles" / "ncu_traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


class CpuReference:
    """The reference's per-segment Torch path (oracle port) on the host cores.

    One sample = one whole layer of the workload (2 RMSNorms + 7 projections,
    shrink+expand, bf16, unsharded); throughput is scaled to the full step
    (tokens per step / (layers x seconds per layer)).
    """

    def __init__(self, wl: Workload):
        from oracle.torch_port import TorchPortBackend, rmsnorm

        self.wl = wl
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        ids, info, lens = routing(wl, 0)
        indptr = [0]
        for n in lens:
            indptr.append(indptr[-1] + n)
        self.be = TorchPortBackend(torch.tensor(indptr, dtype=torch.int32),
                                   torch.tensor(info.weight_indices, dtype=torch.int32),
                                   torch.tensor(info.lora_ranks, dtype=torch.int32),
                                   torch.tensor(info.scalings, dtype=torch.bfloat16), len(lens))
        self.rmsnorm = rmsnorm
        g = torch.Generator().manual_seed(7)
        dt = torch.bfloat16
        K, R, T = wl.adapters, wl.rank, wl.tokens
        self.A = {n: ((torch.rand(K, R, i, generator=g) * 2 - 1) / math.sqrt(i)).to(dt) for n, i, _, _ in wl.projs}
        self.B = {n: (torch.randn(K, o, R, generator=g) * 0.02).to(dt) for n, _, o, _ in wl.projs}
        self.y = {n: torch.randn(T, o, generator=g).to(dt) for n, _, o, _ in wl.projs}
        self.h = torch.randn(T, wl.hidden, generator=g).to(dt)
        self.w = torch.ones(wl.hidden, dtype=dt)
        self.xd = torch.randn(T, wl.inter, generator=g).to(dt)

    def layer(self) -> float:
        t0 = time.perf_counter()
        be, A, B, y = self.be, self.A, self.B, self.y
        xn1 = self.rmsnorm(self.h, self.w, EPS)
        for n in ("q", "k", "v", "o"):
            be.apply_lora(xn1, A[n], B[n], y[n])
        xn2 = self.rmsnorm(self.h, self.w, EPS)
        for n in ("gate", "up"):
            be.apply_lora(xn2, A[n], B[n], y[n])
        be.apply_lora(self.xd, A["down"], B["down"], y["down"])
        return time.perf_counter() - t0

    def step(self, layers: int) -> float:
        """Seconds for one step of ``layers`` layers."""
        t0 = time.perf_counter()
        for _ in range(layers):
            self.layer()
        return time.perf_counter() - t0

    def measure(self, seconds: float = 12.0) -> dict:
        self.layer()
        n, el = 0, 0.0
        while el < seconds or n < 2:
            el += self.layer()
            n += 1
        per_layer = el / n
        wl = self.wl
        return {"value": wl.tokens / (wl.layers * per_layer), "unit": UNIT, "cores": self.threads, "kind": "port",
                "sample": f"{n} {wl.name} layers (2 RMSNorm + 7 projections, bf16) in {el:.1f}s; "
                          f"x{wl.layers} layers per step",
                "per_layer_ms": round(per_layer * 1e3, 3)}


REF_BUDGET_S = 240.0  # wall-clock bound of the reference arm's warm-up + timed steps

POOL_SLOTS = 64
ZIPF_S = 1.1
CFG4_RANKS = (8, 16, 32, 64)
CFG4_TEMPLATES = 8  # distinct host weight sets per rank (adapters share them; every load still copies its bank)


def admit(queue: list, slots: int, resident=(), n_deferred: int = 0, resident_first: bool = False):
    """cfg4 admission through the library's AdmissionPolicy: returns (admitted names
    in queue order, deferred names in retry order, admitted adapters)."""
    from multi_lora_b200.admission import AdmissionPolicy

    adm = AdmissionPolicy(slots, resident_first=resident_first).admit(queue, resident=resident,
                                                                      n_deferred=n_deferred)
    return [queue[i] for i in adm.admitted], [queue[i] for i in adm.deferred], adm.adapters


def module_keys(layers: int):
    proj = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
            "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    return {(l, n): f"layers.{l}.{proj[n]}" for l in range(layers) for n in proj}


def run_pool_workload(args, wl: Workload, dev) -> None:
    """cfg4: every step admits tokens, makes their adapters resident in the
    64-slot pool (LRU eviction, pinned-host loads on the copy stream), writes
    the routing and replays the graph of the 32-layer LoRA forward. Timed end
    to end (loads included) with CUDA events and the host clock."""
    import numpy as np

    from multi_lora_b200 import _native
    from multi_lora_b200.backend import CudaLoRABackend
    from multi_lora_b200.batch_info import (BatchLoRAInfo, empty_kernel_input_metadata, group_rows,
                                            write_kernel_input_metadata)
    from multi_lora_b200.pool import LoRAMemoryPool
    from multi_lora_b200.weights import AdapterWeights

    dt = torch.bfloat16
    keys = module_keys(wl.layers)
    dims = {n: (i, o) for n, i, o, _ in wl.projs}
    sum_in = sum(dims[n][0] for _, n in keys)
    sum_out = sum(dims[n][1] for _, n in keys)
    g = torch.Generator(device=dev).manual_seed(4321)
    templates = {}
    for r in CFG4_RANKS:
        templates[r] = []
        for _ in range(CFG4_TEMPLATES):
            a_all = ((torch.rand(r, sum_in, generator=g, device=dev) * 2 - 1) / 64).to(dt).cpu()
            b_all = (torch.randn(sum_out, r, generator=g, device=dev) * 0.02).to(dt).cpu()
            mods, ia, ob = {}, 0, 0
            for (l, n), key in keys.items():
                i, o = dims[n]
                mods[key] = (a_all[:, ia:ia + i], b_all[ob:ob + o])
                ia += i
                ob += o
            templates[r].append(AdapterWeights(rank=r, scaling=2.0, modules=mods))
    rng = np.random.default_rng(0)
    ranks = rng.choice(CFG4_RANKS, size=wl.adapters)
    store = {f"a{i}": templates[int(ranks[i])][i % CFG4_TEMPLATES] for i in range(wl.adapters)}
    bank_bytes = {r: r * (sum_in + sum_out) * 2 for r in CFG4_RANKS}

    pool = LoRAMemoryPool(POOL_SLOTS, wl.rank, dev, dtype=dt)
    pool.ensure_buffers(templates[64][0])
    T = wl.tokens
    layers = []
    gl = torch.Generator(device=dev).manual_seed(99)
    for l in range(wl.layers):
        L = Layer()
        L.A, L.B, L.y = {}, {}, {}
        for n, i, o, _ in wl.projs:
            L.A[n], L.B[n] = pool.get_module_buffers(keys[(l, n)])
            L.y[n] = torch.randn(T, o, generator=gl, device=dev).to(dt)
        H = wl.hidden
        L.h1 = torch.randn(T, H, generator=gl, device=dev).to(dt)
        L.h2 = torch.randn(T, H, generator=gl, device=dev).to(dt)
        L.w1 = (1 + 0.1 * torch.randn(H, generator=gl, device=dev)).to(dt)
        L.w2 = (1 + 0.1 * torch.randn(H, generator=gl, device=dev)).to(dt)
        L.xn1 = torch.empty(T, H, device=dev, dtype=dt)
        L.xn2 = torch.empty(T, H, device=dev, dtype=dt)
        xo = torch.randn(T, H, generator=gl, device=dev).to(dt)
        xd = torch.randn(T, wl.inter, generator=gl, device=dev).to(dt)
        L.x = {"q": L.xn1, "k": L.xn1, "v": L.xn1, "o": xo, "gate": L.xn2, "up": L.xn2, "down": xd}
        layers.append(L)

    # Zipf(s) over the adapters; AdmissionPolicy picks the tokens (at most 64 adapters), the rest deferred
    p_zipf = 1.0 / np.arange(1, wl.adapters + 1) ** ZIPF_S
    p_zipf /= p_zipf.sum()
    pending: list = []

    def next_batch():
        nonlocal pending
        draws = list(rng.choice(wl.adapters, size=T - len(pending), p=p_zipf))
        admitted, pending, distinct = admit(pending + [f"a{int(i)}" for i in draws], POOL_SLOTS,
                                            resident=pool.name_to_slot.keys(), n_deferred=len(pending),
                                            resident_first=args.resident_first)
        return admitted, distinct

    be = CudaLoRABackend()
    meta = empty_kernel_input_metadata(device=dev, dtype=dt)
    stats = {"tokens": 0, "loads": 0, "h2d_bytes": 0, "distinct": 0, "steps": 0, "scatters": 0}

    def schedule(count: bool):
        nonlocal meta
        admitted, distinct = next_batch()
        before = set(pool.name_to_slot)
        pool.prepare_lora_batch(distinct, weight_store=store)
        new = [n for n in distinct if n not in before]
        names, lens = group_rows(admitted, [])
        info = pool.build_batch_info(names)
        pad = T - len(names)  # fixed segment capacity: empty segments past the batch
        padded = BatchLoRAInfo(weight_indices=list(info.weight_indices) + [0] * pad, lora_ranks=info.lora_ranks,
                               scalings=info.scalings)
        meta = write_kernel_input_metadata(meta, padded, device=dev, dtype=dt, seq_lens=list(lens) + [0] * pad)
        be.set_kernel_input_metadata(meta)
        if count:
            stats["tokens"] += len(admitted)
            stats["loads"] += len(new)
            per_rank: dict = {}
            for n in new:
                per_rank[store[n].rank] = per_rank.get(store[n].rank, 0) + 1
            stats["scatters"] += sum((c + 3) // 4 for c in per_rank.values())  # one launch per 4 banks
            stats["h2d_bytes"] += sum(bank_bytes[store[n].rank] for n in new)
            stats["distinct"] += len(distinct)
            stats["steps"] += 1

    schedule(False)
    step_graph = capture(lambda: run_step(wl, layers, be))
    path = _native.capi().mlora_last_apply_path()
    per_layer = launches_per_layer(wl, True, path, 1)
    launches = wl.layers * (per_layer["lora"] + per_layer["rmsnorm"])
    for _ in range(max(args.warmup, 3)):  # fills the pool
        schedule(False)
        step_graph.replay()
    torch.cuda.synchronize()
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    clocks = ClockSampler(visible[0].strip() if visible else 0)
    clocks.start()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(st)
    for _ in range(args.steps):
        schedule(True)
        step_graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    clk = clocks.stop()
    ms = max(e0.elapsed_time(e1), wall_ms) / args.steps
    g_c = capture(lambda: run_step(wl, layers, be))  # compute alone, the last step's routing
    compute_ms = time_graph(g_c, 20)
    del g_c
    pool.buffers.check_status()
    be.check_routing()
    value = stats["tokens"] / (ms * args.steps / 1e3)
    per_step_h2d = stats["h2d_bytes"] / args.steps
    out = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded; 8 distinct host weight sets per rank shared by the 256 adapters)",
           "config": {"workload": wl.desc, "global_batch": T, "seq_len": 1, "layers": wl.layers,
                      "adapters": wl.adapters, "pool_slots": POOL_SLOTS, "max_rank": wl.rank,
                      "parallelism": "single", "l2": "no flush: GBs of pool weights and host loads per step"},
           "pool": {"tokens_per_step": round(stats["tokens"] / args.steps, 1),
                    "distinct_adapters_per_step": round(stats["distinct"] / args.steps, 1),
                    "loads_per_step": round(stats["loads"] / args.steps, 2),
                    "h2d_gb_per_step": round(per_step_h2d / 1e9, 3),
                    "h2d_gbs_achieved": round(per_step_h2d / (ms / 1e3) / 1e9, 1),
                    "compute_ms_per_step_alone": round(compute_ms, 4), "deferred_at_end": len(pending),
                    "admission": "resident-first" if args.resident_first else "queue order"},
           "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": round(per_step_h2d),
                   "d2h_bytes_per_step": 0, "path": "admission + pool.prepare_lora_batch (evict, pinned H2D, "
                                                    "scatter) + routing write + graph replay, every step"},
           "gpu_launches": launches * args.steps + stats["scatters"], "clocks": clk, "pdl": _native.get_pdl(),
           "apply_path": APPLY_PATH_NAMES.get(path, str(path))}
    print(json.dumps(out), flush=True)
    del step_graph


def config_block(wl: Workload, n: int) -> dict:
    return {"workload": wl.desc, "global_batch": wl.tokens, "seq_len": 1, "layers": wl.layers,
            "adapters": wl.adapters, "rank": wl.rank,
            "parallelism": f"tp{n} (q/k/v/gate/up column-parallel, o/down row-parallel; fp32 [T, r] shrink "
                           f"partials summed over the ranks)" if n > 1 else "single",
            "l2": "no flush: each step streams the distinct per-layer adapter weights (GBs, > 126 MB L2)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 400 for this library, 20 for the reference's CPU path)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the workload's layer count (small cases for profiler captures only; "
                         "the reported numbers are then not the workload's)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--resident-first", action=argparse.BooleanOptionalAction, default=True,
                    help="cfg4: admit tokens whose adapter is resident before the others (fewer loads)")
    ap.add_argument("--row-exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: sum the row-parallel shrink partials through peer memory inside the kernels "
                         "(p2p) or with an NCCL all-reduce (nccl)")
    ap.add_argument("--ungrouped", action="store_true",
                    help="one apply_lora call per projection instead of grouping q/k/v and gate/up")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else 400
    wl = WORKLOADS[args.workload]
    if args.layers > 0:
        wl.layers = args.layers
        wl.desc += f" [layers overridden to {args.layers}: profiling case]"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(args.gpus, world)

    if args.impl == "reference":
        # the reference's CPU path on the host cores; rank 0 alone. Each timed
        # step runs every layer of the workload (2 RMSNorms + 7 projections per
        # layer), so steps x ms_per_step is the time actually spent; only when
        # that would pass REF_BUDGET_S does a step shrink to fewer layers, and
        # the line then says so (config.layers is what one step ran).
        if rank != 0:
            return
        ref = CpuReference(wl)
        est = ref.layer()  # one layer sizes the run
        layers = wl.layers
        if (args.steps + args.warmup) * wl.layers * est > REF_BUDGET_S:
            layers = max(1, int(REF_BUDGET_S / ((args.steps + args.warmup) * est)))
        for _ in range(args.warmup):
            ref.step(layers)
        times = [ref.step(layers) for _ in range(args.steps)]
        ms = statistics.mean(times) * 1e3
        value = wl.tokens / (ms / 1e3)
        cfg = config_block(wl, n)
        sample = f"each step: {layers} {wl.name} layers (2 RMSNorm + 7 projections each, bf16, unsharded)"
        if layers != wl.layers:
            cfg["layers"] = layers
            cfg["workload"] += f" [reference step shortened to {layers} of {wl.layers} layers to fit the run budget]"
        out = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": n,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic", "config": cfg,
               "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.threads, "kind": "port",
                                "sample": sample},
               "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return

    if wl.name == "cfg4":
        if world > 1:
            raise SystemExit("cfg4 is a single-GPU workload (one slot pool per GPU)")
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        run_pool_workload(args, wl, dev)
        return

    tp = world
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)

    from multi_lora_b200 import _native
    from multi_lora_b200.backend import CudaLoRABackend
    from multi_lora_b200.batch_info import empty_kernel_input_metadata, write_kernel_input_metadata

    _native.ops()
    ids, info, lens = routing(wl, 0)  # the same tokens on every TP rank
    layers = build_workload(wl, dev, tp_rank=rank, tp=tp)
    be = CudaLoRABackend()
    meta = write_kernel_input_metadata(empty_kernel_input_metadata(device=dev, dtype=torch.bfloat16), info,
                                       device=dev, dtype=torch.bfloat16, seq_lens=lens)
    be.set_kernel_input_metadata(meta)
    if world > 1:  # communicator up before any capture
        w = torch.ones(1, device=dev)
        torch.distributed.all_reduce(w)
    torch.cuda.synchronize()

    parity = None
    exchange = None
    if world > 1 and args.row_exchange == "p2p":
        from multi_lora_b200.tensor_parallel import PeerExchange

        exchange = PeerExchange.create(device=dev, max_rows=wl.tokens, max_rank=wl.rank)
    if world > 1:  # one checked layer before anything is timed
        parity = tp_parity_check(wl, dev, be, rank, tp, exchange=exchange)
        if parity["parity"] != "ok":
            if rank == 0:
                print(json.dumps({"metric": METRIC, "error": "tensor-parallel parity mismatch", **parity}),
                      flush=True)
            torch.distributed.destroy_process_group()
            raise SystemExit(3)
        be.set_kernel_input_metadata(meta)

    grouped = not args.ungrouped
    graphs = []
    step_graph = capture(lambda: run_step(wl, layers, be, grouped=grouped, tp=tp, tp_rank=rank,
                                          exchange=exchange))
    graphs.append(step_graph)
    be.apply_lora(layers[0].x["q"], layers[0].A["q"], layers[0].B["q"], layers[0].y["q"].clone())
    path = _native.capi().mlora_last_apply_path()
    per_layer = launches_per_layer(wl, grouped, path, tp)
    launches_per_step = wl.layers * (per_layer["lora"] + per_layer["rmsnorm"])

    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    dev_index = dev.index if dev.index is not None else 0
    clocks = ClockSampler(visible[dev_index].strip() if dev_index < len(visible) else dev_index)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        step_graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    value = wl.tokens / (ms / 1e3)

    # ---- roofline of the dominant kernel (the apply_lora launches), timed alone ----
    ab = algorithmic_bytes(wl, ids, tp)
    pk = peaks()
    g_lora = capture(lambda: run_step(wl, layers, be, parts=("lora",), grouped=grouped, tp=tp, tp_rank=rank,
                                       exchange=exchange))
    graphs.append(g_lora)
    lora_ms = max_over_ranks(time_graph(g_lora, max(20, args.steps // 4)))
    g_rms = capture(lambda: run_step(wl, layers, be, parts=("rmsnorm",), tp=tp, tp_rank=rank))
    graphs.append(g_rms)
    rms_ms = max_over_ranks(time_graph(g_rms, max(20, args.steps // 4)))
    lora_launches = wl.layers * per_layer["lora"]
    per_launch_bytes = ab["lora"] / lora_launches
    per_launch_ms = lora_ms / lora_launches
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    if tp > 1:
        kernel = ("lora part per rank: apply_fused_kernel (column) + streaming shrink/expand with the partials "
                  + ("exchanged over peer memory (row)" if exchange is not None else "NCCL-all-reduced (row)"))
    else:
        kernel = APPLY_KERNELS.get(path, "unknown")
    # ncu DRAM bytes per launch of this workload's kernel(s), one GPU only
    tr = read_traffic()
    traffic = (tr.get(f"{wl.name}:{kernel}", tr.get(kernel) if wl.name == "cfg2" else None)
               if tp == 1 else None)
    step_bytes = ab["lora"] + ab["rmsnorm"]
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic, "kernel": kernel,
                "peak_source": pk["src"], "bytes_per_launch": round(per_launch_bytes),
                "launch_us": round(per_launch_ms * 1e3, 3), "launches_timed": lora_launches,
                "tensor": {"achieved_tflops": round(ab["lora_flops"] / (lora_ms / 1e3) / 1e12, 2),
                           "peak_tflops": pk["bf16_tflops"],
                           "frac": round(ab["lora_flops"] / (lora_ms / 1e3) / 1e12 / pk["bf16_tflops"], 4)}}
    step_achieved = step_bytes / (ms / 1e3) / 1e9
    step_roofline = {"bytes_per_step": step_bytes, "achieved": round(step_achieved, 1),
                     "frac": round(step_achieved / pk["hbm_gbs"], 4), "unit": "GB/s",
                     "lora_ms_alone": round(lora_ms, 4), "rmsnorm_ms_alone": round(rms_ms, 4),
                     "distinct_adapters": ab["distinct_adapters"], "per_rank": tp > 1}
    if grouped:  # the same work as one apply_lora call per projection, for comparison
        g_u = capture(lambda: run_step(wl, layers, be, grouped=False, tp=tp, tp_rank=rank, exchange=exchange))
        graphs.append(g_u)
        step_roofline["ungrouped_ms_per_step"] = round(max_over_ranks(time_graph(g_u, max(20, args.steps // 4))), 4)

    # ---- e2e: public API with host buffers, copies inside the timed region ----
    last = layers[-1].y["down"]
    h_in = torch.randn(wl.tokens, wl.hidden).bfloat16().pin_memory()
    y_out = torch.empty(tuple(last.shape), dtype=torch.bfloat16).pin_memory()
    meta_bytes = meta._packed.words * 4 if meta._packed is not None else 0
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for _ in range(args.steps):
        write_kernel_input_metadata(meta, info, device=dev, dtype=torch.bfloat16, seq_lens=lens)
        layers[0].h1.copy_(h_in, non_blocking=True)
        step_graph.replay()
        y_out.copy_(last, non_blocking=True)
        st.synchronize()
    e3.record(st)
    e3.synchronize()
    e2e_ms = max_over_ranks(max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3) / args.steps)
    e2e = {"value": wl.tokens / (e2e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": meta_bytes + h_in.numel() * 2, "d2h_bytes_per_step": y_out.numel() * 2,
           "ms_per_step": e2e_ms,
           "path": "write_kernel_input_metadata (pinned H2D) + input hidden H2D + graph of the public-API "
                   "step + output D2H + host sync, every step"}

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu_baseline:
        cpu = CpuReference(wl).measure()

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": n, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded; random-init adapters of the named shapes)",
               "config": config_block(wl, n), "roofline": roofline, "step_roofline": step_roofline,
               "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
               "clocks": clk, "pdl": _native.get_pdl(), "grouped": grouped,
               "apply_path": APPLY_PATH_NAMES.get(path, str(path))}
        if parity is not None:
            out["parity"] = parity["parity"]
            out["parity_check"] = parity
            out["row_exchange"] = args.row_exchange
        print(json.dumps(out), flush=True)
    # graphs that hold NCCL calls go before the process group
    del step_graph, g_lora, g_rms
    if grouped:
        del g_u
    graphs.clear()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
        if exchange is not None:
            exchange.close()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
