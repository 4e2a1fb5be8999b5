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

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

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

# (name, in, out) of Llama-2-7B projections
LLAMA2_7B = [("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
             ("gate", 4096, 11008), ("up", 4096, 11008), ("down", 11008, 4096)]
HIDDEN = 4096
LAYERS = 32
TOKENS = 64
ADAPTERS = 32
RANK = 16
SCALING = 32 / 16
EPS = 1e-6


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def cfg2_routing(seed: int = 0):
    """Adapter id per token (uniform over 32) -> grouped segments (adjacent equal ids merge)."""
    from multi_lora_b200.batch_info import BatchLoRAInfo, group_rows

    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, ADAPTERS, (TOKENS,), generator=g).tolist()
    names, lens = group_rows(ids, [])  # adapter i lives in slot i
    info = BatchLoRAInfo(weight_indices=list(names), lora_ranks=[RANK] * ADAPTERS,
                         scalings=[SCALING] * ADAPTERS)
    return ids, info, lens


def algorithmic_bytes(ids) -> dict:
    """Bytes a perfect kernel moves per step (adapter rows up to the rank only)."""
    d = len(set(ids))
    T, es = TOKENS, 2
    shrink = expand = 0
    for _, n_in, n_out in LLAMA2_7B:
        shrink += d * RANK * n_in * es + T * n_in * es + T * RANK * es
        expand += d * RANK * n_out * es + 2 * T * n_out * es + T * RANK * es
    rms = 2 * (2 * T * HIDDEN * es + HIDDEN * es)
    return {"shrink": shrink * LAYERS, "expand": expand * LAYERS, "rmsnorm": rms * LAYERS,
            "distinct_adapters": d}


class Layer:
    pass


def build_workload(dev, seed: int = 0):
    """Per-layer adapter slots and activations, generated on the device."""
    g = torch.Generator(device=dev).manual_seed(1234 + seed)
    dt = torch.bfloat16
    layers = []
    for _ in range(LAYERS):
        L = Layer()
        L.A, L.B, L.x, L.y = {}, {}, {}, {}
        for name, n_in, n_out in LLAMA2_7B:
            bound = 1.0 / math.sqrt(n_in)  # kaiming-uniform(a=sqrt(5)) of an [r, in] weight
            L.A[name] = ((torch.rand(ADAPTERS, RANK, n_in, generator=g, device=dev) * 2 - 1) * bound).to(dt)
            L.B[name] = (torch.randn(ADAPTERS, n_out, RANK, generator=g, device=dev) * 0.02).to(dt)
            L.y[name] = torch.randn(TOKENS, n_out, generator=g, device=dev).to(dt)
        L.h1 = torch.randn(TOKENS, HIDDEN, generator=g, device=dev).to(dt)
        L.h2 = torch.randn(TOKENS, HIDDEN, generator=g, device=dev).to(dt)
        L.w1 = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=dev)).to(dt)
        L.w2 = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device=dev)).to(dt)
        L.xn1 = torch.empty(TOKENS, HIDDEN, device=dev, dtype=dt)
        L.xn2 = torch.empty(TOKENS, HIDDEN, device=dev, dtype=dt)
        L.xo = torch.randn(TOKENS, HIDDEN, generator=g, device=dev).to(dt)       # attention output
        L.xd = torch.randn(TOKENS, 11008, generator=g, device=dev).to(dt)        # act(gate) * up
        L.x = {"q": L.xn1, "k": L.xn1, "v": L.xn1, "o": L.xo, "gate": L.xn2, "up": L.xn2, "down": L.xd}
        layers.append(L)
    return layers


def run_step(layers, be, parts=("rmsnorm", "lora"), grouped=True):
    """One forward of the LoRA hot path over all layers.

    grouped: q/k/v (shared input) and gate/up (shared input) each go through one
    ``apply_lora_group`` call, which is the dependency structure of the model
    (rmsnorm -> {q,k,v} -> o -> rmsnorm -> {gate,up} -> down); otherwise every
    projection is its own ``apply_lora`` call.
    """
    from multi_lora_b200.rmsnorm import rmsnorm_out

    if grouped and "lora" in parts:
        for L in layers:
            if "rmsnorm" in parts:
                rmsnorm_out(L.h1, L.w1, EPS, L.xn1)
            qkv = ("q", "k", "v")
            be.apply_lora_group(L.xn1, [L.A[n] for n in qkv], [L.B[n] for n in qkv], [L.y[n] for n in qkv])
            be.apply_lora(L.x["o"], L.A["o"], L.B["o"], L.y["o"])
            if "rmsnorm" in parts:
                rmsnorm_out(L.h2, L.w2, EPS, L.xn2)
            gu = ("gate", "up")
            be.apply_lora_group(L.xn2, [L.A[n] for n in gu], [L.B[n] for n in gu], [L.y[n] for n in gu])
            be.apply_lora(L.x["down"], L.A["down"], L.B["down"], L.y["down"])
        return
    for L in layers:
        if "rmsnorm" in parts:
            rmsnorm_out(L.h1, L.w1, EPS, L.xn1)
        for name in ("q", "k", "v", "o"):
            if "lora" in parts:
                be.apply_lora(L.x[name], L.A[name], L.B[name], L.y[name])
            elif "shrink" in parts:
                be.run_lora_a_sgemm(L.x[name], L.A[name])
            elif "expand" in parts:
                be.run_lora_b_sgemm(be._mid[:TOKENS], L.B[name], base_output=L.y[name])
        if "rmsnorm" in parts:
            rmsnorm_out(L.h2, L.w2, EPS, L.xn2)
        for name in ("gate", "up", "down"):
            if "lora" in parts:
                be.apply_lora(L.x[name], L.A[name], L.B[name], L.y[name])
            elif "shrink" in parts:
                be.run_lora_a_sgemm(L.x[name], L.A[name])
            elif "expand" in parts:
                be.run_lora_b_sgemm(be._mid[:TOKENS], L.B[name], base_output=L.y[name])


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

    One sample = one whole cfg2 layer (2 RMSNorms + 7 projections,
    shrink+expand, bf16); throughput is scaled to the 32-layer step
    (tokens per step / (32 x seconds per layer)).
    """

    def __init__(self):
        from oracle.torch_port import TorchPortBackend, rmsnorm

        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        ids, info, lens = cfg2_routing(0)
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
        self.A = {n: ((torch.rand(ADAPTERS, RANK, i, generator=g) * 2 - 1) / math.sqrt(i)).to(dt)
                  for n, i, _ in LLAMA2_7B}
        self.B = {n: (torch.randn(ADAPTERS, o, RANK, generator=g) * 0.02).to(dt) for n, _, o in LLAMA2_7B}
        self.y = {n: torch.randn(TOKENS, o, generator=g).to(dt) for n, _, o in LLAMA2_7B}
        self.h = torch.randn(TOKENS, HIDDEN, generator=g).to(dt)
        self.w = torch.ones(HIDDEN, dtype=dt)
        self.xd = torch.randn(TOKENS, 11008, generator=g).to(dt)

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

    def measure(self, seconds: float = 12.0) -> dict:
        self.layer()
        n, el = 0, 0.0
        while el < seconds or n < 2:
            el += self.layer()
            n += 1
        per_layer = el / n
        return {"value": TOKENS / (LAYERS * per_layer), "unit": UNIT, "cores": self.threads, "kind": "port",
                "sample": f"{n} cfg2 layers (2 RMSNorm + 7 projections, bf16) in {el:.1f}s; x32 layers per step",
                "per_layer_ms": round(per_layer * 1e3, 3)}


def config_block(n: int) -> dict:
    return {"workload": "cfg2 Llama-2-7B-shaped decode: 32 layers x 7 LoRA projections + 2 RMSNorm, "
                        "64 tokens, 32 adapters r16 (alpha 32), bf16",
            "global_batch": TOKENS * n, "seq_len": 1, "layers": LAYERS, "adapters": ADAPTERS, "rank": RANK,
            "parallelism": f"replicas{n}" if n > 1 else "single",
            "l2": "no flush: each step streams ~2.6 GB of distinct per-layer adapter weights (> 126 MB L2)"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ungrouped", action="store_true",
                    help="one apply_lora call per projection instead of grouping q/k/v and gate/up")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(args.gpus, world)

    if args.impl == "reference":
        # the reference's CPU path on the host cores; rank 0 alone
        if rank != 0:
            return
        ref = CpuReference()
        for _ in range(args.warmup):
            ref.layer()
        per_layer = statistics.mean(ref.layer() for _ in range(args.steps))
        value = TOKENS / (LAYERS * per_layer)
        out = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": n,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_layer * LAYERS * 1e3,
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic", "config": config_block(1),
               "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.threads, "kind": "port",
                                "sample": f"each step: one cfg2 layer (2 RMSNorm + 7 projections), x32 layers"},
               "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)

    from multi_lora_b200 import _native
    from multi_lora_b200.backend import CudaLoRABackend
    from multi_lora_b200.batch_info import empty_kernel_input_metadata, write_kernel_input_metadata

    _native.ops()
    ids, info, lens = cfg2_routing(0)
    layers = build_workload(dev, seed=rank)
    be = CudaLoRABackend()
    meta = write_kernel_input_metadata(empty_kernel_input_metadata(device=dev, dtype=torch.bfloat16), info,
                                       device=dev, dtype=torch.bfloat16, seq_lens=lens)
    be.set_kernel_input_metadata(meta)
    torch.cuda.synchronize()

    grouped = not args.ungrouped
    step_graph = capture(lambda: run_step(layers, be, grouped=grouped))
    fused = _native.capi().mlora_last_apply_path() == 1
    lora_calls = 4 if grouped else 7
    launches_per_step = LAYERS * (2 + lora_calls * (1 if fused else 2))

    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

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
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = TOKENS * n / (ms / 1e3)

    # ---- roofline of the dominant kernel (the apply_lora launches), timed alone ----
    ab = algorithmic_bytes(ids)
    pk = peaks()
    g_lora = capture(lambda: run_step(layers, be, parts=("lora",), grouped=grouped))
    lora_ms = time_graph(g_lora, max(20, args.steps // 4))
    del g_lora
    g_rms = capture(lambda: run_step(layers, be, parts=("rmsnorm",)))
    rms_ms = time_graph(g_rms, max(20, args.steps // 4))
    del g_rms
    lora_launches = LAYERS * lora_calls * (1 if fused else 2)
    lora_bytes = ab["shrink"] + ab["expand"]
    per_launch_bytes = lora_bytes / lora_launches
    per_launch_ms = lora_ms / lora_launches
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    kernel = "apply_fused_kernel" if fused else "shrink_kernel+expand_kernel"
    traffic = read_traffic().get(kernel)
    step_bytes = lora_bytes + ab["rmsnorm"]
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic, "kernel": kernel,
                "peak_source": pk["src"], "bytes_per_launch": round(per_launch_bytes),
                "launch_us": round(per_launch_ms * 1e3, 3), "launches_timed": lora_launches}
    step_achieved = step_bytes / (ms / 1e3) / 1e9
    step_roofline = {"bytes_per_step": step_bytes, "achieved": round(step_achieved, 1),
                     "frac": round(step_achieved / pk["hbm_gbs"], 4), "unit": "GB/s",
                     "lora_ms_alone": round(lora_ms, 4), "rmsnorm_ms_alone": round(rms_ms, 4),
                     "distinct_adapters": ab["distinct_adapters"]}
    if grouped:  # the same work as one apply_lora call per projection, for comparison
        g_u = capture(lambda: run_step(layers, be, grouped=False))
        step_roofline["ungrouped_ms_per_step"] = round(time_graph(g_u, max(20, args.steps // 4)), 4)
        del g_u

    # ---- e2e: public API with host buffers, copies inside the timed region ----
    h_in = torch.randn(TOKENS, HIDDEN).bfloat16().pin_memory()
    y_out = torch.empty(TOKENS, HIDDEN, dtype=torch.bfloat16).pin_memory()
    meta_bytes = meta._packed.words * 4 if meta._packed is not None else 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for _ in range(args.steps):
        write_kernel_input_metadata(meta, info, device=dev, dtype=torch.bfloat16, seq_lens=lens)
        layers[0].h1.copy_(h_in, non_blocking=True)
        step_graph.replay()
        y_out.copy_(layers[-1].y["down"], non_blocking=True)
        st.synchronize()
    e3.record(st)
    e3.synchronize()
    e2e_ms = max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": TOKENS * n / (e2e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": meta_bytes + h_in.numel() * 2, "d2h_bytes_per_step": y_out.numel() * 2,
           "ms_per_step": e2e_ms,
           "path": "write_kernel_input_metadata (pinned H2D) + input hidden H2D + graph of the public-API "
                   "step + output D2H + host sync, every step"}

    cpu = None
    if rank == 0 and n == 1 and not args.no_cpu_baseline:
        cpu = CpuReference().measure()

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": n, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded; random-init adapters of the named shapes)",
               "config": config_block(n), "roofline": roofline, "step_roofline": step_roofline,
               "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
               "clocks": clk, "pdl": _native.get_pdl(), "grouped": grouped, "fused_path": fused}
        print(json.dumps(out), flush=True)
    del step_graph
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
