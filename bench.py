#!/usr/bin/env python
"""Benchmark of the B200-native GLM MoE block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode1|decode2|prefill256]
    python bench.py --impl reference ...      # CPU restatement of the reference path

Workload (default decode1): the full-size decode MoE layer (d=4096, 128
experts, top-8, 8 groups / 4 kept, F=1536, one shared expert, scale 2.5) at
M=1 token; decode2 is the width-two MTP verify (M=2); prefill256 is M=256.
A step is one MoE-layer forward.  Steps cycle through `--layers` (default 8)
independently generated layers so that no step finds its weights in L2
(8 x 1.33 GB of weights > 126 MB L2).  Each layer's forward is a CUDA graph
captured from the public module call; the timed region is K graph replays
bracketed by CUDA events.  With N > 1 each rank runs its own replica
(decode shards by independent token streams; no collective on the data
path) and `value` is the sum over ranks.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {"decode1": 1, "decode2": 2, "prefill256": 256}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel, from an ncu capture of this bench's command (workload, stage)
MEASURED_TRAFFIC = {
    ("decode1", "gate_up"): 80.53e6,
}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4000)
    p.add_argument("--warmup", type=int, default=200)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=tuple(WORKLOADS), default="decode1")
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline sample")
    return p.parse_args(argv)


# ----------------------------------------------------------------- utils ---

def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
        except (KeyError, ValueError):
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"livglm_clocks_{os.getpid()}_{gpu_index}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.count(",") >= 8]
        try:
            self.path.unlink()
        except OSError:
            pass
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def layer_bytes(cfg, M: int, unique: float) -> dict:
    """Algorithmic HBM bytes of one layer call and of its gate/up stage."""
    d, F, E, k = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts, cfg.num_experts_per_tok
    Fs = cfg.shared_intermediate_size
    per_proj = F * d // 2 + F * d // 32
    gate_up = unique * 2 * per_proj + 2 * Fs * d * 2 + M * d * 2 + (M * k * F + M * Fs) * 2
    down = unique * per_proj + Fs * d * 2 + (M * k * F + M * Fs) * 2 + (M * k * d + M * d) * 2
    router = E * d * 4 + E * 4 + M * d * 2 + M * E * 4
    combine = (M * k * d + M * d) * 2 + M * k * 4 + M * d * 4
    layer = unique * 3 * per_proj + 3 * Fs * d * 2 + E * d * 4 + E * 4 + M * d * 2 + M * d * 4
    return {"gate_up": gate_up, "down": down, "router": router, "combine": combine, "layer": layer,
            "per_expert": 3 * per_proj}


# -------------------------------------------------------------- CPU side ---

def cpu_sample(cfg, tn: dict, x_bits, budget_s: float) -> dict:
    """Time the oracle port of the layer on host cores, one token per call,
    until the budget is spent (at least two tokens)."""
    from oracle import moe_oracle as mo

    n_threads = os.cpu_count() or 1
    mo.moe_forward(x_bits[:1], tn, cfg)  # warm caches / build
    t0 = time.perf_counter()
    n = 0
    while True:
        mo.moe_forward(x_bits[n % len(x_bits):n % len(x_bits) + 1], tn, cfg)
        n += 1
        el = time.perf_counter() - t0
        if (el >= budget_s and n >= 2) or n >= 10_000:
            break
    return {"value": n / el, "unit": "tokens/s", "cores": n_threads, "kind": "port",
            "sample": f"{n} single-token calls of the NumPy/C oracle (dequantise-then-matmul, BLAS threads="
                      f"{n_threads}) on one cfg1 layer, {el:.1f} s"}


def run_reference(args) -> None:
    """--impl reference: the CPU restatement of the reference path."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch

    from livglm_b200 import synthetic
    from livglm_b200.config import CONFIGS
    from oracle import moe_oracle as mo
    from oracle.torch_bridge import bank_to_numpy

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = CONFIGS["cfg1"]
    M = WORKLOADS[args.workload]
    t = synthetic.layer_weights(cfg, seed=0, device="cpu")
    tn = bank_to_numpy(t)
    x = mo.f32_to_bf16_bits(np.random.default_rng(0).standard_normal((max(M, 8), cfg.hidden_size)).astype(np.float32))
    for _ in range(min(args.warmup, 1)):
        mo.moe_forward(x[:M], tn, cfg)
    budget = 60.0
    t0 = time.perf_counter()
    n = 0
    while n < args.steps:
        mo.moe_forward(x[:M], tn, cfg)
        n += 1
        if time.perf_counter() - t0 > budget:
            break
    el = time.perf_counter() - t0
    value = n * M / el
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 * el / n,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"cfg1-{args.workload}", "M": M, "hidden_size": 4096, "n_routed_experts": 128,
                   "num_experts_per_tok": 8, "moe_intermediate_size": 1536},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} of {args.steps} requested steps (M={M}) of the NumPy/C restatement of "
                                   f"kg36/livglm moe.py/expert_ssd.py in {el:.1f} s (MLX, the reference's own "
                                   "runtime, is not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU side ---

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from livglm_b200 import _native, synthetic
    from livglm_b200.config import CONFIGS
    from livglm_b200.moe import build_layer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    cfg = CONFIGS["cfg1"]
    M = WORKLOADS[args.workload]
    L = max(1, args.layers)
    _native.load()
    layers, xs = [], []
    for i in range(L):
        t = synthetic.layer_weights(cfg, layer=i, seed=rank, device=dev)
        layers.append(build_layer(cfg, t, layer_idx=i))
        xs.append(synthetic.hidden_states(cfg, M, seed=1000 * rank + i, device=dev))
    torch.cuda.synchronize()

    # routing statistics (distinct experts per call) for the byte count
    uniq = []
    for i in range(L):
        _, _, idx = layers[i](xs[i], return_route=True)
        uniq.append(len(set(idx.view(torch.int32).reshape(-1).tolist())))
    U = sum(uniq) / len(uniq)

    # warm every layer once outside capture (workspace allocation)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for i in range(L):
            layers[i](xs[i])
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize()

    def capture(traced: bool):
        if traced:
            _native.trace_enable(L)  # one trace slot per captured layer
        gs = []
        for i in range(L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                layers[i](xs[i])
            gs.append(g)
        torch.cuda.synchronize()
        return gs

    def capture_stack():
        """One graph of all L layers in order, as a decode step through the
        model's MoE layers is captured: consecutive layers chain by
        programmatic dependent launch like the kernels inside a layer."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(L):
                layers[i](xs[i])
        torch.cuda.synchronize()
        return g

    def timed(gs, steps: int, stack=None) -> float:
        """Exactly `steps` layer forwards: whole replays of the L-layer graph,
        then single-layer graphs for the remainder."""
        def run(n: int) -> None:
            full = n // L if stack is not None else 0
            for _ in range(full):
                stack.replay()
            for s in range(n - full * L):
                gs[s % L].replay()
        run(max(args.warmup, 3))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        run(steps)
        ev1.record()
        torch.cuda.synchronize()
        return ev0.elapsed_time(ev1)

    # (1) the timed region: plain graphs (kernels chained by programmatic
    #     dependent launch, no trace events between them)
    graphs = capture(traced=False)
    stack = capture_stack()
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.25)
        ms = timed(graphs, args.steps, stack)
    del stack
    # (2) per-stage device times: the same graphs with CUDA events between the
    #     stages (which serialises the stages), replayed for the same steps
    traced_graphs = capture(traced=True)
    ms_traced = timed(traced_graphs, args.steps)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stages = _native.trace_read(L)  # last replay of each layer's traced graph
    del traced_graphs
    _native.trace_enable(0)

    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())

    # ---- e2e: public module call with pinned host buffers (eager) ----------
    K_e2e = min(args.steps, 2000)
    x_host = torch.empty(M, cfg.hidden_size, dtype=torch.bfloat16, pin_memory=True)
    x_host.copy_(xs[0].cpu())
    out_host = torch.empty(M, cfg.hidden_size, dtype=torch.float32, pin_memory=True)
    x_dev = torch.empty_like(xs[0])

    def e2e_step(s: int, host_api: bool) -> None:
        if host_api:  # tokens and result in page-locked host memory, handed to the module
            layers[s % L](x_host, out=out_host)
        else:         # device tensors, with the caller's own copies
            x_dev.copy_(x_host, non_blocking=True)
            out_host.copy_(layers[s % L](x_dev), non_blocking=True)

    def e2e_ms(host_api: bool) -> float:
        for s in range(max(args.warmup, 3) if args.warmup < 50 else 50):
            e2e_step(s, host_api)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(K_e2e):
            e2e_step(s, host_api)
        e1.record()
        torch.cuda.synchronize()
        ms_ = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([ms_], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms_ = float(tt.item())
        return ms_

    ms_e2e = e2e_ms(True)
    ms_e2e_copies = e2e_ms(False)

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.torch_bridge import bank_to_numpy, to_numpy

        t0 = synthetic.layer_weights(cfg, layer=0, seed=0, device=dev)
        tn = bank_to_numpy(t0)
        del t0
        cpu = cpu_sample(cfg, tn, to_numpy(synthetic.hidden_states(cfg, 8, seed=0, device=dev)), args.cpu_seconds)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = measured_peaks()
    by = layer_bytes(cfg, M, U)
    # kernels per layer call: decode chain 5 (router logits, select + dispatch,
    # gate/up, down, combine), plus the activation split of the tensor-core
    # down kernel for one token (on unless LIVGLM_TC_DOWN=0)
    tc_down = M == 1 and os.environ.get("LIVGLM_TC_DOWN", "1") != "0"
    launches_per_step = (6 if tc_down else 5) if M <= 4 else 6
    mean = {k: statistics.fmean(s[k] for s in stages) for k in _native.TRACE_STAGES} if stages else {}
    dominant = max(mean, key=mean.get) if mean else "gate_up"
    dom_ms = mean.get(dominant, float("nan"))
    dom_bytes = by[dominant]
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9 if dom_ms and dom_ms > 0 else None
    ms_step = ms / args.steps
    value = world * M * args.steps / (ms * 1e-3)
    layer_gbs = by["layer"] / (ms_step * 1e-3) / 1e9
    line = {
        "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) bf16 tokens; N(0,0.02) weights, routed MXFP4 g32, shared bf16)",
        "config": {"workload": f"cfg1-{args.workload}", "M": M, "hidden_size": cfg.hidden_size,
                   "n_routed_experts": cfg.n_routed_experts, "num_experts_per_tok": cfg.num_experts_per_tok,
                   "n_group": cfg.n_group, "topk_group": cfg.topk_group,
                   "moe_intermediate_size": cfg.moe_intermediate_size, "layers_rotated": L,
                   "graph": f"one CUDA graph of the {L} layers, replayed",
                   "l2": f"inputs larger than L2: {L} distinct layers cycled ({L * 1.33:.1f} GB of weights)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "operands": "x bf16, routed w MXFP4 (E2M1+E8M0), shared w bf16, f32 accumulate, f32 out"},
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": (achieved / peaks["hbm_gbs"]) if achieved else None,
                     "traffic": MEASURED_TRAFFIC.get((args.workload, dominant)), "peak_source": peaks["source"],
                     "algorithmic_bytes_per_launch": dom_bytes, "launch_ms": dom_ms},
        "e2e": {"value": world * M * K_e2e / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": M * cfg.hidden_size * 2, "d2h_bytes_per_step": M * cfg.hidden_size * 4,
                "steps": K_e2e,
                "path": "ExpertSSDMoE.__call__(x_host, out=out_host) eager (ctypes -> C ABI): bf16 tokens and "
                        "f32 result in page-locked host memory, read and written by the kernels over the host link",
                "with_caller_copies": {"value": world * M * K_e2e / (ms_e2e_copies * 1e-3),
                                       "path": "device tensors; the caller copies x in and the result out "
                                               "with non-blocking copies around each call"}},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": sampler.summary(),
        "extra": {"layer_hbm_gbs": layer_gbs, "layer_hbm_frac": layer_gbs / peaks["hbm_gbs"],
                  "layer_bytes": by["layer"], "unique_experts_per_call": U,
                  "stage_ms": mean, "ms_per_step_stages_serialised": ms_traced / args.steps},
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
