#!/usr/bin/env python
"""Benchmark of the B200-native GLM MoE block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg3|cfg4|prefill256|decode1|decode2]
    python bench.py --impl reference ...      # the CPU restatement of the reference path

Workloads (the benchmark plan's configs; d=4096, 128 experts, top-8, 8 groups /
4 kept, F=1536, one shared expert, routed scale 2.5; seeded synthetic data):
  cfg3 (default)  42 stacked MoE layers at M=4096 tokens, an unweighted RMSNorm
                  between layers (livglm_b200/stack.py); a step is one pass of
                  the 4096 tokens through the 42 layers.  With N > 1 GPUs the
                  routed experts are sharded expert-parallel (128/N per GPU,
                  NCCL all-to-all dispatch and return, livglm_b200/ep.py), each
                  rank bringing its own 4096 tokens (weak scaling).
  cfg4            one layer at M=16384 with the Zipf(1.2) correction bias
                  (livglm_b200/workloads.py); N > 1: expert-parallel, the 16384
                  tokens split over the ranks (strong scaling).
  prefill256      config 2: one layer at M=256.
  decode1/2       config 1: one layer at M=1 / M=2 (MTP width-two verify);
                  N > 1 runs N independent replicas.
Single-layer workloads cycle through `--layers` independently generated
layers (weights > L2).  Without expert parallelism every step is replayed
from a CUDA graph captured from the public module call.  `value` is MoE-layer
tokens/s (tokens x layers per step / time), summed over ranks.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    "cfg3": {"cfg": "cfg3", "M": 4096, "layers": 42, "kind": "stack", "steps": 10},
    "cfg4": {"cfg": "cfg4", "M": 16384, "layers": 2, "kind": "layer", "steps": 200, "zipf": True},
    "prefill256": {"cfg": "cfg2", "M": 256, "layers": 8, "kind": "layer", "steps": 200},
    "decode1": {"cfg": "cfg1", "M": 1, "layers": 8, "kind": "layer", "steps": 4000},
    "decode2": {"cfg": "cfg1", "M": 2, "layers": 8, "kind": "layer", "steps": 4000},
    # the MTP width-two verify at its call site: hyper-connections (4 streams)
    # around the block, model.py:132-136
    "site2": {"cfg": "cfg1", "M": 2, "layers": 8, "kind": "layer", "steps": 4000, "site": 4},
}
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel, from an ncu capture of this bench's command (workload -> bytes)
MEASURED_TRAFFIC = {
    "decode1": 80.53e6,
    "decode2": 119.0e6,  # gate_up_stream_kernel<2>, 16 distinct experts' gate/up + shared
    # gate/up stage of one layer: route split 2 MB + routed gate/up 891 MB + shared gate/up 27 MB
    "prefill256": 920.7e6,
    # gate/up stage of one layer: route gather 298 MB + routed gate/up 1,230 MB + shared gate/up 59 MB
    "cfg3": 1.587e9,
    # gate/up stage at M = 16384: gather 1,895 MB + routed gate/up 2,053 MB + shared gate/up 200 MB
    "cfg4": 4.148e9,
}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default per workload)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=tuple(WORKLOADS), default="cfg3")
    p.add_argument("--layers", type=int, default=None, help="layers cycled (single-layer workloads)")
    p.add_argument("--ep-impl", choices=("native", "python"), default="native",
                   help="expert parallelism through lg_moe_ep_forward (native) or the torch.distributed steps")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline sample")
    a = p.parse_args(argv)
    wl = WORKLOADS[a.workload]
    if a.steps is None:
        a.steps = wl["steps"]
    if a.layers is None:
        a.layers = wl["layers"]
    a.warmup = max(a.warmup, 3)
    return a


# ----------------------------------------------------------------- utils ---

def measured_peaks() -> dict:
    """HBM and bf16 peaks measured on this pool (MEASURED_PEAKS.json), else the
    pool's recorded fallback."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            sus = d.get("bf16_tflops_sustained")
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_tflops_sustained": float(sus) if sus else None, "source": "measured"}
        except (KeyError, ValueError):
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def fp4_peak_tflops() -> dict:
    """Dense kind::mxf4 tcgen05 throughput measured on this GPU by the
    self-test library's MMA-rate kernel (M=128, N=256, K=64 per MMA, one
    issuing thread per SM), or the nominal 9 PFLOP/s when it is not built."""
    try:
        import torch

        lib = ctypes.CDLL(str(ROOT / "tests" / "_build" / "liblivglm_umma_selftest.so"))
        fn = lib.lg_umma_mma_rate
        fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                       ctypes.c_void_p]
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        cyc = torch.zeros(sms, dtype=torch.int64, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        fn(0, 256, 20, sms, cyc.data_ptr(), st.data_ptr(), None)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        groups = 200
        e0.record()
        rc = fn(0, 256, groups, sms, cyc.data_ptr(), st.data_ptr(), None)
        e1.record()
        torch.cuda.synchronize()
        if rc == 0 and int(st.item()) == 0:
            flop = 2 * 128 * 256 * 64 * 64 * groups * sms
            return {"tflops": flop / e0.elapsed_time(e1) / 1e9, "source": "measured (tcgen05 kind::mxf4 MMA rate)"}
    except (OSError, AttributeError, RuntimeError):
        pass
    return {"tflops": 9000.0, "source": "nominal (dense FP4, B200)"}


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


def layer_work(cfg, M: int, unique: float) -> dict:
    """Algorithmic HBM bytes and FLOPs of one layer call and of its stages
    (weights read once per call; activations once each way)."""
    d, F, E, k = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts, cfg.num_experts_per_tok
    Fs = cfg.shared_intermediate_size
    per_proj = F * d // 2 + F * d // 32
    gate_up = unique * 2 * per_proj + 2 * Fs * d * 2 + M * d * 2 + (M * k * F + M * Fs) * 2
    down = unique * per_proj + Fs * d * 2 + (M * k * F + M * Fs) * 2 + (M * k * d + M * d) * 2
    router = E * d * 4 + E * 4 + M * d * 2 + M * E * 4
    combine = (M * k * d + M * d) * 2 + M * k * 4 + M * d * 4
    layer = unique * 3 * per_proj + 3 * Fs * d * 2 + E * d * 4 + E * 4 + M * d * 2 + M * d * 4
    flops = {"gate_up": 2 * M * k * 2 * d * F, "gate_up_shared": 2 * M * 2 * d * Fs,
             "down": 2 * M * k * d * F, "down_shared": 2 * M * d * Fs, "router": 2 * M * d * E}
    flops["layer"] = sum(flops.values())
    return {"bytes": {"gate_up": gate_up, "down": down, "router": router, "combine": combine, "layer": layer},
            "flops": flops, "per_expert_bytes": 3 * per_proj}


def expert_path(cfg, M: int) -> str:
    """The routed-expert path lg_moe_forward takes for M tokens (moe_capi.cu):
    decode chain (M <= 4), CUDA-core grouped GEMV (5..63 tokens), tensor-core
    grouped GEMMs with E2M1 activation terms (kind::mxf4), or with the weights
    widened to bf16 (kind::f16) once experts average 128 routes."""
    if M <= 4:
        return "decode"
    if M < 64:
        return "gemv"
    if M * cfg.num_experts_per_tok >= 128 * cfg.n_routed_experts:
        return "bf16"
    return "mxf4"


def kernels_per_layer(M: int, path: str, ep: bool = False, native_ep: bool = False,
                      shared_dq: bool = False) -> int:
    """Kernels of this library launched by one layer call (lg_moe_forward, or
    the expert-parallel layer's entry points)."""
    if ep:
        # router logits, select, histogram, dispatch, send-buffer pack, shared
        # gate/up and down (plus its chunk and SwiGLU tables on the
        # widened-weight kernel), then on the received rows: histogram,
        # dispatch, route chunks, SwiGLU table, row gather, routed gate/up,
        # routed down; finally the merge through the inverse permutation.  The
        # C call adds the exchange-id renumbering and the count message.
        return 15 + (2 if shared_dq else 0) + (2 if native_ep else 0)
    if M == 1:
        return 6  # router logits, select+dispatch, gate/up, activation split, tensor-core down, combine
    if path == "decode":
        return 5
    if path == "mxf4":
        # router logits, select, dispatch, route tiles, inverse permutation,
        # route split, routed / shared gate/up, routed / shared down, combine
        return 11
    if path == "bf16":
        # router logits, select, dispatch, route chunks, SwiGLU table, token
        # gather, routed / shared gate/up, routed / shared down, combine
        return 11
    return 6  # router logits, select, dispatch, gate/up GEMV, down GEMV, combine


# -------------------------------------------------------------- CPU side ---

def cpu_sample(cfg, tn: dict, x_bits, tokens_per_call: int, budget_s: float) -> dict:
    """Layer-tokens/s of the CPU restatement of the reference path on the host
    cores (oracle/experts_ref.c + router_ref.c: MXFP4 decoded on the fly,
    OpenMP over all host threads): calls of `tokens_per_call` tokens through
    one layer until the budget is spent (at least two calls)."""
    from oracle import moe_oracle as mo

    n_threads = os.cpu_count() or 1
    n = max(1, tokens_per_call)
    mo.moe_forward_c(x_bits[:n], tn, cfg)  # warm caches / build
    t0 = time.perf_counter()
    calls = 0
    while True:
        mo.moe_forward_c(x_bits[:n], tn, cfg)
        calls += 1
        el = time.perf_counter() - t0
        if (el >= budget_s and calls >= 2) or calls >= 10_000:
            break
    return {"value": calls * n / el, "unit": "tokens/s", "cores": n_threads, "kind": "port",
            "sample": f"{calls} calls of {n} token(s) through one cfg1-shaped layer with the C restatement "
                      f"(E2M1/E8M0 decoded on the fly, OpenMP threads={n_threads}), {el:.1f} s"}


CPU_TOKENS_PER_CALL = 128  # the CPU arm's bounded sample of a batched workload


def run_reference(args) -> None:
    """--impl reference: the CPU restatement of the reference path, rank 0."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch

    from livglm_b200 import synthetic
    from livglm_b200.config import CONFIGS
    from oracle import moe_oracle as mo
    from oracle.torch_bridge import bank_to_numpy

    wl = WORKLOADS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = CONFIGS[wl["cfg"]]
    M = wl["M"]
    n = min(M, CPU_TOKENS_PER_CALL)  # tokens per CPU call: a bounded sample of the workload
    t = synthetic.layer_weights(cfg, seed=0, device="cpu")
    tn = bank_to_numpy(t)
    x = mo.f32_to_bf16_bits(np.random.default_rng(0).standard_normal((n, cfg.hidden_size)).astype(np.float32))
    mo.moe_forward_c(x, tn, cfg)
    budget = 60.0
    times = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        mo.moe_forward_c(x, tn, cfg)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget:
            break
    el = sum(times)
    value = len(times) * n / el
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup, "ms_per_step": 1e3 * el / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "M": M, "hidden_size": cfg.hidden_size,
                   "n_routed_experts": cfg.n_routed_experts, "num_experts_per_tok": cfg.num_experts_per_tok,
                   "moe_intermediate_size": cfg.moe_intermediate_size},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{len(times)} calls of {n} tokens through one layer of the C "
                                   "restatement of kg36/livglm moe.py/expert_ssd.py/layers.py (E2M1/E8M0 "
                                   f"decoded on the fly, OpenMP threads={cores}; MLX, the reference's own "
                                   "runtime, is not installable here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU side ---

def setup_dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, local, dev


def timed_region(run_steps, steps: int, warmup: int, world: int, sampler=None, per_step: list | None = None) -> float:
    """Device time (ms, max over ranks) of exactly `steps` steps after
    `warmup` untimed ones, bracketed by a barrier and synchronisation.  With
    `per_step` (a list), the device time of each step on this rank is appended
    (events recorded between the steps on the same stream)."""
    import torch
    import torch.distributed as dist

    run_steps(warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler is not None:
        sampler.__enter__()
        time.sleep(0.2)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)] if per_step is not None else None
    ev0.record()
    run_steps(steps, marks)
    ev1.record()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.__exit__(None, None, None)
    ms = ev0.elapsed_time(ev1)
    if marks:
        prev = ev0
        for m in marks:
            per_step.append(prev.elapsed_time(m))
            prev = m
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def build_layers(args, wl, cfg, world, rank, dev, M_rank):
    """The workload's layers on this rank: single-GPU ExpertSSDMoE layers, or
    ExpertParallelMoE layers holding E / world local experts."""
    from livglm_b200 import synthetic, workloads
    from livglm_b200.moe import build_layer

    bias = workloads.cfg4_bias(dev) if wl.get("zipf") else None
    ep = world > 1 and (wl["kind"] == "stack" or bool(wl.get("zipf")))
    layers = []
    comm = None
    if ep and args.ep_impl == "native":
        from livglm_b200.ep import EpCommunicator

        comm = EpCommunicator(max_tokens=M_rank)
    for i in range(args.layers):
        if ep:
            from livglm_b200.ep import ExpertParallelMoE

            per = cfg.n_routed_experts // world
            t = synthetic.layer_weights(cfg, layer=i, seed=0, device=dev, router_bias=bias, experts=per,
                                        expert_seed=1 + rank)
            layers.append(ExpertParallelMoE(cfg, i, t, comm=comm))
        else:
            t = synthetic.layer_weights(cfg, layer=i, seed=rank, device=dev, router_bias=bias)
            layer = build_layer(cfg, t, layer_idx=i)
            if wl.get("site"):
                from livglm_b200.ffn_site import HcConfig, HyperConnection, MoEFFNSite

                sw = synthetic.ffn_site_weights(cfg, wl["site"], layer=i, seed=rank, device=dev)
                hc = HyperConnection(HcConfig(hc_mult=wl["site"]), cfg.hidden_size)
                hc.fn, hc.base, hc.scale = sw["fn"], sw["base"], sw["scale"]
                layer = MoEFFNSite(layer, hc, sw["norm_weight"])
            layers.append(layer)
        del t
    return layers, ep


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from livglm_b200 import _native, synthetic, workloads
    from livglm_b200.config import CONFIGS
    from livglm_b200.stack import MoEStack

    wl = WORKLOADS[args.workload]
    world, rank, local, dev = setup_dist()
    cfg = CONFIGS[wl["cfg"]]
    _native.load()
    stack_kind = wl["kind"] == "stack"
    M = wl["M"]
    if wl.get("zipf") and world > 1:
        M = wl["M"] // world  # config 4: the 16384 tokens split over the ranks
    layers, ep = build_layers(args, wl, cfg, world, rank, dev, M)
    L = len(layers)
    if wl.get("site"):
        xs = [synthetic.streams(cfg, M, wl["site"], seed=1000 * rank + i, device=dev) for i in range(L)]
    else:
        xs = [synthetic.hidden_states(cfg, M, seed=1000 * rank + i, device=dev)
              for i in range(1 if stack_kind else L)]
    torch.cuda.synchronize()

    # routing statistics of one call (distinct experts, load per expert)
    idx = layers[0](xs[0], return_route=True)[2]
    U = float(len(set(idx.view(torch.int32).reshape(-1).tolist())))
    stats = workloads.load_stats(idx, cfg.n_routed_experts)

    stack = MoEStack(layers) if stack_kind else None
    use_graph = not ep

    def forward(i: int):
        return stack(xs[0]) if stack_kind else layers[i % L](xs[i % L])

    # one CUDA graph per step shape (eager under expert parallelism: the
    # exchange sizes reach the host every layer)
    graphs = []
    if use_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for i in range(1 if stack_kind else L):
                forward(i)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        for i in range(1 if stack_kind else L):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                forward(i)
            graphs.append(g)
        torch.cuda.synchronize()

    def run_steps(n: int, marks=None) -> None:
        for i in range(n):
            if use_graph:
                graphs[i % len(graphs)].replay()
            else:
                forward(i)
            if marks:
                marks[i].record()

    sampler = ClockSampler(local)
    step_times: list = []
    ms = timed_region(run_steps, args.steps, args.warmup, world, sampler, per_step=step_times)
    ms_step = ms / args.steps
    layers_per_step = L if stack_kind else 1
    value = world * M * layers_per_step * args.steps / (ms * 1e-3)
    del graphs

    # per-stage device times of one layer (single GPU; the stages serialise
    # under the trace events)
    stage = {}
    if world == 1:
        _native.trace_enable(4)
        for _ in range(4):
            layers[0](xs[0])
        torch.cuda.synchronize()
        st = _native.trace_read(4)
        _native.trace_enable(0)
        stage = {k: statistics.fmean(s_[k] for s_ in st) for k in _native.TRACE_STAGES}

    # ---- e2e: the public call with the tokens and the result on the host ----
    x_host = torch.empty(xs[0].shape, dtype=torch.bfloat16, pin_memory=True)
    x_host.copy_(xs[0].cpu())
    out_host = torch.empty(xs[0].shape, dtype=torch.float32, pin_memory=True)
    x_dev = torch.empty_like(xs[0])
    K_e2e = max(1, min(args.steps, 2000))

    # decode calls take the tokens and the result in page-locked host memory
    # (ExpertSSDMoE's host-buffer form: the library's kernels read the tokens
    # once from host memory and write the f32 result there); other workloads
    # copy around the call
    host_io = (not stack_kind) and (not ep) and (not wl.get("site")) and M <= 4

    def e2e_steps(n: int, marks=None) -> None:
        for i in range(n):
            if host_io:
                layers[i % L](x_host, out=out_host)
                continue
            x_dev.copy_(x_host, non_blocking=True)
            y = stack(x_dev) if stack_kind else layers[i % L](x_dev)
            out_host.copy_(y, non_blocking=True)

    ms_e2e = timed_region(e2e_steps, K_e2e, max(3, args.warmup), world)

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.torch_bridge import bank_to_numpy, to_numpy

        t0 = synthetic.layer_weights(cfg, layer=0, seed=0, device=dev)
        tn = bank_to_numpy(t0)
        del t0
        n_cpu = min(M, CPU_TOKENS_PER_CALL)
        cpu = cpu_sample(cfg, tn, to_numpy(synthetic.hidden_states(cfg, n_cpu, seed=0, device=dev)), n_cpu,
                         args.cpu_seconds)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = measured_peaks()
    fp4 = fp4_peak_tflops()
    work = layer_work(cfg, M, U)
    # the local experts of an expert-parallel rank see about M*k routes over E/world experts
    path = expert_path(cfg.replace(n_routed_experts=cfg.n_routed_experts // world, num_experts_per_tok=1),
                       M * cfg.num_experts_per_tok) if ep else expert_path(cfg, M)
    # tensor peak of the MMA kind the path runs: kind::f16 (bf16) for the
    # widened weights, kind::mxf4 (FP4) for the E2M1-term path
    if path == "bf16":
        tc_peak = {"tflops": peaks["bf16_tflops"], "source": f"{peaks['source']} (bf16 tensor, cuBLAS)"}
    else:
        tc_peak = fp4
    # dominant stage and its roofline: the larger of its HBM and tensor times
    if stage:
        dominant = max(stage, key=stage.get)
        dom_ms = stage[dominant]
    else:
        dominant, dom_ms = "layer", ms_step / layers_per_step
    dom_bytes = work["bytes"].get(dominant, work["bytes"]["layer"])
    dom_flops = {"gate_up": work["flops"]["gate_up"] + work["flops"]["gate_up_shared"],
                 "down": work["flops"]["down"] + work["flops"]["down_shared"],
                 "router": work["flops"]["router"]}.get(dominant, work["flops"]["layer"])
    t_hbm = dom_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tc = dom_flops / (tc_peak["tflops"] * 1e12)
    if t_tc > t_hbm:
        bound, achieved, peak, unit = "tensor", dom_flops / (dom_ms * 1e-3) / 1e12, tc_peak["tflops"], "TFLOP/s"
    else:
        bound, achieved, peak, unit = "hbm", dom_bytes / (dom_ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
    layer_ms = ms_step / layers_per_step
    layer_t_hbm = work["bytes"]["layer"] / (peaks["hbm_gbs"] * 1e9)
    layer_t_tc = work["flops"]["layer"] / (tc_peak["tflops"] * 1e12)
    workload_name = {"cfg3": f"cfg3: {L} stacked layers, M={M} per rank",
                     "cfg4": f"cfg4: Zipf(1.2) bias, M={M} per rank",
                     "prefill256": "cfg2: M=256", "decode1": "cfg1: M=1", "decode2": "cfg1: M=2 (MTP verify)",
                     "site2": "cfg1: M=2 (MTP verify) at the FFN site: hyper-connections of 4 bf16 streams, "
                              "RMSNorm, MoE block, hyper-residual (model.py:132-136)"}
    routed_gb = L * work["per_expert_bytes"] * cfg.n_routed_experts / world / 1e9
    line = {
        "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if (wl.get("zipf") and world > 1) else "weak", "vs_baseline": None,
        "dtype": {"mxf4": "mxf4 (E2M1 weights x E2M1-term activations), f32 accumulate",
                  "bf16": "bf16 x bf16 (MXFP4 weights widened exactly to bf16 in shared memory), f32 accumulate",
                  }.get(path, "fp4 weights x f16/bf16 activations, f32 accumulate"),
        "data": "synthetic (seeded N(0,1) bf16 tokens; N(0,0.02) weights, routed MXFP4 g32, shared bf16)",
        "config": {"workload": workload_name[args.workload], "M": M, "layers_per_step": layers_per_step,
                   "hidden_size": cfg.hidden_size, "n_routed_experts": cfg.n_routed_experts,
                   "num_experts_per_tok": cfg.num_experts_per_tok, "n_group": cfg.n_group,
                   "topk_group": cfg.topk_group, "moe_intermediate_size": cfg.moe_intermediate_size,
                   "graph": "one CUDA graph per step, replayed" if use_graph else "eager (expert-parallel)",
                   "l2": f"inputs larger than L2: {L} distinct layers, {routed_gb:.1f} GB of routed weights per GPU",
                   "parallelism": (f"expert-parallel x{world} ({cfg.n_routed_experts // world} experts/GPU, NCCL "
                                   "all-to-all)") if ep else (f"replicas x{world}" if world > 1 else "single GPU")},
        "roofline": {"bound": bound, "kernel": f"{dominant} stage", "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak if peak else None,
                     # captured on one GPU; the expert-parallel ranks run other shapes
                     "traffic": MEASURED_TRAFFIC.get(args.workload) if dominant == "gate_up" and world == 1 else None,
                     "peak_source": peaks["source"] if unit == "GB/s" else tc_peak["source"],
                     "algorithmic_bytes_per_launch": dom_bytes, "algorithmic_flops_per_launch": dom_flops,
                     "launch_ms": dom_ms,
                     # the bf16 GEMM peak measured over seconds at the power cap, for a
                     # stage timed right after the long timed region
                     "peak_sustained": (peaks["bf16_tflops_sustained"]
                                        if unit == "TFLOP/s" and path == "bf16" else None),
                     "frac_sustained": (achieved / peaks["bf16_tflops_sustained"]
                                        if unit == "TFLOP/s" and path == "bf16"
                                        and peaks.get("bf16_tflops_sustained") else None)},
        "e2e": {"value": world * M * layers_per_step * K_e2e / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 4,
                "steps": K_e2e,
                "path": ("pinned host tokens read by the public module call's kernels, f32 result written to "
                         "pinned host memory, every step" if host_io else
                         "pinned host tokens -> device copy -> public module call(s) -> f32 result copied to "
                         "pinned host memory, every step")},
        "gpu_launches": (kernels_per_layer(M, path, ep, ep and args.ep_impl == "native",
                                           M * cfg.num_experts_per_tok >= 128 * cfg.n_routed_experts)
                         + (3 if wl.get("site") else 0))  # hyper-connection mix, finish, residual
                        * layers_per_step * args.steps,
        "clocks": sampler.summary(),
        "extra": {"layer_ms": layer_ms,
                  "expert_path": path,
                  "ep_impl": args.ep_impl if ep else None,
                  "layer_roofline": {"hbm_us": layer_t_hbm * 1e6, "tensor_us": layer_t_tc * 1e6,
                                     "frac": max(layer_t_hbm, layer_t_tc) / (layer_ms * 1e-3),
                                     "hbm_frac": layer_t_hbm / (layer_ms * 1e-3),
                                     "tensor_frac": layer_t_tc / (layer_ms * 1e-3),
                                     "fp4_frac": work["flops"]["layer"] / (fp4["tflops"] * 1e12) / (layer_ms * 1e-3)},
                  "layer_bytes": work["bytes"]["layer"], "layer_flops": work["flops"]["layer"],
                  "fp4_peak_tflops": fp4["tflops"], "fp4_peak_source": fp4["source"],
                  "bf16_peak_tflops": peaks["bf16_tflops"],
                  "unique_experts_per_call": U, "stage_ms": stage,
                  "step_ms": ({"median": statistics.median(step_times),
                               "p99": sorted(step_times)[min(len(step_times) - 1, int(0.99 * len(step_times)))],
                               "min": min(step_times), "max": max(step_times), "rank": 0}
                              if step_times else None),
                  "stack_tokens_per_s": world * M * args.steps / (ms * 1e-3) if stack_kind else None,
                  "load": {k: v for k, v in stats.items() if k != "counts"},
                  "expert_counts": stats["counts"] if wl.get("zipf") else None},
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
