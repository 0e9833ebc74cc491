"""Workloads of the benchmark plan beyond one layer call.

config 3  42 MoE layers of config 1's shapes in sequence (stack.py), M = 4096
          tokens, independent weights per layer; expert-parallel over W GPUs
          (ep.py) with 128 / W experts per GPU.
config 4  config 1's layer at M = 16384 tokens with the correction bias set so
          that expert popularity follows Zipf(s = 1.2) over the 128 experts:
          the skewed-routing stress case of the grouped GEMMs.

The config-4 bias is bias_e = beta * log p_e with p the Zipf(1.2) law over
expert ids (expert 0 most popular) and beta fitted by a golden-section search:
with top-k routing an expert is picked at most once per token, so the
popularity that can be matched is the per-token selection probability, whose
Zipf target is k * p_e water-filled under the cap 1 (sum k).  The fit routes a
seeded calibration batch with a float32 torch restatement of the router
(sigmoid scores, group-limited top-k; the kernels' canonical arithmetic is not
needed to measure popularity) and minimises the L1 distance between measured
and target selection frequencies.  livglm_b200/data/make_cfg4_bias.py writes
the fitted bias to livglm_b200/data/cfg4_zipf_bias.json.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import torch

from .config import CONFIGS, MoEConfig

DATA = Path(__file__).resolve().parent / "data"
CFG4_BIAS_PATH = DATA / "cfg4_zipf_bias.json"
CFG3_LAYERS = 42
CFG3_TOKENS = 4096
CFG4_TOKENS = 16384
ZIPF_S = 1.2


def zipf_law(E: int, s: float = ZIPF_S) -> torch.Tensor:
    p = torch.arange(1, E + 1, dtype=torch.float64) ** (-s)
    return p / p.sum()


def zipf_selection_target(E: int, k: int, s: float = ZIPF_S) -> torch.Tensor:
    """Per-token selection probability of each expert: k * p water-filled
    under the cap 1 so that it sums to k."""
    p = zipf_law(E, s)
    q = torch.zeros(E, dtype=torch.float64)
    free = torch.ones(E, dtype=torch.bool)
    left = float(k)
    while True:
        share = p * free / (p * free).sum() * left
        over = free & (share >= 1.0)
        if not bool(over.any()):
            q[free] = share[free]
            return q
        q[over] = 1.0
        free &= ~over
        left -= float(over.sum())


def route_torch(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor, cfg: MoEConfig) -> torch.Tensor:
    """Expert ids [M, k] chosen by the router of kg36/livglm moe.py:36-58 in
    float32 torch arithmetic (workload calibration only)."""
    scores = torch.sigmoid(x.float() @ W.float().T)
    choice = scores + bias.float()
    M, E = choice.shape
    G, g, k = cfg.n_group, cfg.topk_group, cfg.num_experts_per_tok
    grouped = choice.view(M, G, E // G)
    gscore = grouped.topk(2, dim=-1).values.sum(-1)
    keep = gscore.topk(g, dim=-1).indices
    mask = torch.zeros(M, G, dtype=torch.bool, device=x.device)
    mask.scatter_(1, keep, True)
    choice = choice.masked_fill(~mask.repeat_interleave(E // G, dim=1), float("-inf"))
    return choice.topk(k, dim=-1).indices


def selection_frequency(indices: torch.Tensor, E: int) -> torch.Tensor:
    """Fraction of tokens that picked each expert."""
    return torch.bincount(indices.reshape(-1).long(), minlength=E).double() / indices.shape[0]


def load_stats(indices: torch.Tensor, E: int) -> dict:
    """Per-expert route counts and their imbalance (max / mean, p50, p99)."""
    c = torch.bincount(indices.reshape(-1).long().cpu(), minlength=E).double()
    mean = float(c.mean())
    srt = torch.sort(c).values
    return {"counts": [int(v) for v in c.tolist()], "max_over_mean": float(c.max()) / mean if mean else 0.0,
            "p50": float(srt[len(srt) // 2]), "p99": float(srt[min(len(srt) - 1, int(0.99 * len(srt)))]),
            "experts_used": int((c > 0).sum())}


def calibrate_zipf_bias(cfg: MoEConfig | None = None, *, s: float = ZIPF_S, tokens: int = 4096, seed: int = 4,
                        lo: float = 0.0, hi: float = 0.5, iters: int = 40) -> dict:
    """Fit beta of bias = beta * log(Zipf(s)) on a seeded calibration batch
    (router weight N(0, 0.02), tokens N(0, 1), generated on the CPU)."""
    cfg = cfg or CONFIGS["cfg4"]
    E, k, d = cfg.n_routed_experts, cfg.num_experts_per_tok, cfg.hidden_size
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(E, d, generator=g) * 0.02
    x = torch.randn(tokens, d, generator=g).to(torch.bfloat16).float()
    logp = torch.log(zipf_law(E, s)).float()
    target = zipf_selection_target(E, k, s)

    def loss(beta: float) -> float:
        idx = route_torch(x, W, beta * logp, cfg)
        return float((selection_frequency(idx, E) - target).abs().sum())

    invphi = (math.sqrt(5.0) - 1.0) / 2.0
    a, b = lo, hi
    c1, c2 = b - invphi * (b - a), a + invphi * (b - a)
    f1, f2 = loss(c1), loss(c2)
    for _ in range(iters):
        if f1 <= f2:
            b, c2, f2 = c2, c1, f1
            c1 = b - invphi * (b - a)
            f1 = loss(c1)
        else:
            a, c1, f1 = c1, c2, f2
            c2 = a + invphi * (b - a)
            f2 = loss(c2)
    beta = (a + b) / 2.0
    idx = route_torch(x, W, beta * logp, cfg)
    freq = selection_frequency(idx, E)
    return {"s": s, "beta": beta, "l1_to_target": float((freq - target).abs().sum()),
            "bias": (beta * logp).tolist(), "calibration": {"tokens": tokens, "seed": seed},
            "measured_selection": freq.tolist(), "target_selection": target.tolist(),
            "stats": load_stats(idx, E)}


def cfg4_bias(device="cuda") -> torch.Tensor:
    """The committed config-4 correction bias (f32 [E])."""
    data = json.loads(CFG4_BIAS_PATH.read_text())
    return torch.tensor(data["bias"], dtype=torch.float32, device=device)
