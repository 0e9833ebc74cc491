"""Seeded synthetic inputs and weights for the MoE block.

No checkpoint or dataset is reachable from this build, so every workload uses
generated tensors with the distributions of the benchmark plan:
hidden states bf16 N(0,1); router weight f32 N(0,0.02); correction bias
U(-0.01,0.01); routed gate/up/down f32 N(0,0.02) quantised to MXFP4 g32;
shared expert bf16 N(0,0.02).  Each tensor has its own torch.Generator seeded
from (seed, layer, tensor id), so any tensor can be regenerated alone.
Generation runs on the target device (CUDA for full-size layers).
"""

from __future__ import annotations

import torch

from .config import MoEConfig
from .mxfp4 import quantize_mxfp4

_TENSOR_IDS = {
    "hidden": 1, "router_weight": 2, "router_bias": 3, "gate": 4, "up": 5, "down": 6,
    "shared_gate": 7, "shared_up": 8, "shared_down": 9,
    "streams": 10, "hc_fn": 11, "hc_base": 12, "norm_weight": 13,
}


def _gen(device, seed: int, layer: int, name: str) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + layer * 10_007 + _TENSOR_IDS[name]) & 0x7FFF_FFFF_FFFF_FFFF)
    return g


def hidden_states(cfg: MoEConfig, tokens: int, *, seed: int = 0, device="cuda") -> torch.Tensor:
    g = _gen(device, seed, 0, "hidden")
    return torch.randn(tokens, cfg.hidden_size, generator=g, device=device).to(torch.bfloat16)


def streams(cfg: MoEConfig, tokens: int, hc_mult: int, *, seed: int = 0, device="cuda") -> torch.Tensor:
    """Hyper-connection residual streams: bf16 N(0,1) [tokens, hc_mult, d]."""
    g = _gen(device, seed, 0, "streams")
    return torch.randn(tokens, hc_mult, cfg.hidden_size, generator=g, device=device).to(torch.bfloat16)


def ffn_site_weights(cfg: MoEConfig, hc_mult: int, *, layer: int = 0, seed: int = 0, device="cuda") -> dict:
    """The FFN site's hyper-connection and norm tensors (no checkpoint values
    are reachable): fn f32 N(0, 1/(hc*d)) so the mixed logits are O(1) on
    RMS-normalised streams, base f32 U(-0.2, 0.2), scale (0.5, 0.75, 1.25),
    post-attention norm weight bf16 1 + N(0, 0.1)."""
    d, R = cfg.hidden_size, hc_mult * (hc_mult + 2)
    K = hc_mult * d
    fn = torch.randn(R, K, generator=_gen(device, seed, layer, "hc_fn"), device=device) / K ** 0.5
    base = torch.rand(R, generator=_gen(device, seed, layer, "hc_base"), device=device) * 0.4 - 0.2
    norm = 1 + 0.1 * torch.randn(d, generator=_gen(device, seed, layer, "norm_weight"), device=device)
    return {"fn": fn.contiguous(), "base": base.contiguous(),
            "scale": torch.tensor([0.5, 0.75, 1.25], dtype=torch.float32, device=device),
            "norm_weight": norm.to(torch.bfloat16).contiguous()}


def layer_weights(cfg: MoEConfig, *, layer: int = 0, seed: int = 0, device="cuda",
                  expert_chunk: int = 16, router_bias: torch.Tensor | None = None,
                  experts: int | None = None, expert_seed: int | None = None) -> dict:
    """One MoE layer's tensors, stacked per expert (the HBM bank layout).

    experts / expert_seed: generate routed banks for only that many experts,
    from their own seed (an expert-parallel rank's local slice; the router and
    shared expert still follow `seed`, so every rank holds the same ones)."""
    d, F, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts
    n_banks = E if experts is None else experts
    bank_seed = seed if expert_seed is None else expert_seed
    Fs = cfg.shared_intermediate_size
    out: dict[str, torch.Tensor] = {}
    g = _gen(device, seed, layer, "router_weight")
    out["router_weight"] = torch.randn(E, d, generator=g, device=device) * 0.02
    if router_bias is None:
        g = _gen(device, seed, layer, "router_bias")
        router_bias = (torch.rand(E, generator=g, device=device) * 0.02 - 0.01)
    out["router_bias"] = router_bias.to(device=device, dtype=torch.float32).contiguous()
    for proj, rows, cols in (("gate", F, d), ("up", F, d), ("down", d, F)):
        packed = torch.empty(n_banks, rows, cols // 2, dtype=torch.uint8, device=device)
        scale = torch.empty(n_banks, rows, cols // 32, dtype=torch.uint8, device=device)
        g = _gen(device, bank_seed, layer, proj)
        for e0 in range(0, n_banks, expert_chunk):
            e1 = min(n_banks, e0 + expert_chunk)
            w = torch.randn(e1 - e0, rows, cols, generator=g, device=device) * 0.02
            packed[e0:e1], scale[e0:e1] = quantize_mxfp4(w)
            del w
        out[f"{proj}_packed"] = packed
        out[f"{proj}_scale"] = scale
    if Fs > 0:
        for name, rows, cols in (("shared_gate", Fs, d), ("shared_up", Fs, d), ("shared_down", d, Fs)):
            g = _gen(device, seed, layer, name)
            out[name] = (torch.randn(rows, cols, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return out


def zipf_bias(cfg: MoEConfig, *, s: float = 1.2, beta: float = 1.0, device="cuda") -> torch.Tensor:
    """Correction bias beta * log(p_e) for a Zipf(s) popularity over experts
    (rank order = expert id).  Calibrate beta against measured popularity."""
    ranks = torch.arange(1, cfg.n_routed_experts + 1, dtype=torch.float64)
    p = ranks ** (-s)
    p = p / p.sum()
    return (beta * torch.log(p)).to(torch.float32).to(device)
