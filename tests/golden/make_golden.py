"""Generate tests/golden/cfg0.npz: the CPU-runnable MoE layer of the
benchmark plan (d=256, 16 experts, top-4, 4 groups, top-2 groups, F=128,
one shared expert of width 128, scale 2.5, 8 tokens, seed 0), its inputs and
the CPU oracle's outputs.

    python tests/golden/make_golden.py

Inputs: bf16 N(0,1) activations; router weight f32 N(0,0.02); bias
U(-0.01,0.01); routed weights f32 N(0,0.02) -> MXFP4 g32; shared bf16
N(0,0.02).  NumPy's default_rng(SeedSequence([0, tensor_id])) per tensor.
The oracle's outputs are stored so that later oracle or kernel changes are
caught against a frozen record (the reference itself cannot run here: it
needs MLX, which is absent).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from livglm_b200.config import CONFIGS  # noqa: E402
from livglm_b200.mxfp4 import quantize_mxfp4  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402

OUT = Path(__file__).resolve().parent / "cfg0.npz"


def rng(tensor_id: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([0, tensor_id]))


def inputs(cfg, tokens: int = 8) -> dict:
    d, F, E, Fs = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts, cfg.shared_intermediate_size
    x = rng(1).standard_normal((tokens, d)).astype(np.float32)
    t = {"x": mo.f32_to_bf16_bits(x)}
    t["router_weight"] = (rng(2).standard_normal((E, d)) * 0.02).astype(np.float32)
    t["router_bias"] = rng(3).uniform(-0.01, 0.01, E).astype(np.float32)
    for i, (proj, rows, cols) in enumerate((("gate", F, d), ("up", F, d), ("down", d, F))):
        w = (rng(4 + i).standard_normal((E, rows, cols)) * 0.02).astype(np.float32)
        p, s = quantize_mxfp4(torch.from_numpy(w))
        t[f"{proj}_packed"], t[f"{proj}_scale"] = p.numpy(), s.numpy()
    for i, (name, rows, cols) in enumerate((("shared_gate", Fs, d), ("shared_up", Fs, d), ("shared_down", d, Fs))):
        w = (rng(7 + i).standard_normal((rows, cols)) * 0.02).astype(np.float32)
        t[name] = mo.f32_to_bf16_bits(w)
    return t


def main() -> None:
    cfg = CONFIGS["cfg0"]
    t = inputs(cfg)
    ref = mo.moe_forward(t["x"], t, cfg)
    counts, offsets, perm = mo.dispatch(ref["indices"], cfg.n_routed_experts)
    np.savez_compressed(
        OUT, **t,
        logits=ref["logits"], weights=ref["weights"], indices=ref["indices"],
        counts=counts, offsets=offsets, perm=perm,
        y=mo.f32_to_bf16_bits(ref["y"]), shared=mo.f32_to_bf16_bits(ref["shared"]), out=ref["out"],
    )
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
