"""Generate tests/golden/cfg1.npz: frozen CPU-oracle records of config 1's
layer (d=4096, 128 experts, top-8, 8 groups, top-4 groups, F=1536, one bf16
shared expert, scale 2.5) at M = 1, M = 2 and one M = 256 sample.

    python tests/golden/make_golden_cfg1.py

The layer's 1.3 GB of weights are not stored: weights(seed) redraws them from
NumPy generators in a few seconds on any host (SeedSequence([seed,
tensor_id])): routed MXFP4 bytes drawn directly (packed nibbles uniform over
all 16 codes, UE8M0 scale bytes uniform in [116, 120], i.e. magnitudes up to
6 * 2^-7), router weight f32 N(0, 0.02), bias U(-0.01, 0.01), shared bf16
N(0, 0.02).  Tokens: bf16 N(0, 1).

Stored per record: the tokens, the oracle's routing (indices, weights) for
every token and its f32 outputs for every token (M = 1, 2) or for a fixed
sample of 16 tokens (M = 256).  The reference itself cannot run here (it
needs MLX): the records freeze the oracle so later oracle or kernel changes
are caught, and they are what the GPU tests compare against.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from livglm_b200.config import CONFIGS  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402

OUT = Path(__file__).resolve().parent / "cfg1.npz"
SEED = 1
SAMPLE_256 = np.arange(0, 256, 16)  # tokens of the M = 256 record whose outputs are stored


def _rng(seed: int, tensor_id: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence([seed, tensor_id]))


def weights(cfg, seed: int = SEED) -> dict:
    """The record's layer weights (numpy, bank layout of synthetic.layer_weights)."""
    d, F, E, Fs = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts, cfg.shared_intermediate_size
    t = {"router_weight": (_rng(seed, 2).standard_normal((E, d)) * 0.02).astype(np.float32),
         "router_bias": _rng(seed, 3).uniform(-0.01, 0.01, E).astype(np.float32)}
    for i, (proj, rows, cols) in enumerate((("gate", F, d), ("up", F, d), ("down", d, F))):
        g = _rng(seed, 4 + i)
        t[f"{proj}_packed"] = g.integers(0, 256, (E, rows, cols // 2), dtype=np.uint8)
        t[f"{proj}_scale"] = g.integers(116, 121, (E, rows, cols // 32), dtype=np.uint8)
    for i, (name, rows, cols) in enumerate((("shared_gate", Fs, d), ("shared_up", Fs, d), ("shared_down", d, Fs))):
        w = (_rng(seed, 7 + i).standard_normal((rows, cols)) * 0.02).astype(np.float32)
        t[name] = mo.f32_to_bf16_bits(w)
    return t


def tokens(cfg, M: int, seed: int = SEED) -> np.ndarray:
    x = _rng(seed, 100 + M).standard_normal((M, cfg.hidden_size)).astype(np.float32)
    return mo.f32_to_bf16_bits(x)


def main() -> None:
    cfg = CONFIGS["cfg1"]
    bank = weights(cfg)
    rec = {}
    for M in (1, 2, 256):
        x = tokens(cfg, M)
        _, w, idx = mo.router(x, bank["router_weight"], bank["router_bias"], cfg)
        sel = np.arange(M) if M <= 2 else SAMPLE_256
        out = mo.moe_forward(x, bank, cfg, tokens=sel)["out"]
        rec[f"x{M}"], rec[f"weights{M}"], rec[f"indices{M}"] = x, w, idx
        rec[f"sel{M}"], rec[f"out{M}"] = sel.astype(np.int64), out
    np.savez_compressed(OUT, **rec)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
