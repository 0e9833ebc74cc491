"""Near-tie statistics of the router at config-4 scale: how many top-k
selections of the canonical f32 router arithmetic (oracle/router_ref.c, which
the CUDA router matches bit-for-bit) differ from a float64 evaluation of
TopKRouter.__call__ (kg36/livglm src/glm53flash/moe.py:36-63).

    python tests/golden/near_ties.py [tokens]   # default 16384; writes near_ties_cfg4.json

MLX evaluates the router in f32 with its own summation order and sigmoid, so
neither the canonical arithmetic nor float64 is the reference's exact result;
the float64 evaluation is the order-free value both approximate.  A token
whose selected expert set differs between the two is one whose k-th and
(k+1)-th choices (or the kept groups) lie within f32 rounding of each other:
the size of the routing risk against the real reference.

Inputs: config 4's layer with its committed Zipf(1.2) correction bias
(livglm_b200/data/cfg4_zipf_bias.json), router weight f32 N(0, 0.02) and bf16
N(0, 1) tokens from NumPy generators (SeedSequence([4, id])).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from livglm_b200.config import CONFIGS  # noqa: E402
from livglm_b200.workloads import CFG4_BIAS_PATH, CFG4_TOKENS  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402

OUT = Path(__file__).resolve().parent / "near_ties_cfg4.json"


def router_f64(x_bits: np.ndarray, W: np.ndarray, bias: np.ndarray, cfg):
    """moe.py:36-63 in float64 -> (scores [M,E], choice [M,E] after the group
    mask, indices [M,k] best first)."""
    x = mo.bf16_bits_to_f32(x_bits).astype(np.float64)
    logits = x @ W.astype(np.float64).T
    scores = 1.0 / (1.0 + np.exp(-logits))
    choice = scores + bias.astype(np.float64)
    M, E = choice.shape
    G, g, k = cfg.n_group, cfg.topk_group, cfg.num_experts_per_tok
    grouped = choice.reshape(M, G, E // G)
    top2 = np.sort(grouped, axis=-1)[..., -2:].sum(-1)
    keep = np.argsort(top2, axis=-1, kind="stable")[:, -g:]
    mask = np.zeros((M, G), bool)
    np.put_along_axis(mask, keep, True, axis=-1)
    choice = np.where(np.repeat(mask, E // G, axis=1), choice, -np.inf)
    idx = np.argsort(choice, axis=-1, kind="stable")[:, ::-1][:, :k]
    return scores, choice, idx


def inputs(cfg, tokens: int):
    d, E = cfg.hidden_size, cfg.n_routed_experts
    rng = lambda i: np.random.default_rng(np.random.SeedSequence([4, i]))  # noqa: E731
    W = (rng(2).standard_normal((E, d)) * 0.02).astype(np.float32)
    bias = np.asarray(json.loads(CFG4_BIAS_PATH.read_text())["bias"], np.float32)
    x = mo.f32_to_bf16_bits(rng(100).standard_normal((tokens, d)).astype(np.float32))
    return x, W, bias


def stats(tokens: int) -> dict:
    cfg = CONFIGS["cfg4"]
    x, W, bias = inputs(cfg, tokens)
    _, _, idx32 = mo.router(x, W, bias, cfg)
    _, choice64, idx64 = router_f64(x, W, bias, cfg)
    set32 = np.sort(idx32.astype(np.int64), axis=1)
    set64 = np.sort(idx64, axis=1)
    differ = np.any(set32 != set64, axis=1)
    # margin of the f64 selection: gap between the k-th and (k+1)-th masked choice
    srt = np.sort(choice64, axis=1)[:, ::-1]
    k = cfg.num_experts_per_tok
    gap = srt[:, k - 1] - srt[:, k]
    return {
        "tokens": int(tokens), "routes": int(tokens * k),
        "tokens_with_different_expert_set": int(differ.sum()),
        "fraction_of_tokens": float(differ.mean()),
        "routes_differing": int(sum(len(set(a) ^ set(b)) // 2 for a, b in zip(set32[differ], set64[differ]))),
        "tokens_with_kth_gap_below_1e-6": int((gap < 1e-6).sum()),
        "tokens_with_kth_gap_below_1e-7": int((gap < 1e-7).sum()),
        "median_kth_gap": float(np.median(gap)),
    }


def main() -> None:
    tokens = int(sys.argv[1]) if len(sys.argv) > 1 else CFG4_TOKENS
    s = stats(tokens)
    OUT.write_text(json.dumps(s, indent=1) + "\n")
    print(json.dumps(s, indent=1))


if __name__ == "__main__":
    main()
