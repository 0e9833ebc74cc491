"""A small GLM-layout checkpoint for loader tests (test infrastructure):
config 0's committed layer (tests/golden/cfg0.npz) written under the
checkpoint's tensor names, with the shared expert stored as block-FP8
(E4M3FN bytes + f32 128x128 block scales, as the official checkpoint stores
it), split over two shards with an index."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import moe_oracle as mo
from tests import st_writer

LAYER = 3


def fp8_weight(rng, rows: int, cols: int, block: int = 128):
    """Random finite E4M3FN bytes (never 0x7F / 0xFF) and block scales near 2^-8."""
    w = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] ^= 0x01  # NaN codes -> the largest finite magnitude
    s = (2.0 ** rng.integers(-10, -6, (rows // block, cols // block))).astype(np.float32)
    s *= rng.uniform(0.75, 1.25, s.shape).astype(np.float32)
    return w, s


def build(directory: Path, golden: dict, cfg, seed: int = 5) -> dict:
    """Write the checkpoint; returns the oracle's bank for the same layer
    (shared expert = the FP8 weights widened by the oracle)."""
    rng = np.random.default_rng(seed)
    E = cfg.n_routed_experts
    p = f"model.language_model.layers.{LAYER}.mlp."
    resident = {p + "gate.weight": ("F32", golden["router_weight"]),
                p + "gate.e_score_correction_bias": ("F32", golden["router_bias"])}
    bank = {k: golden[k] for k in ("router_weight", "router_bias", "gate_packed", "gate_scale", "up_packed",
                                   "up_scale", "down_packed", "down_scale")}
    d, Fs = cfg.hidden_size, cfg.shared_intermediate_size
    for name, rows, cols in (("gate_proj", Fs, d), ("up_proj", Fs, d), ("down_proj", d, Fs)):
        w, s = fp8_weight(rng, rows, cols)
        resident[p + f"shared_experts.{name}.weight"] = ("F8_E4M3", w)
        resident[p + f"shared_experts.{name}.weight_scale_inv"] = ("F32", s)
        bank["shared_" + name.split("_")[0]] = mo.fp8_block_dequant_bf16(w, s)
    experts = {}
    for e in range(E):
        for proj in ("gate", "up", "down"):
            for part, key in (("weight_packed", "packed"), ("weight_scale", "scale")):
                experts[p + f"experts.{e}.{proj}_proj.{part}"] = ("U8", golden[f"{proj}_{key}"][e])
    st_writer.write_checkpoint(directory, {"model-00001-of-00002.safetensors": resident,
                                           "model-00002-of-00002.safetensors": experts})
    return bank
