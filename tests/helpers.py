"""Conversions between the CUDA path's torch tensors and the oracle's NumPy arrays."""

from __future__ import annotations

import numpy as np

from oracle.torch_bridge import (BF16_KEYS, bank_to_device, bank_to_numpy,  # noqa: F401
                                  to_device, to_numpy)

# Output tolerance for floating-point parity of the f32 layer output
# (max-abs and cosine against the CPU oracle on identical inputs).
MAX_ABS = 2e-2
MIN_COSINE = 0.9995


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


def assert_close(out: np.ndarray, ref: np.ndarray, *, max_abs: float = MAX_ABS,
                 min_cos: float = MIN_COSINE) -> None:
    err = float(np.max(np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64))))
    cos = cosine(out, ref)
    assert err <= max_abs and cos >= min_cos, f"max-abs {err:.3e} (<= {max_abs}), cosine {cos:.7f} (>= {min_cos})"
