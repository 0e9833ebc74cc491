"""Torch <-> NumPy conversions for feeding the CPU oracle -- TEST INFRASTRUCTURE ONLY.

bf16 tensors become uint16 bit patterns (the oracle's bf16 representation);
uint32 tensors become uint32 arrays.
"""

from __future__ import annotations

import numpy as np
import torch

BF16_KEYS = ("x", "shared_gate", "shared_up", "shared_down")
BANK_KEYS = ("router_weight", "router_bias", "gate_packed", "gate_scale", "up_packed", "up_scale",
             "down_packed", "down_scale", "shared_gate", "shared_up", "shared_down")


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


def to_device(a: np.ndarray, device, bf16: bool = False) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if bf16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(device).view(torch.uint32)
    return torch.from_numpy(a).to(device)


def bank_to_numpy(tensors: dict) -> dict:
    return {k: to_numpy(v) for k, v in tensors.items()}


def bank_to_device(arrays: dict, device) -> dict:
    return {k: to_device(arrays[k], device, bf16=k in BF16_KEYS) for k in BANK_KEYS if k in arrays}
