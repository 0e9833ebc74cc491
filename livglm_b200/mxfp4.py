"""OCP-MX MXFP4 (group 32) encoding used to synthesise expert records.

The reference reads experts that were already quantised (INCModel3 AutoRound
records, kg36/livglm README.md:1-16) and quantises resident weights with
mx.quantize(mode="mxfp4", group_size=32) (layers.py:89-94).  Benchmarks
here need synthetic records of the same byte layout:

  weight_packed U8 [rows, cols/2]  E2M1 nibbles, low nibble = even column
  weight_scale  U8 [rows, cols/32] E8M0, value = 2^(s-127)

(expert_source.py:189-229).  The quantiser follows the OCP MX v1.0 recipe:
shared exponent floor(log2(amax)) - 2 (E2M1's largest exponent), elements
rounded to nearest-even on the E2M1 grid and saturated at +-6.  Its bytes
are inputs to both the CUDA path and the checker, so its rounding choices do
not affect parity.  Works on any torch device.
"""

from __future__ import annotations

import torch

E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def quantize_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[..., rows, cols] float -> (packed u8 [..., rows, cols/2], scale u8 [..., rows, cols/32])."""
    if w.shape[-1] % 32:
        raise ValueError(f"MXFP4 needs cols % 32 == 0, got {tuple(w.shape)}")
    lead = w.shape[:-1]
    g = w.float().reshape(*lead, w.shape[-1] // 32, 32)
    amax = g.abs().amax(dim=-1)
    _, ex = torch.frexp(amax)  # amax = m * 2^ex, m in [0.5, 1)
    shared = (ex.to(torch.int32) - 1 - 2).clamp(-127, 127)
    shared = torch.where(amax > 0, shared, torch.full_like(shared, -127))
    v = torch.ldexp(g, (-shared).unsqueeze(-1).to(g.dtype))
    a = v.abs()
    mag = ((a > 0.25).to(torch.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75)
           + (a > 2.5) + (a >= 3.5) + (a > 5.0))
    codes = mag.to(torch.uint8) | ((v < 0).to(torch.uint8) << 3)
    codes = codes.reshape(*lead, w.shape[-1])
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).contiguous()
    scale = (shared + 127).to(torch.uint8).contiguous()
    return packed, scale


def dequantize_mxfp4(packed: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Inverse layout helper (float32); used for host-side diagnostics only."""
    grid = torch.tensor(E2M1_GRID + tuple(-x for x in E2M1_GRID), dtype=torch.float32,
                        device=packed.device)
    lo = (packed & 0x0F).long()
    hi = (packed >> 4).long()
    codes = torch.stack((lo, hi), dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    vals = grid[codes]
    s = torch.ldexp(torch.ones_like(scale, dtype=torch.float32), scale.to(torch.float32) - 127)
    s = torch.where(scale == 255, torch.full_like(s, float("nan")), s)
    return (vals.reshape(*scale.shape, 32) * s.unsqueeze(-1)).reshape(vals.shape)
