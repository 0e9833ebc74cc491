"""Stacked MoE layers: the config-3 workload harness.

Config 3 of the benchmark plan runs 42 MoE layers of config 1's shapes in
sequence on M tokens.  Between two layers the decoder applies its pre-FFN
norm (`self.mlp(self.post_attention_layernorm(...))`, kg36/livglm
src/glm53flash/model.py:132-136); the harness stands in for the rest of the
decoder with the reference's UnweightedRMSNorm (layers.py:134-140:
`mx.fast.rms_norm(x.astype(float32), None, eps)`), so layer l + 1 sees
bf16(rmsnorm(f32 output of layer l)).  eps is 1e-6, the value of the
reference's test configuration (tests/helpers.py:23).

The layers share one workspace: they run in order on one stream, so one
scratch area of the largest size serves every call.
"""

from __future__ import annotations

import torch

from .moe import ExpertSSDMoE, Workspace

RMS_EPS = 1e-6


def unweighted_rmsnorm_bf16(y: torch.Tensor, eps: float = RMS_EPS) -> torch.Tensor:
    """f32 [M, d] -> bf16 of y * rsqrt(mean(y^2) + eps), computed in f32."""
    y = y.float()
    return (y * torch.rsqrt(y.square().mean(dim=-1, keepdim=True) + eps)).to(torch.bfloat16)


class MoEStack:
    """ExpertSSDMoE layers applied in sequence with the unweighted RMSNorm in
    between; __call__ returns the last layer's f32 output."""

    def __init__(self, layers: list[ExpertSSDMoE], eps: float = RMS_EPS):
        if not layers:
            raise ValueError("a stack needs at least one layer")
        self.layers = layers
        self.eps = eps
        self.workspace = Workspace()
        for layer in layers:  # expert-parallel layers keep their own scratch
            if hasattr(layer, "use_workspace"):
                layer.use_workspace(self.workspace)

    def __call__(self, x: torch.Tensor, *, inputs: list | None = None,
                 outputs: list | None = None) -> torch.Tensor:
        """x: bf16 [M, d].  With `inputs` / `outputs` (lists), the bf16 input
        and the f32 output of every layer are appended (layer-by-layer checks)."""
        h = x
        out = None
        for i, layer in enumerate(self.layers):
            if inputs is not None:
                inputs.append(h)
            out = layer(h)
            if outputs is not None:
                outputs.append(out)
            if i + 1 < len(self.layers):
                h = unweighted_rmsnorm_bf16(out, self.eps)
        return out
