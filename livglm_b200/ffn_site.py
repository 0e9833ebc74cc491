"""FFN site of a MoE decoder layer: hyper-connections around the MoE block.

The reference runs its MoE block inside manifold-constrained hyper-connections
(kg36/livglm src/glm53flash/model.py:132-136):

    residual = hidden_states                               # [B, S, hc, d]
    post, comb, collapsed = self.ffn_hc(hidden_states)     # mhc.py:23-48
    fed_forward = self.mlp(self.post_attention_layernorm(collapsed))
    return hyper_residual(residual, fed_forward, post, comb)  # mhc.py:51-60

and the MTP width-two verify (runtime.py:657-661) reaches it with two tokens
per call.  MoEFFNSite is that site over ExpertSSDMoE, one C call
(lg_moe_ffn_site): the hyper-connection mix and its RMSNorm, the MoE block,
the hyper-residual.  HyperConnection and hyper_residual are the two halves on
their own (lg_hc_pre, lg_hc_post), with the reference's names and attributes
(fn, base, scale).

Streams are bf16 (the dtype the MoE boundary takes); the output is f32, as
MLX promotes bf16(post) * f32 MoE output.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native
from .config import ContractError
from .moe import ExpertSSDMoE, _stream_ptr, require_weight


@dataclass(frozen=True)
class HcConfig:
    """GLMTextConfig's hyper-connection fields (model_config.py:23-26)."""

    hc_mult: int = 4
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    rms_norm_eps: float = 1e-6

    def native(self) -> _native.LgHcConfig:
        if self.hc_mult < 1 or self.hc_sinkhorn_iters < 1:  # model_config.py:165-166
            raise ContractError("hyper-connection settings must be positive")
        return _native.LgHcConfig(self.hc_mult, self.hc_sinkhorn_iters, float(self.hc_eps),
                                  float(self.rms_norm_eps))


def _streams(x: torch.Tensor, hc: int, d: int) -> torch.Tensor:
    if not isinstance(x, torch.Tensor) or x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ContractError("hyper-connection streams must be a bf16 CUDA tensor")
    if x.ndim < 2 or tuple(x.shape[-2:]) != (hc, d):
        raise ContractError(f"streams must end in [{hc}, {d}], got {tuple(x.shape)}")
    return x.contiguous().reshape(-1, hc, d)


class HyperConnection:
    """HyperConnection (mhc.py:12-48): fn f32 [hc*(hc+2), hc*d], base f32
    [hc*(hc+2)], scale f32 [3]; __call__(streams [..., hc, d] bf16) ->
    (post f32 [..., hc], comb f32 [..., hc, hc], collapsed bf16 [..., d])."""

    def __init__(self, config: HcConfig, hidden_size: int):
        self.config = config
        self.hidden_size = hidden_size
        self.hc_mult = config.hc_mult
        self.hc_sinkhorn_iters = config.hc_sinkhorn_iters
        self.hc_eps = config.hc_eps
        self.fn = None
        self.base = None
        self.scale = None
        self._ws: torch.Tensor | None = None

    def native_weights(self, norm_weight: torch.Tensor | None = None) -> _native.LgHcWeights:
        hc, d = self.hc_mult, self.hidden_size
        R = hc * (hc + 2)
        for name, t, shape in (("fn", self.fn, (R, hc * d)), ("base", self.base, (R,)), ("scale", self.scale, (3,))):
            t = require_weight(t, f"hyper_connection.{name}")
            if t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_cuda or not t.is_contiguous():
                raise ContractError(f"hyper_connection.{name} must be a contiguous f32 CUDA tensor of shape {shape}")
        w = _native.LgHcWeights(self.fn.data_ptr(), self.base.data_ptr(), self.scale.data_ptr(), None)
        if norm_weight is not None:
            if norm_weight.dtype != torch.bfloat16 or tuple(norm_weight.shape) != (d,) or not norm_weight.is_cuda:
                raise ContractError(f"post_attention_layernorm.weight must be bf16 [{d}] on the GPU")
            w.norm_weight = norm_weight.contiguous().data_ptr()
        return w

    def __call__(self, streams: torch.Tensor):
        hc, d = self.hc_mult, self.hidden_size
        rows = _streams(streams, hc, d)
        M, dev = rows.shape[0], rows.device
        lib = _native.load()
        cfg = self.config.native()
        need = lib.lg_hc_workspace_size(cfg, d, max(M, 1))
        if self._ws is None or self._ws.numel() < need or self._ws.device != dev:
            self._ws = torch.empty(need, dtype=torch.uint8, device=dev)
        post = torch.empty(M, hc, dtype=torch.float32, device=dev)
        comb = torch.empty(M, hc, hc, dtype=torch.float32, device=dev)
        collapsed = torch.empty(M, d, dtype=torch.bfloat16, device=dev)
        _native.check(lib.lg_hc_pre(cfg, self.native_weights(), d, rows.data_ptr(), M, post.data_ptr(),
                                    comb.data_ptr(), collapsed.data_ptr(), None, self._ws.data_ptr(),
                                    self._ws.numel(), _stream_ptr(dev)), "lg_hc_pre")
        lead = streams.shape[:-2]
        return post.reshape(*lead, hc), comb.reshape(*lead, hc, hc), collapsed.reshape(*lead, d)


def hyper_residual(residual: torch.Tensor, sublayer_output: torch.Tensor, post: torch.Tensor, comb: torch.Tensor,
                   config: HcConfig) -> torch.Tensor:
    """mhc.py:51-60: residual bf16 [..., hc, d], sublayer_output f32 [..., d]
    -> f32 [..., hc, d]."""
    hc, d = config.hc_mult, residual.shape[-1]
    rows = _streams(residual, hc, d)
    M, dev = rows.shape[0], rows.device
    sub = sublayer_output.to(torch.float32).contiguous().reshape(M, d)
    post = post.to(torch.float32).contiguous().reshape(M, hc)
    comb = comb.to(torch.float32).contiguous().reshape(M, hc, hc)
    out = torch.empty(M, hc, d, dtype=torch.float32, device=dev)
    _native.check(_native.load().lg_hc_post(config.native(), d, rows.data_ptr(), sub.data_ptr(), post.data_ptr(),
                                            comb.data_ptr(), M, out.data_ptr(), _stream_ptr(dev)), "lg_hc_post")
    return out.reshape(residual.shape)


class MoEFFNSite:
    """The FFN half of GLMDecoderLayer around ExpertSSDMoE (model.py:132-136)
    as one C call.  post_attention_layernorm_weight: bf16 [d]."""

    def __init__(self, mlp: ExpertSSDMoE, ffn_hc: HyperConnection, post_attention_layernorm_weight: torch.Tensor):
        if ffn_hc.hidden_size != mlp.config.hidden_size:
            raise ContractError("hyper-connection and MoE block differ in hidden size")
        self.mlp = mlp
        self.ffn_hc = ffn_hc
        self.post_attention_layernorm_weight = post_attention_layernorm_weight
        self._ws: torch.Tensor | None = None

    def __call__(self, hidden_states: torch.Tensor, *, return_route: bool = False):
        c, hc = self.mlp.config, self.ffn_hc.hc_mult
        d = c.hidden_size
        rows = _streams(hidden_states, hc, d)
        M, dev, k = rows.shape[0], rows.device, c.num_experts_per_tok
        lib = _native.load()
        hcfg = self.ffn_hc.config.native()
        need = lib.lg_moe_ffn_site_workspace_size(self.mlp._cfg, hcfg, max(M, 1))
        if need == 0:
            _native.check(_native.LG_ERR_INVALID_ARG, "lg_moe_ffn_site_workspace_size")
        if self._ws is None or self._ws.numel() < need or self._ws.device != dev:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=dev)  # status word starts at 0
        out = torch.empty(M, hc, d, dtype=torch.float32, device=dev)
        weights = torch.empty(M, k, dtype=torch.float32, device=dev)
        indices = torch.empty(M, k, dtype=torch.uint32, device=dev)
        hw = self.ffn_hc.native_weights(self.post_attention_layernorm_weight)
        _native.check(lib.lg_moe_ffn_site(self.mlp._cfg, self.mlp.native_weights(), hcfg, hw, rows.data_ptr(), M,
                                          out.data_ptr(), weights.data_ptr(), indices.data_ptr(),
                                          self._ws.data_ptr(), self._ws.numel(), _stream_ptr(dev)),
                      "lg_moe_ffn_site")
        result = out.reshape(hidden_states.shape)
        if return_route:
            lead = hidden_states.shape[:-2]
            return result, weights.reshape(*lead, k), indices.reshape(*lead, k)
        return result

    def status(self) -> int:
        """Device status word of the site's workspace (0 = ok)."""
        return 0 if self._ws is None else int(self._ws[:4].view(torch.int32).item())
