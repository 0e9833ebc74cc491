"""CPU oracle of the MoE layer's FFN site -- TEST INFRASTRUCTURE ONLY.

Only tests/ and __graft_entry__.smoke() may import this module, as the
checker; the product (livglm_b200) never imports it.

Restates, in NumPy:

* HyperConnection.__call__ (manifold-constrained hyper-connections)
                                         kg36/livglm src/glm53flash/mhc.py:23-48
* hyper_residual                         mhc.py:51-60
* RMSNorm / UnweightedRMSNorm            layers.py:119-140 (mx.fast.rms_norm)
* the FFN half of GLMDecoderLayer       model.py:132-136:
      post, comb, collapsed = ffn_hc(streams)
      out = hyper_residual(streams, moe(post_attention_layernorm(collapsed)), post, comb)

Rounding points follow MLX's dtype rules for bf16 streams: the
hyper-connection mixes in f32 and `collapsed` is cast back to the streams'
dtype; mx.fast.rms_norm normalises in f32 and rounds x * rsqrt(mean(x^2) +
eps) to the input dtype before the weight multiply (rounded again); in
hyper_residual `post` is cast to the streams' dtype, times the f32 MoE
output gives f32, and comb^T @ streams is a bf16 matmul (f32 sums, one
rounding), added in f32.

Pinning: the hyper-connection and hyper_residual arithmetic is checked
against the reference's own test inputs and formulas (tests/test_mhc.py:
hidden 2, hc_mult 2, three Sinkhorn iterations), restated independently in
tests/test_ffn_site_oracle.py.  The two rms_norm rounding points are MLX's
kernel's as documented above; MLX is absent here, so that detail is
"parity unpinned" (it moves results by at most one bf16 ulp of the MoE
input).
"""

from __future__ import annotations

import numpy as np

from .moe_oracle import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: float, bf16: bool) -> np.ndarray:
    """mx.fast.rms_norm over the last axis (layers.py:126-131, 139-140).
    x f32 values (bf16-representable when bf16); weight f32 values or None."""
    x = x.astype(np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    n = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    y = (x * n).astype(np.float32)
    if bf16:
        y = round_bf16(y)
    if weight is not None:
        y = (y * weight.astype(np.float32)).astype(np.float32)
        if bf16:
            y = round_bf16(y)
    return y


def hyper_connection(streams: np.ndarray, fn: np.ndarray, base: np.ndarray, scale: np.ndarray,
                     hc: int, iters: int, hc_eps: float, rms_eps: float, bf16: bool = True):
    """mhc.py:23-48.  streams [..., hc, d] f32 values -> (post [..., hc] f32,
    comb [..., hc, hc] f32, collapsed [..., d] in the streams' dtype)."""
    lead = streams.shape[:-2]
    d = streams.shape[-1]
    flat = streams.reshape(*lead, hc * d).astype(np.float32)
    flat = rms_norm(flat, None, rms_eps, bf16=False)  # UnweightedRMSNorm works in f32
    mixed = (flat.astype(np.float64) @ fn.astype(np.float64).T).astype(np.float32)
    pre_w, post_w, comb_w = mixed[..., :hc], mixed[..., hc:2 * hc], mixed[..., 2 * hc:]
    pre_b, post_b, comb_b = base[:hc], base[hc:2 * hc], base[2 * hc:]
    pre = _sigmoid(pre_w * scale[0] + pre_b) + np.float32(hc_eps)
    post = (2.0 * _sigmoid(post_w * scale[1] + post_b)).astype(np.float32)
    logits = comb_w.reshape(*lead, hc, hc) * scale[2] + comb_b.reshape(hc, hc)
    logits = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(logits.astype(np.float64))
    comb = (e / e.sum(axis=-1, keepdims=True)).astype(np.float32) + np.float32(hc_eps)
    comb = comb / (comb.sum(axis=-2, keepdims=True) + np.float32(hc_eps))
    for _ in range(iters - 1):
        comb = comb / (comb.sum(axis=-1, keepdims=True) + np.float32(hc_eps))
        comb = comb / (comb.sum(axis=-2, keepdims=True) + np.float32(hc_eps))
    collapsed = np.sum(pre[..., None].astype(np.float32) * streams.astype(np.float32), axis=-2)
    if bf16:
        collapsed = round_bf16(collapsed.astype(np.float32))
    return post.astype(np.float32), comb.astype(np.float32), collapsed.astype(np.float32)


def hyper_residual(residual: np.ndarray, sublayer: np.ndarray, post: np.ndarray, comb: np.ndarray,
                   bf16: bool = True) -> np.ndarray:
    """mhc.py:51-60.  residual [..., hc, d] (streams' dtype values), sublayer
    [..., d] f32 -> f32 [..., hc, d]."""
    p = round_bf16(post) if bf16 else post
    placed = p[..., :, None].astype(np.float32) * sublayer[..., None, :].astype(np.float32)
    c = round_bf16(comb) if bf16 else comb
    mixed = np.swapaxes(c, -1, -2).astype(np.float64) @ residual.astype(np.float64)
    mixed = round_bf16(mixed.astype(np.float32)) if bf16 else mixed.astype(np.float32)
    return (placed + mixed).astype(np.float32)


def ffn_site(streams_bits: np.ndarray, site: dict, moe, hc: int, iters: int, hc_eps: float,
             rms_eps: float) -> dict:
    """model.py:132-136 on bf16 streams [M, hc, d] (uint16 bits).  site:
    fn, base, scale (f32), norm_weight (uint16 bits).  moe(x_bits [M, d]) ->
    f32 [M, d] is the MoE block's oracle.  Returns post, comb, x (the MoE
    input, bits), ffn (f32) and out (f32 [M, hc, d])."""
    streams = bf16_bits_to_f32(streams_bits)
    post, comb, collapsed = hyper_connection(streams, site["fn"], site["base"], site["scale"], hc, iters,
                                             hc_eps, rms_eps, bf16=True)
    x = rms_norm(collapsed, bf16_bits_to_f32(site["norm_weight"]), rms_eps, bf16=True)
    x_bits = f32_to_bf16_bits(x)
    ffn = moe(x_bits)
    out = hyper_residual(streams, ffn, post, comb, bf16=True)
    return {"post": post, "comb": comb, "collapsed": collapsed, "x": x_bits, "ffn": ffn, "out": out}
