"""The MoE layer's FFN site on the GPU (hyper-connections around the block,
kg36/livglm model.py:132-136) against the CPU oracle.

Bar: the hyper-connection gates and Sinkhorn matrix to f32 rounding (rtol
1e-5, atol 1e-6, the reference test's own tolerance); collapsed and the
normalised MoE input within one bf16 ulp (their f32 sums run in another
order than NumPy's); the MoE's routing bit-exact and its output within the
block's parity bar on the GPU's own MoE input; the hyper-residual output
within one bf16 ulp of its mixed part on identical inputs (the normalised
input within two, nearly all exact); the site end to
end within max-abs 2e-2 and cosine >= 0.9995.  Width two (the MTP verify)
and one token at config 1's shapes with four streams, and config 0 at eight
tokens.
"""

import numpy as np
import pytest
import torch

from livglm_b200 import _native, synthetic
from livglm_b200.config import CONFIGS, ContractError
from livglm_b200.ffn_site import HcConfig, HyperConnection, MoEFFNSite, hyper_residual
from livglm_b200.moe import _stream_ptr, build_layer
from oracle import ffn_site_oracle as fo
from oracle import moe_oracle as mo
from tests.helpers import assert_close, bank_to_numpy, to_numpy

pytestmark = pytest.mark.gpu


def bf16_ulps(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - a, a)  # sign-magnitude -> ordered integers
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


def assert_residual_close(got: np.ndarray, ref: np.ndarray, post: np.ndarray, sub: np.ndarray) -> None:
    """hyper_residual outputs on identical inputs: the mixed part
    (bf16(comb)^T @ streams, rounded to bf16) may land one bf16 ulp away
    when its f32 sum runs in another order; the placed part is exact."""
    placed = mo.round_bf16(post)[..., :, None] * sub[..., None, :]
    mixed = ref - placed
    assert np.all(np.abs(got - ref) <= 2 ** -7 * np.abs(mixed) + 1e-6), float(np.max(np.abs(got - ref)))


def test_hyper_connection_reference_test_inputs(cuda, native_lib):
    """The inputs of kg36/livglm tests/test_mhc.py:12-47 (hidden 2, two streams,
    three Sinkhorn iterations) through lg_hc_pre / lg_hc_post."""
    hc = HcConfig(hc_mult=2, hc_sinkhorn_iters=3, hc_eps=1e-6, rms_norm_eps=1e-6)
    streams = np.array([[[[0.5, -1.0], [1.5, 0.25]]]], np.float32)
    fn = np.arange(8 * 4, dtype=np.float32).reshape(8, 4) / 80.0 - 0.2
    base = np.linspace(-0.2, 0.2, 8, dtype=np.float32)
    scale = np.array([0.5, 0.75, 1.25], np.float32)
    layer = HyperConnection(hc, 2)
    layer.fn, layer.base, layer.scale = (torch.from_numpy(a).to(cuda) for a in (fn, base, scale))
    s_dev = torch.from_numpy(streams).to(cuda).to(torch.bfloat16)  # values are bf16-exact
    post, comb, collapsed = layer(s_dev)
    torch.cuda.synchronize()
    e_post, e_comb, e_col = fo.hyper_connection(streams, fn, base, scale, 2, 3, 1e-6, 1e-6, bf16=False)
    np.testing.assert_allclose(to_numpy(post), e_post, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_numpy(comb), e_comb, rtol=1e-5, atol=1e-6)
    col = to_numpy(collapsed.float())
    np.testing.assert_allclose(col, e_col, rtol=2 ** -8, atol=1e-6)  # collapsed is cast to bf16

    sub = torch.tensor([[[0.2, -0.3]]], dtype=torch.float32, device=cuda)
    out = hyper_residual(s_dev, sub, post, comb, hc)
    torch.cuda.synchronize()
    ref = fo.hyper_residual(streams, to_numpy(sub), to_numpy(post), to_numpy(comb), bf16=True)
    assert_residual_close(to_numpy(out), ref, to_numpy(post), to_numpy(sub))


def _site(cfg, hc, M, seed, cuda):
    t = synthetic.layer_weights(cfg, seed=seed, device=cuda)
    moe = build_layer(cfg, t)
    sw = synthetic.ffn_site_weights(cfg, hc.hc_mult, seed=seed, device=cuda)
    layer = HyperConnection(hc, cfg.hidden_size)
    layer.fn, layer.base, layer.scale = sw["fn"], sw["base"], sw["scale"]
    site = MoEFFNSite(moe, layer, sw["norm_weight"])
    streams = synthetic.streams(cfg, M, hc.hc_mult, seed=100 + seed, device=cuda)
    return t, moe, sw, layer, site, streams


@pytest.mark.parametrize("name,M", [("cfg1", 2), ("cfg1", 1), ("cfg0", 8)])
def test_ffn_site_matches_oracle(cuda, native_lib, name, M):
    cfg = CONFIGS[name]
    hc = HcConfig(hc_mult=4, hc_sinkhorn_iters=20, hc_eps=1e-6, rms_norm_eps=1e-6)
    t, moe, sw, layer, site, streams = _site(cfg, hc, M, seed=3, cuda=cuda)
    d, H = cfg.hidden_size, hc.hc_mult
    lib = _native.load()

    # the pre half through the C ABI, with both optional outputs
    post = torch.empty(M, H, dtype=torch.float32, device=cuda)
    comb = torch.empty(M, H, H, dtype=torch.float32, device=cuda)
    collapsed = torch.empty(M, d, dtype=torch.bfloat16, device=cuda)
    x = torch.empty(M, d, dtype=torch.bfloat16, device=cuda)
    need = lib.lg_hc_workspace_size(hc.native(), d, M)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    _native.check(lib.lg_hc_pre(hc.native(), layer.native_weights(sw["norm_weight"]), d, streams.data_ptr(), M,
                                post.data_ptr(), comb.data_ptr(), collapsed.data_ptr(), x.data_ptr(),
                                ws.data_ptr(), need, _stream_ptr(cuda)), "lg_hc_pre")
    out, w, idx = site(streams, return_route=True)
    torch.cuda.synchronize()

    sn = {k: to_numpy(v) for k, v in sw.items()}
    s_bits = to_numpy(streams)
    s_f32 = mo.bf16_bits_to_f32(s_bits)
    e_post, e_comb, e_col = fo.hyper_connection(s_f32, sn["fn"], sn["base"], sn["scale"], H, hc.hc_sinkhorn_iters,
                                                hc.hc_eps, hc.rms_norm_eps, bf16=True)
    np.testing.assert_allclose(to_numpy(post), e_post, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(to_numpy(comb), e_comb, rtol=1e-5, atol=1e-6)
    assert bf16_ulps(to_numpy(collapsed), mo.f32_to_bf16_bits(e_col)).max() <= 1
    e_x = mo.f32_to_bf16_bits(fo.rms_norm(mo.bf16_bits_to_f32(to_numpy(collapsed)),
                                          mo.bf16_bits_to_f32(sn["norm_weight"]), hc.rms_norm_eps, bf16=True))
    ulps = bf16_ulps(to_numpy(x), e_x)
    assert ulps.max() <= 2 and ulps.mean() < 0.01  # rms factor summed in another order

    # the MoE on the GPU's own input: routing bit-exact, output in the bar
    tn = bank_to_numpy(t)
    x_bits = to_numpy(x)
    ref_moe = mo.moe_forward(x_bits, tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref_moe["indices"])
    ffn = moe(x)
    torch.cuda.synchronize()
    assert_close(to_numpy(ffn), ref_moe["out"])

    # the post half on identical inputs, then the site end to end
    e_out_same = fo.hyper_residual(s_f32, to_numpy(ffn), to_numpy(post), to_numpy(comb), bf16=True)
    got = to_numpy(out)
    assert_residual_close(got, e_out_same, to_numpy(post), to_numpy(ffn))
    full = fo.ffn_site(s_bits, sn, lambda xb: mo.moe_forward(xb, tn, cfg)["out"], H, hc.hc_sinkhorn_iters,
                       hc.hc_eps, hc.rms_norm_eps)
    assert_close(got, full["out"])
    assert site.status() == 0


def test_ffn_site_argument_errors(cuda, native_lib):
    cfg = CONFIGS["cfg0"]
    hc = HcConfig(hc_mult=4)
    t, moe, sw, layer, site, streams = _site(cfg, hc, 2, seed=4, cuda=cuda)
    with pytest.raises(ContractError):
        site(streams[:, :3])  # three streams for a four-stream site
    with pytest.raises(ContractError):
        site(streams.float())
    bad = HcConfig(hc_mult=5)
    lib = _native.load()
    assert lib.lg_hc_workspace_size(bad.native(), cfg.hidden_size, 2) == 0
    rc = lib.lg_moe_ffn_site(moe._cfg, moe.native_weights(), hc.native(), layer.native_weights(sw["norm_weight"]),
                             streams.data_ptr(), 2, 16, None, None, 256, 16, None)
    assert rc == _native.LG_ERR_WORKSPACE
    empty = site(streams[:0])
    assert empty.shape == (0, hc.hc_mult, cfg.hidden_size)
