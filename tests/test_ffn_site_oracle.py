"""The FFN-site oracle (hyper-connections, hyper_residual, rms_norm) pinned on
the CPU.

The first case takes the inputs of the reference's own hyper-connection
test (kg36/livglm tests/test_mhc.py:12-47: hidden 2, hc_mult 2, three
Sinkhorn iterations, eps 1e-6) and restates the published mHC arithmetic
there independently, with scalar loops, at its tolerances (rtol 1e-5,
atol 1e-6; 1e-3 / 1e-4 for hyper_residual, whose f32 matmul the reference
test also checks loosely).
"""

import math

import numpy as np

from oracle import ffn_site_oracle as fo
from oracle.moe_oracle import bf16_bits_to_f32, f32_to_bf16_bits


def _scalar_reference(streams, fn, base, scale, hc, iters, eps, rms_eps):
    d = streams.shape[-1]
    flat = [float(v) for v in streams.reshape(-1)]
    inv = 1.0 / math.sqrt(sum(v * v for v in flat) / len(flat) + rms_eps)
    flat = [v * inv for v in flat]
    mixed = [sum(flat[j] * float(fn[r, j]) for j in range(len(flat))) for r in range(fn.shape[0])]
    sig = lambda z: 1.0 / (1.0 + math.exp(-z))  # noqa: E731
    pre = [sig(mixed[h] * scale[0] + base[h]) + eps for h in range(hc)]
    post = [2.0 * sig(mixed[hc + h] * scale[1] + base[hc + h]) for h in range(hc)]
    logits = [[mixed[2 * hc + i * hc + j] * scale[2] + base[2 * hc + i * hc + j] for j in range(hc)]
              for i in range(hc)]
    comb = []
    for row in logits:
        m = max(row)
        ex = [math.exp(v - m) for v in row]
        s = sum(ex)
        comb.append([v / s + eps for v in ex])

    def col_norm(c):
        sums = [sum(c[i][j] for i in range(hc)) + eps for j in range(hc)]
        return [[c[i][j] / sums[j] for j in range(hc)] for i in range(hc)]

    def row_norm(c):
        return [[v / (sum(row) + eps) for v in row] for row in c]

    comb = col_norm(comb)
    for _ in range(iters - 1):
        comb = col_norm(row_norm(comb))
    collapsed = [sum(pre[h] * float(streams.reshape(hc, d)[h, i]) for h in range(hc)) for i in range(d)]
    return np.array(post), np.array(comb), np.array(collapsed)


def test_hyper_connection_matches_reference_test_inputs():
    streams = np.array([[[[0.5, -1.0], [1.5, 0.25]]]], np.float32)
    fn = np.arange(8 * 4, dtype=np.float32).reshape(8, 4) / 80.0 - 0.2
    base = np.linspace(-0.2, 0.2, 8, dtype=np.float32)
    scale = np.array([0.5, 0.75, 1.25], np.float32)
    post, comb, collapsed = fo.hyper_connection(streams, fn, base, scale, hc=2, iters=3, hc_eps=1e-6,
                                                rms_eps=1e-6, bf16=False)
    e_post, e_comb, e_collapsed = _scalar_reference(streams, fn, base, scale, 2, 3, 1e-6, 1e-6)
    np.testing.assert_allclose(post.reshape(-1), e_post, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(comb.reshape(2, 2), e_comb, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(collapsed.reshape(-1), e_collapsed, rtol=1e-5, atol=1e-6)
    # Sinkhorn leaves comb (nearly) doubly stochastic
    np.testing.assert_allclose(comb.reshape(2, 2).sum(axis=0), 1.0, atol=1e-5)

    sublayer = np.array([[[0.2, -0.3]]], np.float32)
    out = fo.hyper_residual(streams, sublayer, post, comb, bf16=False)
    expected = np.array(e_post)[:, None] * sublayer.reshape(1, 2) + np.array(e_comb).T @ streams.reshape(2, 2)
    np.testing.assert_allclose(out.reshape(2, 2), expected, rtol=1e-3, atol=1e-4)


def test_rms_norm_rounding_points():
    rng = np.random.default_rng(3)
    x = bf16_bits_to_f32(f32_to_bf16_bits(rng.standard_normal((3, 64)).astype(np.float32)))
    w = bf16_bits_to_f32(f32_to_bf16_bits((1 + 0.1 * rng.standard_normal(64)).astype(np.float32)))
    y = fo.rms_norm(x, w, 1e-6, bf16=True)
    assert np.array_equal(y, bf16_bits_to_f32(f32_to_bf16_bits(y)))  # bf16 values
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True) + 1e-6) * w
    np.testing.assert_allclose(y, ref, rtol=1.6e-2, atol=1e-3)  # two bf16 roundings


def test_ffn_site_bf16_flow():
    rng = np.random.default_rng(5)
    hc, d, M = 4, 32, 2
    streams = f32_to_bf16_bits(rng.standard_normal((M, hc, d)).astype(np.float32))
    site = {"fn": (0.02 * rng.standard_normal((hc * (hc + 2), hc * d))).astype(np.float32),
            "base": (0.1 * rng.standard_normal(hc * (hc + 2))).astype(np.float32),
            "scale": np.array([0.5, 0.75, 1.25], np.float32),
            "norm_weight": f32_to_bf16_bits(np.ones(d, np.float32))}
    calls = []

    def moe(x_bits):
        calls.append(x_bits)
        return 0.5 * bf16_bits_to_f32(x_bits)

    r = fo.ffn_site(streams, site, moe, hc, iters=20, hc_eps=1e-6, rms_eps=1e-6)
    assert calls and calls[0].shape == (M, d) and calls[0].dtype == np.uint16
    assert r["out"].shape == (M, hc, d) and r["out"].dtype == np.float32
    np.testing.assert_allclose(r["comb"].sum(axis=-2), 1.0, atol=1e-4)
    np.testing.assert_allclose(r["comb"].sum(axis=-1), 1.0, atol=1e-4)
    assert np.all((r["post"] > 0) & (r["post"] < 2))
