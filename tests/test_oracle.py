"""CPU checks of the oracle itself: the reference's known-answer test, the
MXFP4 codec against ml_dtypes, and the frozen config-0 golden record."""

import ml_dtypes
import numpy as np
import pytest

from livglm_b200.config import CONFIGS, MoEConfig
from oracle import moe_oracle as mo


def tiny(**kw) -> MoEConfig:
    # tests/helpers.py:6-56 of the reference: d=32, 4 experts, top-2, F=32,
    # swiglu_limit 10, scale 2.5, norm_topk_prob True.
    base = dict(hidden_size=32, moe_intermediate_size=32, n_routed_experts=4, num_experts_per_tok=2,
                n_shared_experts=1, n_group=1, topk_group=1)
    base.update(kw)
    return MoEConfig(**base)


def test_router_selects_only_best_group_and_normalizes_original_scores():
    """Port of kg36/livglm tests/test_moe.py:10-23."""
    cfg = tiny(n_routed_experts=4, num_experts_per_tok=2, n_group=2, topk_group=1)
    w = np.zeros((4, 32), np.float32)
    b = np.array([10.0, 9.0, 1.0, 0.0], np.float32)
    x = np.zeros((1, 32), np.uint16)
    _, weights, indices = mo.router(x, w, b, cfg)
    assert set(indices.reshape(-1).tolist()) == {0, 1}
    np.testing.assert_allclose(weights, [[1.25, 1.25]], atol=1e-6)
    # order: ascending choice, best last (moe.py:58)
    assert indices.tolist() == [[1, 0]]


def test_router_tie_order_is_stable_ascending():
    """Equal choices: the last-k slice of a stable ascending sort prefers the
    higher expert index, listed in ascending (value, index) order."""
    cfg = tiny(n_routed_experts=8, num_experts_per_tok=3, n_group=1, topk_group=1)
    w = np.zeros((8, 32), np.float32)
    b = np.zeros(8, np.float32)
    _, weights, indices = mo.router(np.zeros((1, 32), np.uint16), w, b, cfg)
    assert indices.tolist() == [[5, 6, 7]]
    assert np.all(weights == weights[0, 0])


def test_router_matches_float64_reference_semantics():
    """Indices agree with a float64 evaluation of moe.py:36-63 wherever the
    float64 choice margins are far from float32 rounding."""
    cfg = CONFIGS["cfg0"]
    rng = np.random.default_rng(5)
    x = mo.f32_to_bf16_bits(rng.standard_normal((64, cfg.hidden_size)).astype(np.float32))
    w = (rng.standard_normal((cfg.n_routed_experts, cfg.hidden_size)) * 0.02).astype(np.float32)
    b = rng.uniform(-0.01, 0.01, cfg.n_routed_experts).astype(np.float32)
    logits, weights, idx = mo.router(x, w, b, cfg)
    xf = mo.bf16_bits_to_f32(x).astype(np.float64)
    lg = xf @ w.astype(np.float64).T
    np.testing.assert_allclose(logits, lg, rtol=1e-5, atol=1e-5)
    sc = 1 / (1 + np.exp(-lg))
    ch = sc + b
    E, G, g, k = cfg.n_routed_experts, cfg.n_group, cfg.topk_group, cfg.num_experts_per_tok
    grouped = ch.reshape(-1, G, E // G)
    gs = np.sort(grouped, -1)[..., -2:].sum(-1)
    gi = np.argsort(gs, -1, kind="stable")[..., -g:]
    mask = np.zeros_like(gs, bool)
    np.put_along_axis(mask, gi, True, -1)
    chm = np.where(np.repeat(mask, E // G, -1), ch, -np.inf)
    ref = np.argsort(chm, -1, kind="stable")[..., -k:]
    np.testing.assert_array_equal(idx, ref)
    rw = np.take_along_axis(sc, ref, -1)
    rw = rw / (rw.sum(-1, keepdims=True) + 1e-20) * cfg.routed_scaling_factor
    np.testing.assert_allclose(weights, rw, rtol=1e-6)


def test_own_exp_and_sigmoid_error_bounds():
    x = np.linspace(-87, 88, 400_001, dtype=np.float32)
    y = mo.own_exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    assert np.max(np.abs(y - ref) / ref) < 2 * 2.0 ** -24  # within 2 ulp like CUDA's expf
    s = mo.sigmoid(x).astype(np.float64)
    sref = 1 / (1 + np.exp(-x.astype(np.float64)))
    assert np.max(np.abs(s - sref)) < 2.0 ** -23
    assert mo.own_exp(np.array([100.0, -200.0, 0.0], np.float32)).tolist() == [np.inf, 0.0, 1.0]


def test_e2m1_codes_match_ml_dtypes():
    codes = np.arange(16, dtype=np.uint8)
    ref = codes.view(ml_dtypes.float4_e2m1fn).astype(np.float32)
    np.testing.assert_array_equal(mo.E2M1_VALUES, ref)
    assert np.array_equal(np.signbit(mo.E2M1_VALUES), np.signbit(ref))


def test_e8m0_codes_match_ml_dtypes():
    s = np.arange(256, dtype=np.uint8)
    ours = mo.e8m0_to_f32(s)
    ref = s.view(ml_dtypes.float8_e8m0fnu).astype(np.float32)
    np.testing.assert_array_equal(np.isnan(ours), np.isnan(ref))
    np.testing.assert_array_equal(ours[~np.isnan(ours)], ref[~np.isnan(ref)])


def test_packed_bytes_as_le_u32_keep_column_order():
    """expert_source.py:210-215 hands MLX the U8 record viewed as little-endian
    U32; nibble i of word w must be column 8w + i for that view to decode to
    the same elements as the byte layout (low nibble = even column)."""
    rng = np.random.default_rng(1)
    packed = rng.integers(0, 256, (3, 16), dtype=np.uint8)
    words = packed.view("<u4")
    cols = np.stack([(words >> (4 * i)) & 0xF for i in range(8)], -1).reshape(3, -1)
    scale = np.full((3, 1), 127, np.uint8)
    np.testing.assert_array_equal(mo.E2M1_VALUES[cols], mo.mxfp4_dequant(packed, scale))


def test_limited_swiglu_clamps_gate_above_only():
    """docs/v1-impl.md:307-315: gate = min(gate, 10); up = clip(up, -10, 10)."""
    gate = np.array([-20.0, 15.0, 2.0], np.float32)
    up = np.array([15.0, -15.0, 3.0], np.float32)
    out = mo.limited_swiglu_bf16(gate, up, 10.0)
    silu = lambda v: v / (1 + np.exp(-v))  # noqa: E731
    ref = np.array([silu(-20.0) * 10.0, silu(10.0) * -10.0, silu(2.0) * 3.0])
    np.testing.assert_allclose(out, ref, rtol=2e-2)
    assert out[0] < 0  # the gate's lower side is not clamped


def test_dispatch_c_matches_numpy():
    rng = np.random.default_rng(2)
    idx = rng.integers(0, 16, (37, 4)).astype(np.uint32)
    counts, offsets, perm = mo.dispatch(idx, 16)
    c2 = np.zeros(16, np.int32)
    o2 = np.zeros(17, np.int32)
    p2 = np.zeros(idx.size, np.int32)
    mo.lib().oracle_dispatch(idx.reshape(-1), idx.size, 16, c2, o2, p2)
    np.testing.assert_array_equal(counts, c2)
    np.testing.assert_array_equal(offsets, o2)
    np.testing.assert_array_equal(perm, p2)
    flat = idx.reshape(-1)
    assert np.all(np.diff(flat[perm].astype(np.int64)) >= 0)


def test_golden_cfg0_record_is_reproduced(golden_cfg0):
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    ref = mo.moe_forward(z["x"], z, cfg)
    np.testing.assert_array_equal(ref["indices"], z["indices"])
    np.testing.assert_array_equal(ref["weights"].view(np.uint32), z["weights"].view(np.uint32))
    np.testing.assert_array_equal(ref["logits"].view(np.uint32), z["logits"].view(np.uint32))
    np.testing.assert_array_equal(mo.f32_to_bf16_bits(ref["y"]), z["y"])
    np.testing.assert_allclose(ref["out"], z["out"], rtol=0, atol=1e-6)
    counts, offsets, perm = mo.dispatch(z["indices"], cfg.n_routed_experts)
    np.testing.assert_array_equal(perm, z["perm"])


@pytest.mark.parametrize("k,E,G,g", [(1, 4, 1, 1), (4, 16, 4, 2), (8, 128, 8, 4), (8, 288, 1, 1)])
def test_router_geometries_select_k_distinct_experts(k, E, G, g):
    cfg = tiny(n_routed_experts=E, num_experts_per_tok=k, n_group=G, topk_group=g, hidden_size=64)
    rng = np.random.default_rng(k * E)
    x = mo.f32_to_bf16_bits(rng.standard_normal((5, 64)).astype(np.float32))
    w = (rng.standard_normal((E, 64)) * 0.02).astype(np.float32)
    b = rng.uniform(-0.01, 0.01, E).astype(np.float32)
    logits, weights, idx = mo.router(x, w, b, cfg)
    for row in idx:
        assert len(set(row.tolist())) == k
        groups = {int(e) // (E // G) for e in row}
        assert len(groups) <= g
    np.testing.assert_allclose(weights.sum(-1), cfg.routed_scaling_factor, rtol=1e-5)


def test_c_restatement_matches_numpy_oracle_on_golden_cfg0(golden_cfg0):
    """oracle/experts_ref.c (the timed CPU baseline: weights decoded on the
    fly) against the NumPy oracle on the committed config-0 record: routing
    bit-identical, outputs identical at this size."""
    cfg = CONFIGS["cfg0"]
    ref = mo.moe_forward(golden_cfg0["x"], golden_cfg0, cfg)
    got = mo.moe_forward_c(golden_cfg0["x"], golden_cfg0, cfg)
    np.testing.assert_array_equal(got["indices"], ref["indices"])
    np.testing.assert_array_equal(got["weights"].view(np.uint32), ref["weights"].view(np.uint32))
    np.testing.assert_array_equal(got["out"], ref["out"])


def test_c_restatement_on_random_geometry_within_tolerance():
    """A d=512, F=256, 32-expert layer with random MXFP4 bytes (scales
    0..254 near 120) and 40 tokens: the C restatement and the NumPy oracle
    differ only by f32 summation order before the bf16 roundings."""
    from tests.helpers import assert_close

    cfg = MoEConfig(hidden_size=512, moe_intermediate_size=256, n_routed_experts=32, num_experts_per_tok=4,
                    n_shared_experts=1, n_group=4, topk_group=2)
    rng = np.random.default_rng(9)
    E, d, F = 32, 512, 256
    bank = {
        "router_weight": (rng.standard_normal((E, d)) * 0.05).astype(np.float32),
        "router_bias": (rng.standard_normal(E) * 0.01).astype(np.float32),
        "gate_packed": rng.integers(0, 256, (E, F, d // 2), dtype=np.uint8),
        "gate_scale": rng.integers(116, 121, (E, F, d // 32), dtype=np.uint8),
        "up_packed": rng.integers(0, 256, (E, F, d // 2), dtype=np.uint8),
        "up_scale": rng.integers(116, 121, (E, F, d // 32), dtype=np.uint8),
        "down_packed": rng.integers(0, 256, (E, d, F // 2), dtype=np.uint8),
        "down_scale": rng.integers(116, 121, (E, d, F // 32), dtype=np.uint8),
        "shared_gate": mo.f32_to_bf16_bits((rng.standard_normal((F, d)) * 0.02).astype(np.float32)),
        "shared_up": mo.f32_to_bf16_bits((rng.standard_normal((F, d)) * 0.02).astype(np.float32)),
        "shared_down": mo.f32_to_bf16_bits((rng.standard_normal((d, F)) * 0.02).astype(np.float32)),
    }
    x = mo.f32_to_bf16_bits(rng.standard_normal((40, d)).astype(np.float32))
    ref = mo.moe_forward(x, bank, cfg)
    got = mo.moe_forward_c(x, bank, cfg)
    np.testing.assert_array_equal(got["indices"], ref["indices"])
    assert_close(got["out"], ref["out"])


def test_near_tie_routing_risk_against_float64():
    """The canonical f32 router against a float64 evaluation of moe.py:36-63
    on 2048 config-4 tokens (Zipf bias): expert sets agree except where the
    k-th and (k+1)-th choices lie within f32 rounding.  The committed record
    tests/golden/near_ties_cfg4.json holds the 16384-token statistics."""
    import json

    from tests.golden import near_ties

    s = near_ties.stats(2048)
    assert s["fraction_of_tokens"] <= 0.005
    assert s["tokens_with_different_expert_set"] <= s["tokens_with_kth_gap_below_1e-6"]
    full = json.loads(near_ties.OUT.read_text())
    assert full["tokens"] == 16384 and full["fraction_of_tokens"] <= 0.005
