"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Bar: router logits, weights and indices and the dispatch permutation are
bit-exact; the f32 layer output is within max-abs 2e-2 and cosine >= 0.9995
(tests/helpers.py MAX_ABS / MIN_COSINE) of the oracle on identical inputs.
Full-size layers are checked on a sample of tokens (each token's output
depends only on its own row and the weights).
"""

import numpy as np
import pytest
import torch

from livglm_b200 import _native, synthetic
from livglm_b200.config import CONFIGS, ContractError
from livglm_b200.moe import ExpertSSDMoE, ResidentExperts, TopKRouter, build_layer
from oracle import moe_oracle as mo
from tests.helpers import (assert_close, bank_to_device, bank_to_numpy, to_device, to_numpy)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cfg1_layer(cuda, native_lib):
    cfg = CONFIGS["cfg1"]
    t = synthetic.layer_weights(cfg, seed=0, device=cuda)
    return cfg, t, bank_to_numpy(t)


def router_of(cfg, t):
    r = TopKRouter(cfg)
    r.weight, r.e_score_correction_bias = t["router_weight"], t["router_bias"]
    return r


# ---------------------------------------------------------------- golden ---

def test_golden_cfg0_router_dispatch_bit_exact(cuda, native_lib, golden_cfg0):
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    t = bank_to_device(z, cuda)
    x = to_device(z["x"], cuda, bf16=True)
    logits, weights, indices = router_of(cfg, t)(x)
    np.testing.assert_array_equal(to_numpy(logits).view(np.uint32), z["logits"].view(np.uint32))
    np.testing.assert_array_equal(to_numpy(weights).view(np.uint32), z["weights"].view(np.uint32))
    np.testing.assert_array_equal(to_numpy(indices), z["indices"])


def test_golden_cfg0_forward(cuda, native_lib, golden_cfg0):
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    moe = build_layer(cfg, bank_to_device(z, cuda))
    out, w, idx = moe(to_device(z["x"], cuda, bf16=True), return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy(idx), z["indices"])
    # cfg0 outputs are ~0.02 in size, so check a relative bound as well
    assert_close(to_numpy(out), z["out"], max_abs=2e-3)


def test_golden_cfg0_expert_and_shared_entry_points(cuda, native_lib, golden_cfg0):
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    moe = build_layer(cfg, bank_to_device(z, cuda))
    x = to_device(z["x"], cuda, bf16=True)
    y = moe.experts(x, to_device(z["indices"], cuda))
    sh = moe.shared_experts(x)
    yb, shb = to_numpy(y), to_numpy(sh)
    yf, ref_y = mo.bf16_bits_to_f32(yb), mo.bf16_bits_to_f32(z["y"])
    assert_close(yf, ref_y, max_abs=2e-3)
    # most bf16 outputs must agree to the bit; the rest within one ulp
    assert np.mean(yb == z["y"]) > 0.97
    assert_close(mo.bf16_bits_to_f32(shb), mo.bf16_bits_to_f32(z["shared"]), max_abs=2e-3)


# -------------------------------------------------------------- routing ---

@pytest.mark.parametrize("M", [1, 2, 3, 256, 1031, 4096])
def test_router_bit_exact_cfg1(cfg1_layer, cuda, M):
    cfg, t, tn = cfg1_layer
    x = synthetic.hidden_states(cfg, M, seed=M, device=cuda)
    logits, weights, indices = router_of(cfg, t)(x)
    sel = np.arange(M) if M <= 256 else np.random.default_rng(M).choice(M, 128, replace=False)
    rl, rw, ri = mo.router(to_numpy(x)[sel], tn["router_weight"], tn["router_bias"], cfg)
    np.testing.assert_array_equal(to_numpy(indices)[sel], ri)
    np.testing.assert_array_equal(to_numpy(weights)[sel].view(np.uint32), rw.view(np.uint32))
    np.testing.assert_array_equal(to_numpy(logits)[sel].view(np.uint32), rl.view(np.uint32))


def test_router_ties_and_masked_groups(cuda, native_lib):
    """All-zero router weights: every score is 0.5, so choices tie inside a
    group and the stable (value, index) order decides; k larger than the
    experts of the kept groups forces -inf picks, ordered by index."""
    cfg = CONFIGS["cfg0"].replace(num_experts_per_tok=12)
    E, d = cfg.n_routed_experts, cfg.hidden_size
    w = torch.zeros(E, d, device=cuda)
    b = torch.tensor([0.0, 1.0] * (E // 2), device=cuda)
    r = TopKRouter(cfg)
    r.weight, r.e_score_correction_bias = w, b
    x = torch.randn(3, d, device=cuda).to(torch.bfloat16)
    _, weights, idx = r(x)
    rl, rw, ri = mo.router(to_numpy(x), to_numpy(w), to_numpy(b), cfg)
    np.testing.assert_array_equal(to_numpy(idx), ri)
    np.testing.assert_array_equal(to_numpy(weights).view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("M,skew", [(1, False), (2, False), (256, False), (16384, False), (4096, True)])
def test_dispatch_bit_exact(cuda, native_lib, M, skew):
    from livglm_b200 import _native

    cfg = CONFIGS["cfg1"]
    E, k = cfg.n_routed_experts, cfg.num_experts_per_tok
    rng = np.random.default_rng(M)
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** 1.2
        idx = np.stack([rng.choice(E, k, replace=False, p=p / p.sum()) for _ in range(M)])
    else:
        idx = np.stack([rng.choice(E, k, replace=False) for _ in range(M)])
    idx = idx.astype(np.uint32)
    lib = _native.load()
    c = _native.LgConfig.from_config(cfg)
    counts = torch.empty(E, dtype=torch.int32, device=cuda)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    perm = torch.empty(M * k, dtype=torch.int32, device=cuda)
    ws = torch.zeros(lib.lg_moe_workspace_size(c, M), dtype=torch.uint8, device=cuda)
    di = to_device(idx, cuda)
    rc = lib.lg_moe_dispatch(c, di.data_ptr(), M, counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
                             ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    _native.check(rc, "dispatch")
    rc_, ro, rp = mo.dispatch(idx, E)
    np.testing.assert_array_equal(to_numpy(counts), rc_)
    np.testing.assert_array_equal(to_numpy(offsets), ro)
    np.testing.assert_array_equal(to_numpy(perm), rp)


# -------------------------------------------------------------- forward ---

@pytest.mark.parametrize("M", [1, 2, 3, 4, 5])
def test_forward_cfg1_decode(cfg1_layer, cuda, M):
    cfg, t, tn = cfg1_layer
    moe = build_layer(cfg, t)
    x = synthetic.hidden_states(cfg, M, seed=100 + M, device=cuda)
    out, w, idx = moe(x, return_route=True)
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), ref["weights"].view(np.uint32))
    assert_close(to_numpy(out), ref["out"])
    assert moe.device_status() == 0


@pytest.mark.parametrize("M", [256, 4096])
def test_forward_cfg1_batched_sampled(cfg1_layer, cuda, M):
    cfg, t, tn = cfg1_layer
    moe = build_layer(cfg, t)
    x = synthetic.hidden_states(cfg, M, seed=M, device=cuda)
    out, w, idx = moe(x, return_route=True)
    sel = np.random.default_rng(M).choice(M, 4, replace=False)
    ref = mo.moe_forward(to_numpy(x), tn, cfg, tokens=sel)
    np.testing.assert_array_equal(to_numpy(idx)[sel], ref["indices"])
    assert_close(to_numpy(out)[sel], ref["out"])


def test_combine_bit_exact_given_inputs(cfg1_layer, cuda):
    cfg, t, tn = cfg1_layer
    moe = build_layer(cfg, t)
    # M=5 takes the general (non-decode) chain, the same kernels as the
    # separate entry points
    x = synthetic.hidden_states(cfg, 5, seed=9, device=cuda)
    out, w, idx = moe(x, return_route=True)
    y = moe.experts(x, idx)
    sh = moe.shared_experts(x)
    # the fused forward must equal experts + shared + combine run separately
    ref = mo.combine(mo.bf16_bits_to_f32(to_numpy(y)), to_numpy(w), mo.bf16_bits_to_f32(to_numpy(sh)))
    np.testing.assert_array_equal(to_numpy(out).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("M", [1, 2, 6])
def test_forward_deterministic_and_shape_preserving(cfg1_layer, cuda, M):
    cfg, t, _ = cfg1_layer
    moe = build_layer(cfg, t)
    x = synthetic.hidden_states(cfg, 3 * M, seed=3, device=cuda).reshape(M, 3, cfg.hidden_size)
    a = moe(x)
    b = moe(x)
    assert a.shape == (M, 3, cfg.hidden_size) and a.dtype == torch.float32
    assert torch.equal(a, b)
    empty = moe(x[:0])
    assert empty.shape == (0, 3, cfg.hidden_size)


@pytest.mark.parametrize("M", [1, 3, 256])
def test_forward_host_tokens_and_output(cfg1_layer, cuda, M):
    """Tokens and result in page-locked host memory (the reference keeps hidden
    states in unified memory) give the bits of the device-resident call: the
    decode chain stages host tokens with a kernel (M=1, 3), the batched path
    with one copy (M=256); the result is written in place."""
    cfg, t, _ = cfg1_layer
    moe = build_layer(cfg, t)
    x = synthetic.hidden_states(cfg, M, seed=21 + M, device=cuda)
    ref = moe(x)
    x_host = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    x_host.copy_(x)
    out_host = torch.full((M, cfg.hidden_size), float("nan"), dtype=torch.float32, pin_memory=True)
    got = moe(x_host, out=out_host)
    got_dev = moe(x_host)
    out_dev = torch.full_like(ref, float("nan"))
    got_dev2 = moe(x, out=out_dev)
    torch.cuda.synchronize()
    assert got.data_ptr() == out_host.data_ptr() and not got.is_cuda
    assert torch.equal(got, ref.cpu())
    assert got_dev.is_cuda and torch.equal(got_dev, ref)
    assert got_dev2.data_ptr() == out_dev.data_ptr() and torch.equal(got_dev2, ref)


def test_forward_refuses_pageable_host_memory(cfg1_layer, cuda):
    """Pageable host memory is refused by the module and, before anything is
    launched, by the library itself."""
    cfg, t, _ = cfg1_layer
    moe = build_layer(cfg, t)
    x = torch.zeros(1, cfg.hidden_size, dtype=torch.bfloat16)
    with pytest.raises(ContractError, match="page-locked"):
        moe(x)
    with pytest.raises(ContractError, match="page-locked"):
        moe(x.to(cuda), out=torch.empty(1, cfg.hidden_size, dtype=torch.float32))
    lib = _native.load()
    out = torch.empty(1, cfg.hidden_size, dtype=torch.float32, device=cuda)
    ws = torch.zeros(lib.lg_moe_workspace_size(moe._cfg, 1), dtype=torch.uint8, device=cuda)
    rc = lib.lg_moe_forward(moe._cfg, moe.native_weights(), x.data_ptr(), 1, out.data_ptr(), None, None,
                            ws.data_ptr(), ws.numel(), torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _native.LG_ERR_INVALID_ARG
    assert "pageable" in _native.last_error()


def test_rebinding_weights_after_a_call(cuda, native_lib, golden_cfg0):
    """The module caches its native weight table between calls; rebinding a
    router, shared-expert or routed-expert tensor (a new tensor, or new storage
    under the same tensor) must reach the next call."""
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    t = bank_to_device(z, cuda)
    x = to_device(z["x"], cuda, bf16=True)
    moe = build_layer(cfg, t)
    base = moe(x)
    bias2 = t["router_bias"].flip(0).contiguous()
    moe.gate.e_score_correction_bias = bias2
    t2 = dict(t, router_bias=bias2)
    assert torch.equal(moe(x), build_layer(cfg, t2)(x))
    down2 = (t["shared_down"].float() * 0.5).to(torch.bfloat16)
    moe.shared_experts.down_proj.weight.data = down2  # same tensor object, new storage
    t2["shared_down"] = down2
    assert torch.equal(moe(x), build_layer(cfg, t2)(x))
    gate2 = t["gate_packed"].flip(0).contiguous()
    moe.experts.set_banks(gate2, t["gate_scale"], t["up_packed"], t["up_scale"],
                          t["down_packed"], t["down_scale"])
    t2["gate_packed"] = gate2
    got = moe(x)
    assert torch.equal(got, build_layer(cfg, t2)(x))
    assert not torch.equal(got, base)
    up2 = t["up_packed"].flip(0).contiguous()
    moe.experts.up_proj.weight_packed.data = up2  # same tensor object, new storage
    t2["up_packed"] = up2
    assert torch.equal(moe(x), build_layer(cfg, t2)(x))


def test_checkpoint_names_drop_in(cuda, native_lib, golden_cfg0):
    """Binding per-expert checkpoint tensors by their reference names gives the
    same layer as the stacked banks."""
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    L = 3
    tens = {}
    p = f"model.language_model.layers.{L}.mlp."
    tens[p + "gate.weight"] = torch.from_numpy(z["router_weight"])
    tens[p + "gate.e_score_correction_bias"] = torch.from_numpy(z["router_bias"])
    for name, key in (("gate_proj", "shared_gate"), ("up_proj", "shared_up"), ("down_proj", "shared_down")):
        tens[p + f"shared_experts.{name}.weight"] = torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16)
    for e in range(cfg.n_routed_experts):
        for proj, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
            tens[p + f"experts.{e}.{proj}.weight_packed"] = torch.from_numpy(z[f"{key}_packed"][e].copy())
            tens[p + f"experts.{e}.{proj}.weight_scale"] = torch.from_numpy(z[f"{key}_scale"][e].copy())
    moe = ExpertSSDMoE(cfg, L, lambda layer: ResidentExperts(cfg, layer=layer))
    moe.load_checkpoint(tens, device=cuda)
    out = moe(to_device(z["x"], cuda, bf16=True))
    ref = build_layer(cfg, bank_to_device(z, cuda))(to_device(z["x"], cuda, bf16=True))
    assert torch.equal(out, ref)
    assert len(moe.last_route_ids) == z["indices"].size


@pytest.mark.parametrize("M", [1, 3, 7])
@pytest.mark.parametrize("geo", [
    dict(n_routed_experts=48, num_experts_per_tok=1, n_group=1, topk_group=1),
    dict(n_routed_experts=64, num_experts_per_tok=6, n_group=2, topk_group=2, n_shared_experts=2),
    dict(n_routed_experts=32, num_experts_per_tok=8, n_group=4, topk_group=1, moe_intermediate_size=96,
         norm_topk_prob=False, swiglu_limit=0.0),
])
def test_forward_other_geometries(cuda, native_lib, geo, M):
    cfg = CONFIGS["cfg0"].replace(**geo)
    t = synthetic.layer_weights(cfg, seed=1, device=cuda)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=2, device=cuda) * 4
    out, w, idx = build_layer(cfg, t)(x, return_route=True)
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    assert_close(to_numpy(out), ref["out"])


@pytest.mark.parametrize("M", [1, 2, 6])
def test_forward_cfg0_small_batches(cuda, native_lib, golden_cfg0, M):
    """Decode-shaped calls (M <= 4 take the fused decode chain) on config 0."""
    z = golden_cfg0
    cfg = CONFIGS["cfg0"]
    moe = build_layer(cfg, bank_to_device(z, cuda))
    x = z["x"][:M]
    out, w, idx = moe(to_device(x, cuda, bf16=True), return_route=True)
    ref = mo.moe_forward(x, z, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), ref["weights"].view(np.uint32))
    assert_close(to_numpy(out), ref["out"], max_abs=2e-3)


@pytest.mark.parametrize("M", [1, 3])
def test_forward_large_activations(cuda, native_lib, M):
    """Hidden states far outside the f16 range exercise the power-of-two
    prescale of the decode kernels; SwiGLU without a limit keeps the large
    activations flowing into the down projection.  The prescale is exact; the
    bound (relative to max |out|) covers the decode kernels' 8-product f16x2
    partial sums, whose rounding (2^-11 relative) can move a bf16 rounding of
    gate/up by one ulp."""
    cfg = CONFIGS["cfg0"].replace(swiglu_limit=0.0)
    t = synthetic.layer_weights(cfg, seed=3, device=cuda)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=4, device=cuda) * 65536
    out, w, idx = build_layer(cfg, t)(x, return_route=True)
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    o, r = to_numpy(out), ref["out"]
    scale = float(np.max(np.abs(r)))
    assert_close(o / scale, r / scale, max_abs=5e-3)
