"""Configs 3 and 4 of the benchmark plan against the CPU oracle.

config 3  42 stacked layers of config 1's shapes at M = 4096: every layer's
          routing and output are checked on sampled tokens against the oracle
          fed with that layer's own GPU input (each token's output depends
          only on its own row), and the harness's inter-layer norm
          (layers.py:134-140, unweighted RMSNorm) is checked against a float64
          restatement.
config 4  config 1's layer at M = 16384 with the committed Zipf(1.2)
          correction bias: routing and the dispatch permutation bit-exact on
          all 16384 tokens, outputs on 256 sampled tokens.
"""

import numpy as np
import pytest
import torch

from livglm_b200 import synthetic, workloads
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from livglm_b200.stack import MoEStack
from oracle import moe_oracle as mo
from tests.helpers import assert_close, bank_to_numpy, to_numpy

pytestmark = pytest.mark.gpu

CHECKED_LAYERS = (0, 1, 20, 41)


def test_cfg3_stack_layerwise(cuda, native_lib):
    cfg = CONFIGS["cfg3"]
    L, M = workloads.CFG3_LAYERS, workloads.CFG3_TOKENS
    tensors = [synthetic.layer_weights(cfg, layer=layer, seed=3, device=cuda) for layer in range(L)]
    stack = MoEStack([build_layer(cfg, t, layer_idx=i) for i, t in enumerate(tensors)])
    x = synthetic.hidden_states(cfg, M, seed=33, device=cuda)
    inputs: list = []
    outputs: list = []
    out = stack(x, inputs=inputs, outputs=outputs)
    torch.cuda.synchronize()
    assert out.shape == (M, cfg.hidden_size) and bool(torch.isfinite(out).all())
    assert stack.workspace.status() == 0
    assert len(inputs) == len(outputs) == L
    rng = np.random.default_rng(3)
    for layer in CHECKED_LAYERS:
        sel = rng.choice(M, 4, replace=False)
        tn = bank_to_numpy(tensors[layer])
        ref = mo.moe_forward(to_numpy(inputs[layer]), tn, cfg, tokens=sel)
        assert_close(to_numpy(outputs[layer])[sel], ref["out"])
        if layer + 1 < L:  # the next layer's input is bf16(rmsnorm(this layer's f32 output))
            y = outputs[layer].double()
            norm = (y * torch.rsqrt(y.square().mean(-1, keepdim=True) + 1e-6)).float()
            diff = (inputs[layer + 1].float() - norm).abs().max().item()
            assert diff <= 2 ** -7 * norm.abs().max().item()


def test_cfg4_zipf_routing_and_sampled_outputs(cuda, native_lib):
    cfg = CONFIGS["cfg4"]
    M = workloads.CFG4_TOKENS
    t = synthetic.layer_weights(cfg, seed=4, device=cuda, router_bias=workloads.cfg4_bias(cuda))
    tn = bank_to_numpy(t)
    moe = build_layer(cfg, t)
    x = synthetic.hidden_states(cfg, M, seed=44, device=cuda)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    xn = to_numpy(x)
    rl, rw, ri = mo.router(xn, tn["router_weight"], tn["router_bias"], cfg)
    np.testing.assert_array_equal(to_numpy(idx), ri)
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), rw.view(np.uint32))
    stats = workloads.load_stats(idx, cfg.n_routed_experts)
    assert stats["max_over_mean"] > 5.0  # the skew the workload is about
    sel = np.random.default_rng(4).choice(M, 256, replace=False)
    ref = mo.moe_forward(xn, tn, cfg, tokens=sel)
    assert_close(to_numpy(out)[sel], ref["out"])
