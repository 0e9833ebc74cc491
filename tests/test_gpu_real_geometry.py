"""The GLM-5.3-Flash MoE geometry itself (E = 288 routed experts, F = 2048,
top-8, n_group = topk_group = 1, one shared expert), 3.9 GB of routed weights
per layer: the decode chain (M = 1, 2), the E2M1-term batched path (M = 256:
7 routes per expert) and the widened-weight path (M = 8192: 228 routes per
expert) against the oracle — routing bit-exact on every token, outputs on
all tokens for M <= 2 and on sampled tokens beyond."""

import numpy as np
import pytest
import torch

from livglm_b200 import synthetic
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from oracle import moe_oracle as mo
from tests.helpers import assert_close, bank_to_numpy, to_numpy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def real_layer(cuda, native_lib):
    cfg = CONFIGS["glm53flash"]
    t = synthetic.layer_weights(cfg, seed=53, device=cuda)
    return cfg, t, bank_to_numpy(t), build_layer(cfg, t)


@pytest.mark.parametrize("M,n_check", [(1, 1), (2, 2), (256, 16), (8192, 8)])
def test_real_geometry(cuda, real_layer, M, n_check):
    cfg, t, tn, moe = real_layer
    x = synthetic.hidden_states(cfg, M, seed=530 + M, device=cuda)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    xn = to_numpy(x)
    _, rw, ri = mo.router(xn, tn["router_weight"], tn["router_bias"], cfg)
    np.testing.assert_array_equal(to_numpy(idx), ri)
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), rw.view(np.uint32))
    sel = np.random.default_rng(M).choice(M, n_check, replace=False)
    ref = mo.moe_forward(xn, tn, cfg, tokens=sel)
    assert_close(to_numpy(out)[sel], ref["out"])
