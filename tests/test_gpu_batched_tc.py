"""The batched tensor-core path (livglm_b200/csrc/grouped_tc.cuh) against the
CPU oracle.

Calls of at least 64 tokens whose geometry has d a multiple of 1024 and F a
multiple of 512 run
the routed experts as block-scaled kind::mxf4 grouped GEMMs (activations as
six E2M1 terms) and the shared expert as kind::f16 GEMMs.  Bar as in
test_gpu_parity.py: routing bit-exact, f32 output within max-abs 2e-2 and
cosine >= 0.9995 of the oracle on every token checked.

Small geometries (d = 1024, F = 512, 16 experts) are checked on all tokens,
including routes that spread over several 32-route tiles per expert and
experts with none; config 2 (cfg1 shapes at M = 256) on all 256 tokens.
"""

import numpy as np
import pytest
import torch

from livglm_b200 import _native, synthetic
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from oracle import moe_oracle as mo
from tests.helpers import assert_close, bank_to_numpy, to_numpy

pytestmark = pytest.mark.gpu

SMALL = CONFIGS["cfg0"].replace(hidden_size=1024, moe_intermediate_size=512)


def _bias_towards_first(cfg, strength: float, device):
    """Correction bias that makes low expert ids popular (skewed routing)."""
    e = torch.arange(cfg.n_routed_experts, dtype=torch.float32, device=device)
    return -strength * torch.log1p(e)


@pytest.mark.parametrize("M,skew", [(64, 0.0), (100, 0.0), (300, 0.0), (300, 0.3), (2048, 0.3)])
def test_small_geometry_all_tokens(cuda, native_lib, M, skew):
    cfg = SMALL
    bias = _bias_towards_first(cfg, skew, cuda) if skew else None
    t = synthetic.layer_weights(cfg, seed=11, device=cuda, router_bias=bias)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=12 + M, device=cuda)
    moe = build_layer(cfg, t)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), ref["weights"].view(np.uint32))
    assert_close(to_numpy(out), ref["out"])
    if skew:  # several route tiles for the popular experts, none for others
        counts = np.bincount(ref["indices"].reshape(-1).astype(np.int64), minlength=cfg.n_routed_experts)
        assert counts.max() > 64


def test_small_geometry_expert_and_shared_entry_points(cuda, native_lib):
    cfg = SMALL
    M = 160
    t = synthetic.layer_weights(cfg, seed=21, device=cuda)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=22, device=cuda)
    moe = build_layer(cfg, t)
    _, _, idx = moe(x, return_route=True)
    y = moe.experts(x, idx)
    sh = moe.shared_experts(x)
    torch.cuda.synchronize()
    ref_y = mo.expert_outputs(to_numpy(x), tn, to_numpy(idx), cfg)
    ref_sh = mo.shared_expert(to_numpy(x), tn, cfg)
    assert_close(mo.bf16_bits_to_f32(to_numpy(y)), ref_y)
    # the shared expert runs on bf16 operands with f32 accumulation: the only
    # differences to the oracle are bf16 roundings of near-ties
    got_sh = to_numpy(sh)
    assert_close(mo.bf16_bits_to_f32(got_sh), ref_sh, max_abs=5e-3)
    assert np.mean(got_sh == mo.f32_to_bf16_bits(ref_sh)) > 0.97


def test_cfg2_all_tokens(cuda, native_lib):
    """Config 2: the full-size layer (d=4096, 128 experts, top-8, F=1536) at
    M=256 with uniform routing, every token against the oracle."""
    cfg = CONFIGS["cfg2"]
    t = synthetic.layer_weights(cfg, seed=2, device=cuda)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, 256, seed=256, device=cuda)
    moe = build_layer(cfg, t)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), ref["weights"].view(np.uint32))
    assert_close(to_numpy(out), ref["out"])


def test_batched_path_matches_cuda_core_path_in_child(cuda, native_lib):
    """The library reads LIVGLM_BATCHED_TC once per process: a child process
    with the switch off runs the CUDA-core grouped GEMV on the same layer, and
    both stay within the parity bar of each other."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    code = (
        "import sys, torch, numpy as np\n"
        f"sys.path.insert(0, {str(root)!r})\n"
        "from livglm_b200 import synthetic\n"
        "from livglm_b200.config import CONFIGS\n"
        "from livglm_b200.moe import build_layer\n"
        "cfg = CONFIGS['cfg0'].replace(hidden_size=1024, moe_intermediate_size=512)\n"
        "t = synthetic.layer_weights(cfg, seed=31, device='cuda')\n"
        "x = synthetic.hidden_states(cfg, 200, seed=32, device='cuda')\n"
        "out = build_layer(cfg, t)(x)\n"
        "np.save(sys.argv[1], out.cpu().numpy())\n"
    )
    paths = []
    for flag in ("1", "0"):
        p = root / "_build" / f"batched_tc_{flag}.npy"
        p.parent.mkdir(exist_ok=True)
        r = subprocess.run([sys.executable, "-c", code, str(p)], env=dict(os.environ, LIVGLM_BATCHED_TC=flag),
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-3000:]
        paths.append(p)
    a, b = (np.load(p) for p in paths)
    assert_close(a, b)


def test_static_workspace_size_unchanged_below_threshold(native_lib):
    """The batched tensor-core buffers are reserved only from 64 tokens on."""
    c = _native.LgConfig.from_config(CONFIGS["cfg1"])
    lib = native_lib
    assert lib.lg_moe_workspace_size(c, 63) < lib.lg_moe_workspace_size(c, 64)
