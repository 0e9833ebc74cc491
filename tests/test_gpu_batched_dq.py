"""The batched routed experts with bf16-widened weights
(livglm_b200/csrc/grouped_dq.cuh) against the CPU oracle.

Tensor-core calls whose experts average at least 128 routes (M * k >= 128 * E)
run the routed gate/up and down as kind::f16 grouped GEMMs: converter warps
widen the MXFP4 weights to bf16 in shared memory and the B operand is the bf16
token rows (act for down) in dispatch order.  The products are exact, so the
outputs sit much closer to the oracle than the E2M1-term path's; the bar here
is the common one (routing bit-exact, max-abs 2e-2, cosine >= 0.9995) plus a
tighter max-abs that only the exact products meet.

Cases: the widening itself for every scale byte (table path and f32 path),
small geometries (d = 1024, F = 512, 16 experts, top-4) at M = 512 .. 4096
with uniform and strongly skewed routing (experts with thousands of routes:
many 256-route chunks; experts with none), and the path forced on for small
batches in a child process (chunks of one 32-route box).
"""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from livglm_b200 import synthetic
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from oracle import moe_oracle as mo
from tests.helpers import assert_close, bank_to_numpy, to_numpy

pytestmark = pytest.mark.gpu

SMALL = CONFIGS["cfg0"].replace(hidden_size=1024, moe_intermediate_size=512)
ROOT = Path(__file__).resolve().parent.parent
EXACT_MAX_ABS = 5e-3  # exact products: differences are f32 summation order + bf16 near-ties


def _selftest_lib():
    import ctypes

    from tests import build_selftest

    lib = ctypes.CDLL(str(build_selftest.build()))
    lib.lg_dq_widen_selftest.restype = ctypes.c_int
    lib.lg_dq_widen_selftest.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p]
    return lib


def test_widen_every_scale_byte(cuda):
    """E2M1 word x scale byte -> bf16, on all 256 scale bytes: bit-exact with
    the oracle's dequantisation rounded to bf16 (exact here), NaN for 255."""
    rng = np.random.default_rng(5)
    special = np.array([0, 0x88888888, 0x77777777, 0xFFFFFFFF, 0x76543210, 0xFEDCBA98], np.uint32)
    words = np.concatenate([special, rng.integers(0, 2 ** 32, 58, dtype=np.uint64).astype(np.uint32)])
    W = np.repeat(words, 256)
    S = np.tile(np.arange(256, dtype=np.uint8), len(words))
    lib = _selftest_lib()
    wd = torch.from_numpy(W.view(np.int32)).to(cuda)
    sd = torch.from_numpy(S).to(cuda)
    out = torch.empty(len(W) * 4, dtype=torch.int32, device=cuda)
    assert lib.lg_dq_widen_selftest(wd.data_ptr(), sd.data_ptr(), len(W), out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16).reshape(-1, 8)
    # the oracle's dequantisation (moe_oracle.mxfp4_dequant): E2M1 value x 2^(S - 127)
    nib = (W[:, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF
    with np.errstate(over="ignore", invalid="ignore"):
        ref = mo.E2M1_VALUES[nib] * mo.e8m0_to_f32(S)[:, None]
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(mo.bf16_bits_to_f32(got)))
    assert np.array_equal(got[~nan], mo.f32_to_bf16_bits(ref)[~nan])


def _bias_towards_first(cfg, strength: float, device):
    e = torch.arange(cfg.n_routed_experts, dtype=torch.float32, device=device)
    return -strength * torch.log1p(e)


@pytest.mark.parametrize("M,skew", [(512, 0.0), (1000, 0.0), (2048, 0.3), (4096, 1.5)])
def test_small_geometry_all_tokens(cuda, native_lib, M, skew):
    cfg = SMALL
    assert M * cfg.num_experts_per_tok >= 128 * cfg.n_routed_experts  # the bf16 path's range
    bias = _bias_towards_first(cfg, skew, cuda) if skew else None
    t = synthetic.layer_weights(cfg, seed=41, device=cuda, router_bias=bias)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=42 + M, device=cuda)
    moe = build_layer(cfg, t)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    ref = mo.moe_forward(to_numpy(x), tn, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), ref["weights"].view(np.uint32))
    assert_close(to_numpy(out), ref["out"], max_abs=EXACT_MAX_ABS)
    if skew > 1:  # chunks of several 256-route tiles for the popular experts, none for others
        counts = np.bincount(ref["indices"].reshape(-1).astype(np.int64), minlength=cfg.n_routed_experts)
        assert counts.max() > 1024 and (counts == 0).any()


def test_expert_entry_point(cuda, native_lib):
    """lg_moe_experts on the bf16 path: routed outputs bit-for-bit close to
    the oracle's (exact products; bf16 near-ties only)."""
    cfg = SMALL
    M = 1024
    t = synthetic.layer_weights(cfg, seed=51, device=cuda)
    tn = bank_to_numpy(t)
    x = synthetic.hidden_states(cfg, M, seed=52, device=cuda)
    moe = build_layer(cfg, t)
    _, _, idx = moe(x, return_route=True)
    y = moe.experts(x, idx)
    torch.cuda.synchronize()
    ref_y = mo.expert_outputs(to_numpy(x), tn, to_numpy(idx), cfg)
    got = to_numpy(y)
    assert_close(mo.bf16_bits_to_f32(got), ref_y, max_abs=EXACT_MAX_ABS)
    assert np.mean(got == mo.f32_to_bf16_bits(ref_y)) > 0.97


def test_forced_on_small_batches_in_child(cuda, native_lib):
    """LIVGLM_BATCHED_DQ=1 (read once per process) runs the bf16 path for
    batches far below its threshold: every chunk one partly filled 32-route
    box; outputs against the oracle in the parent."""
    code = (
        "import sys, torch, numpy as np\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "from livglm_b200 import synthetic\n"
        "from livglm_b200.config import CONFIGS\n"
        "from livglm_b200.moe import build_layer\n"
        "cfg = CONFIGS['cfg0'].replace(hidden_size=1024, moe_intermediate_size=512)\n"
        "t = synthetic.layer_weights(cfg, seed=61, device='cuda')\n"
        "outs = []\n"
        "for M in (64, 100, 333):\n"
        "    x = synthetic.hidden_states(cfg, M, seed=62 + M, device='cuda')\n"
        "    m = build_layer(cfg, t)\n"
        "    outs.append(m(x).cpu().numpy())\n"
        "    assert m.device_status() == 0\n"
        "np.savez(sys.argv[1], *outs)\n"
    )
    p = ROOT / "_build" / "batched_dq_forced.npz"
    p.parent.mkdir(exist_ok=True)
    r = subprocess.run([sys.executable, "-c", code, str(p)], env=dict(os.environ, LIVGLM_BATCHED_DQ="1"),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    cfg = SMALL
    t = synthetic.layer_weights(cfg, seed=61, device=cuda)
    tn = bank_to_numpy(t)
    with np.load(p) as z:
        outs = [z[f"arr_{i}"] for i in range(3)]
    for M, got in zip((64, 100, 333), outs):
        x = synthetic.hidden_states(cfg, M, seed=62 + M, device=cuda)
        ref = mo.moe_forward(to_numpy(x), tn, cfg)
        assert_close(got, ref["out"], max_abs=EXACT_MAX_ABS)
