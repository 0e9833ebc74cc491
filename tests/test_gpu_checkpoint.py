"""Checkpoint loading on the GPU: block-FP8 widening (lg_fp8_block_dequant)
against the oracle's restatement of fp8.py:43-78, and a layer built with
ExpertSSDMoE.from_checkpoint from a safetensors checkpoint (index + two
shards, FP8 shared expert) against the oracle."""

import numpy as np
import pytest
import torch

from livglm_b200.config import CONFIGS, ContractError
from livglm_b200.moe import ExpertSSDMoE, widen_block_fp8
from oracle import moe_oracle as mo
from tests import checkpoint_fixture as cf
from tests.helpers import assert_close, to_numpy

pytestmark = pytest.mark.gpu


def test_fp8_widening_bit_exact(cuda, native_lib):
    rng = np.random.default_rng(3)
    w, s = cf.fp8_weight(rng, 384, 512)
    w[0, :254] = np.array([c for c in range(256) if c & 0x7F != 0x7F], np.uint8)  # every finite code
    got = widen_block_fp8(torch.from_numpy(w).to(cuda).view(torch.float8_e4m3fn), torch.from_numpy(s).to(cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy(got), mo.fp8_block_dequant_bf16(w, s))


def test_fp8_widening_reference_known_answers(cuda, native_lib):
    """kg36/livglm tests/test_fp8.py:15-29 on the GPU: code 0x38 (1.0) times a
    block scale of 2.5, and a 2 x 2 scale grid over four 128 x 128 quadrants."""
    one = torch.full((128, 128), 0x38, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    got = widen_block_fp8(one, torch.tensor([[2.5]], device=cuda))
    four = torch.full((256, 256), 0x38, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    quad = widen_block_fp8(four, torch.tensor([[1.0, 2.0], [3.0, 4.0]], device=cuda))
    torch.cuda.synchronize()
    assert torch.all(got.float() == 2.5)
    q = quad.float().cpu()
    assert torch.all(q[:128, :128] == 1.0) and torch.all(q[:128, 128:] == 2.0)
    assert torch.all(q[128:, :128] == 3.0) and torch.all(q[128:, 128:] == 4.0)


def test_fp8_widening_refuses_nan(cuda, native_lib):
    rng = np.random.default_rng(4)
    w, s = cf.fp8_weight(rng, 128, 128)
    w[5, 7] = 0x7F
    with pytest.raises(ContractError):
        widen_block_fp8(torch.from_numpy(w).to(cuda).view(torch.float8_e4m3fn), torch.from_numpy(s).to(cuda))


def test_layer_from_checkpoint_matches_oracle(tmp_path, cuda, native_lib, golden_cfg0):
    cfg = CONFIGS["cfg0"]
    bank = cf.build(tmp_path / "ckpt", golden_cfg0, cfg)
    moe = ExpertSSDMoE.from_checkpoint(tmp_path / "ckpt", cfg, cf.LAYER, device=cuda)
    for name in ("gate", "up", "down"):
        np.testing.assert_array_equal(to_numpy(getattr(moe.shared_experts, f"{name}_proj").weight),
                                      bank[f"shared_{name}"])
    x = torch.from_numpy(golden_cfg0["x"].view(np.int16)).to(cuda).view(torch.bfloat16)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    ref = mo.moe_forward(golden_cfg0["x"], bank, cfg)
    np.testing.assert_array_equal(to_numpy(idx), ref["indices"])
    assert_close(to_numpy(out), ref["out"])


@pytest.mark.parametrize("bits", [8, 4])
def test_mx_requantize_bit_exact(cuda, native_lib, bits):
    from livglm_b200 import _native
    from livglm_b200.moe import _stream_ptr

    rng = np.random.default_rng(10 + bits)
    w = (rng.standard_normal((96, 512)) * np.exp(rng.uniform(-8, 3, (96, 1)))).astype(np.float32)
    w[5, :64] = 0.0
    wb = mo.f32_to_bf16_bits(w)
    t = torch.from_numpy(wb.view(np.int16)).to(cuda).view(torch.bfloat16)
    out = torch.empty_like(t)
    assert _native.load().lg_mx_requantize(t.data_ptr(), 96, 512, bits, out.data_ptr(), _stream_ptr(cuda)) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy(out), mo.mx_requantize_bf16(wb, bits))


def test_layer_with_mxfp8_shared_expert(cuda, native_lib, golden_cfg0):
    """quantize_resident_linears_mxfp(8), the reference runtime's default
    resident quantisation, against the oracle fed the same quantised shared
    weights."""
    from livglm_b200.moe import build_layer
    from oracle.torch_bridge import bank_to_device

    cfg = CONFIGS["cfg0"]
    moe = build_layer(cfg, bank_to_device(golden_cfg0, cuda))
    info = moe.quantize_resident_linears_mxfp(8)
    assert info["linears"] == 3 and info["destination_bytes"] < info["source_bytes"]
    # per linear: 2 bytes per bf16 value before, one E4M3 byte per value and
    # one scale byte per 32 after (kg36/livglm tests/test_resident_mxfp8.py:21-22)
    n = 3 * cfg.hidden_size * cfg.shared_intermediate_size
    assert (info["source_bytes"], info["destination_bytes"]) == (2 * n, n + n // 32)
    bank = dict(golden_cfg0)
    for name in ("gate", "up", "down"):
        bank[f"shared_{name}"] = mo.mx_requantize_bf16(golden_cfg0[f"shared_{name}"], 8)
        np.testing.assert_array_equal(to_numpy(getattr(moe.shared_experts, f"{name}_proj").weight),
                                      bank[f"shared_{name}"])
    x = torch.from_numpy(golden_cfg0["x"].view(np.int16)).to(cuda).view(torch.bfloat16)
    out = moe(x)
    torch.cuda.synchronize()
    assert_close(to_numpy(out), mo.moe_forward(golden_cfg0["x"], bank, cfg)["out"])
