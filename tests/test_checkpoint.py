"""Checkpoint reading on the CPU: the safetensors reader against files
written by tests/st_writer.py, its refusal of malformed files, the oracle's
E4M3FN decoding against ml_dtypes, and the oracle's block-FP8 and resident
MXFP8 / MXFP4 transforms against the known answers and bounds of the
reference's own tests (kg36/livglm tests/test_fp8.py,
tests/test_resident_mxfp8.py)."""

import json

import ml_dtypes
import numpy as np
import pytest
import torch

from livglm_b200.config import CONFIGS, ContractError
from livglm_b200.safetensors import SafetensorsCheckpoint
from oracle import moe_oracle as mo
from tests import checkpoint_fixture as cf
from tests import st_writer


def test_reader_returns_every_tensor_byte_for_byte(tmp_path, golden_cfg0):
    cfg = CONFIGS["cfg0"]
    cf.build(tmp_path / "ckpt", golden_cfg0, cfg)
    ckpt = SafetensorsCheckpoint(tmp_path / "ckpt")
    p = f"model.language_model.layers.{cf.LAYER}.mlp."
    layer = ckpt.layer_tensors(cf.LAYER)
    assert len(layer) == 2 + 6 + 6 * cfg.n_routed_experts
    np.testing.assert_array_equal(layer[p + "gate.weight"].numpy(), golden_cfg0["router_weight"])
    for e in (0, 7, cfg.n_routed_experts - 1):
        t = layer[p + f"experts.{e}.down_proj.weight_packed"]
        assert t.dtype == torch.uint8
        np.testing.assert_array_equal(t.numpy(), golden_cfg0["down_packed"][e])
    w = layer[p + "shared_experts.up_proj.weight"]
    assert w.dtype == torch.float8_e4m3fn and tuple(w.shape) == (cfg.shared_intermediate_size, cfg.hidden_size)
    assert ckpt.info(p + "experts.0.gate_proj.weight_scale").shard.name.startswith("model-00002")


def test_reader_single_file_and_bf16(tmp_path):
    x = mo.f32_to_bf16_bits(np.linspace(-2, 2, 64, dtype=np.float32).reshape(8, 8))
    st_writer.write(tmp_path / "one.safetensors", {"a": ("BF16", x), "b": ("I32", np.arange(5, dtype=np.int32))})
    ckpt = SafetensorsCheckpoint(tmp_path / "one.safetensors")
    a = ckpt.tensor("a")
    assert a.dtype == torch.bfloat16
    np.testing.assert_array_equal(a.view(torch.int16).numpy().view(np.uint16), x)
    np.testing.assert_array_equal(ckpt.tensor("b").numpy(), np.arange(5))


def test_reader_refuses_malformed_files(tmp_path):
    st_writer.write(tmp_path / "ok.safetensors", {"a": ("F32", np.zeros(4, np.float32))})
    raw = (tmp_path / "ok.safetensors").read_bytes()
    (tmp_path / "short.safetensors").write_bytes(raw[:-4])  # data cut short
    with pytest.raises(ContractError):
        SafetensorsCheckpoint(tmp_path / "short.safetensors")
    (tmp_path / "hdr.safetensors").write_bytes((10 ** 12).to_bytes(8, "little") + raw[8:])
    with pytest.raises(ContractError):
        SafetensorsCheckpoint(tmp_path / "hdr.safetensors")
    bad = tmp_path / "dir"
    bad.mkdir()
    st_writer.write(bad / "s1.safetensors", {"a": ("F32", np.zeros(4, np.float32))})
    (bad / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"b": "s1.safetensors"}}))
    with pytest.raises(ContractError):
        SafetensorsCheckpoint(bad)
    with pytest.raises(ContractError):
        SafetensorsCheckpoint(tmp_path / "ok.safetensors").tensor("missing")


def test_e4m3fn_decode_matches_ml_dtypes_for_every_code():
    codes = np.arange(256, dtype=np.uint8)
    ref = codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    got = mo.e4m3fn_to_f32(codes)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_array_equal(got[~np.isnan(ref)], ref[~np.isnan(ref)])


def test_fp8_block_dequant_oracle_blocks():
    rng = np.random.default_rng(1)
    w, s = cf.fp8_weight(rng, 256, 384)
    got = mo.bf16_bits_to_f32(mo.fp8_block_dequant_bf16(w, s))
    dec = w.view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    ref = (dec * np.repeat(np.repeat(s, 128, 0), 128, 1)).astype(np.float32)
    np.testing.assert_array_equal(got, mo.bf16_bits_to_f32(mo.f32_to_bf16_bits(ref)))


def test_mx_requantize_oracle_properties():
    """The resident MXFP4 rule agrees with the independent quantizer used for
    the synthetic routed weights (livglm_b200/mxfp4.py); both rules are
    idempotent and keep every value on the element grid times 2^X."""
    from livglm_b200.mxfp4 import dequantize_mxfp4, quantize_mxfp4

    rng = np.random.default_rng(2)
    w = (rng.standard_normal((48, 256)) * np.exp(rng.uniform(-6, 2, (48, 1)))).astype(np.float32)
    w[3, 32:64] = 0.0  # an all-zero group
    wb = mo.f32_to_bf16_bits(w)
    q4 = mo.mx_requantize_bf16(wb, 4)
    p, s = quantize_mxfp4(torch.from_numpy(mo.bf16_bits_to_f32(wb)))
    np.testing.assert_array_equal(mo.bf16_bits_to_f32(q4), dequantize_mxfp4(p, s).numpy())
    for bits in (4, 8):
        q = mo.mx_requantize_bf16(wb, bits)
        np.testing.assert_array_equal(mo.mx_requantize_bf16(q, bits), q)
    q8 = mo.bf16_bits_to_f32(mo.mx_requantize_bf16(wb, 8))
    assert np.all(q8[3, 32:64] == 0)
    rel = np.abs(q8 - mo.bf16_bits_to_f32(wb)) / np.abs(mo.bf16_bits_to_f32(wb)).reshape(48, 8, 32).max(-1).repeat(32, 1)
    assert np.nanmax(rel) <= 0.125 + 1e-6  # 3-bit mantissa, and the OCP rule may clamp a group max into 448


# ------------------------------------------- the reference's known answers ---

def test_e4m3fn_reference_known_values():
    """kg36/livglm tests/test_fp8.py:8-12."""
    codes = np.array([0x00, 0x01, 0x38, 0x3C, 0x7E, 0xB8], np.uint8)
    np.testing.assert_array_equal(mo.e4m3fn_to_f32(codes),
                                  np.array([0.0, 2.0 ** -9, 1.0, 1.5, 448.0, -1.0], np.float32))


def test_block_fp8_reference_scale_and_quadrants():
    """kg36/livglm tests/test_fp8.py:15-29: one block times 2.5; a 2 x 2 scale
    grid maps onto the matrix quadrants."""
    one = np.full((128, 128), 0x38, np.uint8)
    got = mo.bf16_bits_to_f32(mo.fp8_block_dequant_bf16(one, np.array([[2.5]], np.float32)))
    np.testing.assert_array_equal(got, np.full((128, 128), 2.5, np.float32))
    four = np.full((256, 256), 0x38, np.uint8)
    got = mo.bf16_bits_to_f32(mo.fp8_block_dequant_bf16(four, np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)))
    assert np.all(got[:128, :128] == 1.0) and np.all(got[:128, 128:] == 2.0)
    assert np.all(got[128:, :128] == 3.0) and np.all(got[128:, 128:] == 4.0)


def test_block_fp8_reference_non_finite_code():
    """kg36/livglm tests/test_fp8.py:32-36: code 0x7F is NaN (the GPU widening
    refuses it, tests/test_gpu_checkpoint.py)."""
    assert np.isnan(mo.e4m3fn_to_f32(np.array([0x7F, 0xFF], np.uint8))).all()
    got = mo.bf16_bits_to_f32(mo.fp8_block_dequant_bf16(np.full((128, 128), 0x7F, np.uint8),
                                                        np.array([[1.0]], np.float32)))
    assert np.isnan(got).all()


@pytest.mark.parametrize("bits,seed,rtol,atol", [(8, 5308, 0.03, 0.015), (4, 5304, 0.20, 0.04)])
def test_resident_mx_reference_closeness(bits, seed, rtol, atol):
    """kg36/livglm tests/test_resident_mxfp8.py: a 64 x 32 bf16 linear of N(0,
    0.05) weights on two N(0, 0.2) rows stays within the reference test's
    tolerance after resident MXFP8 (rtol 0.03, atol 0.015) / MXFP4 (0.20,
    0.04) quantisation (the byte counts it also checks are checked on the GPU
    module, tests/test_gpu_checkpoint.py)."""
    rng = np.random.default_rng(seed)
    w = mo.f32_to_bf16_bits(rng.normal(0, 0.05, (64, 32)).astype(np.float32))
    x = mo.f32_to_bf16_bits(rng.normal(0, 0.2, (2, 32)).astype(np.float32))

    def linear(wb):  # bf16 x @ W^T with f32 sums, rounded to bf16
        return mo.round_bf16((mo.bf16_bits_to_f32(x).astype(np.float64) @ mo.bf16_bits_to_f32(wb).T
                              .astype(np.float64)).astype(np.float32))

    expected = linear(w)
    actual = linear(mo.mx_requantize_bf16(w, bits))
    np.testing.assert_allclose(actual, expected, rtol=rtol, atol=atol)
