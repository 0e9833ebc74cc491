"""Checkpoint reading on the CPU: the safetensors reader against files
written by tests/st_writer.py, its refusal of malformed files, and the
oracle's E4M3FN decoding against ml_dtypes."""

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
