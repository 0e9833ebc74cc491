"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and rejects bad arguments on the host before touching the GPU."""

import ctypes
import re

import pytest

from livglm_b200 import _native
from livglm_b200.config import CONFIGS, ContractError, MoEConfig
from tests.conftest import ROOT


def declared_symbols(header: str = "livglm_moe.h") -> set[str]:
    text = (ROOT / "include" / header).read_text()
    return set(re.findall(r"\b(lg_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol(native_lib):
    names = declared_symbols()
    assert "lg_moe_forward" in names
    for name in names:
        assert hasattr(native_lib, name), name
    assert names == set(_native.SIGNATURES), names ^ set(_native.SIGNATURES)
    assert native_lib.lg_moe_abi_version() == 1


def test_ep_library_exports_every_declared_symbol(native_lib):
    headers = sorted(p.name for p in (ROOT / "include").glob("*.h"))
    assert headers == ["livglm_moe.h", "livglm_moe_ep.h"], headers
    ep = _native.load_ep()
    names = declared_symbols("livglm_moe_ep.h")
    assert "lg_moe_ep_forward" in names
    for name in names:
        assert hasattr(ep, name), name
    assert names == set(_native.EP_SIGNATURES), names ^ set(_native.EP_SIGNATURES)
    assert ep.lg_ep_unique_id_bytes() == 128


def test_ep_workspace_and_argument_checks(native_lib):
    ep = _native.load_ep()
    c = cfg_of()  # 128 experts
    one = native_lib.lg_moe_workspace_size(c, 64)
    s2 = ep.lg_moe_ep_workspace_size(c, 64, 2)
    s4 = ep.lg_moe_ep_workspace_size(c, 64, 4)
    assert s2 > one and s4 > s2 and s4 % 256 == 0  # receive side grows with the ranks
    assert ep.lg_moe_ep_workspace_size(c, 64, 3) == 0  # 128 experts do not split over 3 ranks
    assert "world" in ep.lg_ep_last_error().decode()
    assert ep.lg_moe_ep_workspace_size(c, 0, 2) == 0
    rc = ep.lg_moe_ep_forward(None, c, None, None, 0, None, None, None, None, 0, None)
    assert rc == _native.LG_ERR_INVALID_ARG
    assert "communicator" in ep.lg_ep_last_error().decode()
    handle = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * 128)()
    assert ep.lg_ep_comm_init(uid, 2, 2, 64, ctypes.byref(handle)) == _native.LG_ERR_INVALID_ARG
    assert ep.lg_ep_comm_init(uid, 2, 0, 0, ctypes.byref(handle)) == _native.LG_ERR_INVALID_ARG
    assert not handle.value
    assert ep.lg_ep_comm_destroy(None) == _native.LG_OK


def cfg_of(**kw):
    return _native.LgConfig.from_config(CONFIGS["cfg1"].replace(**kw) if kw else CONFIGS["cfg1"])


def test_workspace_size_grows_with_tokens(native_lib):
    c = cfg_of()
    s1 = native_lib.lg_moe_workspace_size(c, 1)
    s256 = native_lib.lg_moe_workspace_size(c, 256)
    assert 0 < s1 < s256
    assert s256 % 256 == 0


def test_workspace_size_rejects_bad_geometry(native_lib):
    bad = _native.LgConfig.from_config(CONFIGS["cfg1"])
    bad.n_group = 7  # 128 % 7 != 0
    assert native_lib.lg_moe_workspace_size(bad, 4) == 0
    assert "n_group" in _native.last_error()


@pytest.mark.parametrize("field,value,code", [
    ("hidden_size", 100, _native.LG_ERR_INVALID_ARG),
    ("topk_group", 9, _native.LG_ERR_INVALID_ARG),
    ("num_experts_per_tok", 0, _native.LG_ERR_INVALID_ARG),
    ("num_experts_per_tok", 33, _native.LG_ERR_UNSUPPORTED),
    ("n_routed_experts", 2048, _native.LG_ERR_UNSUPPORTED),
])
def test_router_validates_config_before_launch(native_lib, field, value, code):
    c = cfg_of()
    setattr(c, field, value)
    rc = native_lib.lg_moe_router(c, 16, 1, 16, 16, None, 16, 16, None, 0, None)
    assert rc == code, _native.last_error()


def test_null_pointers_are_argument_errors(native_lib):
    c = cfg_of()
    rc = native_lib.lg_moe_router(c, None, 1, None, None, None, None, None, None, 0, None)
    assert rc == _native.LG_ERR_INVALID_ARG
    assert "NULL" in _native.last_error()
    w = _native.LgWeights()
    rc = native_lib.lg_moe_forward(c, ctypes.byref(w), 16, 1, 16, None, None, None, 0, None)
    assert rc == _native.LG_ERR_INVALID_ARG


def test_misaligned_pointers_are_argument_errors(native_lib):
    c = cfg_of()
    rc = native_lib.lg_moe_router(c, 18, 1, 16, 16, 16, 16, 16, None, 0, None)
    assert rc == _native.LG_ERR_INVALID_ARG
    assert "aligned" in _native.last_error()


def test_missing_workspace_is_reported(native_lib):
    c = cfg_of()
    rc = native_lib.lg_moe_dispatch(c, 16, 4, 16, 16, 16, None, 0, None)
    assert rc == _native.LG_ERR_WORKSPACE


def test_zero_tokens_is_a_no_op(native_lib):
    c = cfg_of()
    assert native_lib.lg_moe_router(c, None, 0, None, None, None, None, None, None, 0, None) == 0
    w = _native.LgWeights()
    assert native_lib.lg_moe_experts(c, ctypes.byref(w), None, None, 0, None, None, 0, None) == 0
    assert native_lib.lg_moe_combine(c, None, None, None, 0, None, None) == 0


def test_check_maps_codes_to_exceptions():
    with pytest.raises(ContractError):
        _native.check(_native.LG_ERR_INVALID_ARG, "x")
    with pytest.raises(RuntimeError):
        _native.check(_native.LG_ERR_CUDA, "x")


def test_config_validation_mirrors_reference():
    """model_config.py:142-176."""
    with pytest.raises(ContractError, match="divisible by n_group"):
        MoEConfig(hidden_size=64, moe_intermediate_size=32, n_routed_experts=10,
                  num_experts_per_tok=2, n_group=3).validate()
    with pytest.raises(ContractError, match="at least two experts"):
        MoEConfig(hidden_size=64, moe_intermediate_size=32, n_routed_experts=4,
                  num_experts_per_tok=2, n_group=4, topk_group=1).validate()
    with pytest.raises(ContractError, match="sigmoid"):
        MoEConfig(hidden_size=64, moe_intermediate_size=32, n_routed_experts=4,
                  num_experts_per_tok=2, scoring_func="softmax").validate()
    text = {"hidden_size": 4096, "moe_intermediate_size": 2048, "n_routed_experts": 288,
            "num_experts_per_tok": 8, "n_shared_experts": 1, "n_group": 1, "topk_group": 1,
            "norm_topk_prob": True, "routed_scaling_factor": 2.5, "swiglu_limit": 10.0,
            "scoring_func": "sigmoid", "topk_method": "noaux_tc", "hidden_act": "silu"}
    assert MoEConfig.from_model_dict({"text_config": text}) == CONFIGS["glm53flash"]
    text["n_group"] = True
    with pytest.raises(ContractError, match="integer"):
        MoEConfig.from_text_config(text)
