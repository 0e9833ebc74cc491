"""ctypes binding of the C ABI in include/livglm_moe.h.

The shared library is built in-tree (livglm_b200/_lib/liblivglm_moe.so) by
livglm_b200/build.py.  There is no fallback: if the library is missing every
call raises, so a GPU run can never silently take another path.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

from .config import ContractError, MoEConfig

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "liblivglm_moe.so"
EP_LIB_PATH = LIB_DIR / "liblivglm_moe_ep.so"

LG_OK = 0
LG_ERR_INVALID_ARG = 1
LG_ERR_UNSUPPORTED = 2
LG_ERR_WORKSPACE = 3
LG_ERR_CUDA = 4
LG_ERR_NCCL = 5
LG_ERR_TIMEOUT = 6

ERROR_NAMES = {
    LG_ERR_INVALID_ARG: "LG_ERR_INVALID_ARG",
    LG_ERR_UNSUPPORTED: "LG_ERR_UNSUPPORTED",
    LG_ERR_WORKSPACE: "LG_ERR_WORKSPACE",
    LG_ERR_CUDA: "LG_ERR_CUDA",
    LG_ERR_NCCL: "LG_ERR_NCCL",
    LG_ERR_TIMEOUT: "LG_ERR_TIMEOUT",
}


class LgConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("moe_intermediate_size", ctypes.c_int32),
        ("n_routed_experts", ctypes.c_int32),
        ("num_experts_per_tok", ctypes.c_int32),
        ("n_shared_experts", ctypes.c_int32),
        ("n_group", ctypes.c_int32),
        ("topk_group", ctypes.c_int32),
        ("norm_topk_prob", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
        ("swiglu_limit", ctypes.c_float),
    ]

    @classmethod
    def from_config(cls, c: MoEConfig) -> "LgConfig":
        return cls(c.hidden_size, c.moe_intermediate_size, c.n_routed_experts,
                   c.num_experts_per_tok, c.n_shared_experts, c.n_group, c.topk_group,
                   int(bool(c.norm_topk_prob)), float(c.routed_scaling_factor),
                   float(c.swiglu_limit))


class LgHcConfig(ctypes.Structure):
    _fields_ = [
        ("hc_mult", ctypes.c_int32),
        ("sinkhorn_iters", ctypes.c_int32),
        ("hc_eps", ctypes.c_float),
        ("rms_norm_eps", ctypes.c_float),
    ]


class LgHcWeights(ctypes.Structure):
    _fields_ = [
        ("fn", ctypes.c_void_p),
        ("base", ctypes.c_void_p),
        ("scale", ctypes.c_void_p),
        ("norm_weight", ctypes.c_void_p),
    ]


class LgWeights(ctypes.Structure):
    _fields_ = [
        ("router_weight", ctypes.c_void_p),
        ("router_bias", ctypes.c_void_p),
        ("gate_packed", ctypes.c_void_p),
        ("gate_scale", ctypes.c_void_p),
        ("up_packed", ctypes.c_void_p),
        ("up_scale", ctypes.c_void_p),
        ("down_packed", ctypes.c_void_p),
        ("down_scale", ctypes.c_void_p),
        ("gate_packed_stride", ctypes.c_int64),
        ("gate_scale_stride", ctypes.c_int64),
        ("up_packed_stride", ctypes.c_int64),
        ("up_scale_stride", ctypes.c_int64),
        ("down_packed_stride", ctypes.c_int64),
        ("down_scale_stride", ctypes.c_int64),
        ("shared_gate", ctypes.c_void_p),
        ("shared_up", ctypes.c_void_p),
        ("shared_down", ctypes.c_void_p),
    ]


# name -> (restype, argtypes); every symbol include/livglm_moe.h declares.
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_CFG = ctypes.POINTER(LgConfig)
_W = ctypes.POINTER(LgWeights)
_HC = ctypes.POINTER(LgHcConfig)
_HW = ctypes.POINTER(LgHcWeights)
SIGNATURES = {
    "lg_moe_abi_version": (ctypes.c_int, []),
    "lg_moe_last_error": (ctypes.c_char_p, []),
    "lg_moe_workspace_size": (ctypes.c_size_t, [_CFG, _I64]),
    "lg_moe_router": (ctypes.c_int, [_CFG, _P, _I64, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_dispatch": (ctypes.c_int, [_CFG, _P, _I64, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_experts": (ctypes.c_int, [_CFG, _W, _P, _P, _I64, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_shared": (ctypes.c_int, [_CFG, _W, _P, _I64, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_combine": (ctypes.c_int, [_CFG, _P, _P, _P, _I64, _P, _P]),
    "lg_moe_combine_gather": (ctypes.c_int, [_CFG, _P, _P, _P, _P, _I64, _P, _P]),
    "lg_moe_ep_pack": (ctypes.c_int, [_CFG, _P, _I64, _P, _P, ctypes.c_int32, _P, _P, _P, _P]),
    "lg_fp8_block_dequant": (ctypes.c_int, [_P, _P, _I64, _I64, ctypes.c_int32, _P, _P, _P]),
    "lg_mx_requantize": (ctypes.c_int, [_P, _I64, _I64, ctypes.c_int32, _P, _P]),
    "lg_moe_forward": (ctypes.c_int, [_CFG, _W, _P, _I64, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_forward_static_scratch": (ctypes.c_int, [_CFG, _W, _P, _I64, _P, _P, _P, _P]),
    "lg_moe_static_scratch_status": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int32), _P]),
    "lg_moe_check_wait_timeout": (ctypes.c_int, [_I64, _P, _P]),
    "lg_moe_trace_enable": (ctypes.c_int, [ctypes.c_int]),
    "lg_hc_workspace_size": (ctypes.c_size_t, [_HC, ctypes.c_int32, _I64]),
    "lg_hc_pre": (ctypes.c_int, [_HC, _HW, ctypes.c_int32, _P, _I64, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "lg_hc_post": (ctypes.c_int, [_HC, ctypes.c_int32, _P, _P, _P, _P, _I64, _P, _P]),
    "lg_moe_ffn_site_workspace_size": (ctypes.c_size_t, [_CFG, _HC, _I64]),
    "lg_moe_ffn_site": (ctypes.c_int, [_CFG, _W, _HC, _HW, _P, _I64, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "lg_moe_trace_read": (ctypes.c_int, [ctypes.POINTER(ctypes.c_float), ctypes.c_int]),
}

# every symbol include/livglm_moe_ep.h declares.
EP_SIGNATURES = {
    "lg_ep_unique_id_bytes": (ctypes.c_int, []),
    "lg_ep_get_unique_id": (ctypes.c_int, [_P]),
    "lg_ep_comm_init": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_int32, _I64, ctypes.POINTER(_P)]),
    "lg_ep_comm_destroy": (ctypes.c_int, [_P]),
    "lg_ep_last_error": (ctypes.c_char_p, []),
    "lg_moe_ep_workspace_size": (ctypes.c_size_t, [_CFG, _I64, ctypes.c_int32]),
    "lg_moe_ep_forward": (ctypes.c_int, [_P, _CFG, _W, _P, _I64, _P, _P, _P, _P, ctypes.c_size_t, _P]),
}

TRACE_STAGES = ("router", "dispatch", "gate_up", "down", "combine")


def trace_enable(capacity_calls: int) -> None:
    check(load().lg_moe_trace_enable(int(capacity_calls)), "lg_moe_trace_enable")


def trace_read(max_calls: int) -> list[dict[str, float]]:
    """Per-call stage durations (ms) of the traced lg_moe_forward calls."""
    buf = (ctypes.c_float * (max_calls * len(TRACE_STAGES)))()
    n = load().lg_moe_trace_read(buf, max_calls)
    if n < 0:
        check(-n, "lg_moe_trace_read")
    k = len(TRACE_STAGES)
    return [dict(zip(TRACE_STAGES, buf[c * k:(c + 1) * k])) for c in range(n)]

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the CUDA library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"livglm_b200 CUDA library missing at {LIB_PATH}; build it with "
                "`python -m livglm_b200.build` (there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


_ep_lib: ctypes.CDLL | None = None


def load_ep() -> ctypes.CDLL:
    """Load the expert-parallel library (liblivglm_moe_ep.so).  torch is
    imported first so that the libnccl.so.2 torch.distributed uses is the one
    the library binds to; the main library is loaded first so that both share
    one instance of it."""
    global _ep_lib
    if _ep_lib is None:
        import torch  # noqa: F401  (loads torch's NCCL)

        load()
        if not EP_LIB_PATH.exists():
            raise RuntimeError(f"livglm_b200 expert-parallel library missing at {EP_LIB_PATH}; build it with "
                               "`python -m livglm_b200.build`")
        lib = ctypes.CDLL(str(EP_LIB_PATH))
        for name, (res, args) in EP_SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _ep_lib = lib
    return _ep_lib


def ep_check(rc: int, what: str) -> None:
    if rc == LG_OK:
        return
    msg = load_ep().lg_ep_last_error()
    text = f"{what}: {ERROR_NAMES.get(rc, rc)}: {msg.decode() if msg else ''}"
    if rc in (LG_ERR_INVALID_ARG, LG_ERR_UNSUPPORTED, LG_ERR_WORKSPACE):
        raise ContractError(text)
    raise RuntimeError(text)


def last_error() -> str:
    msg = load().lg_moe_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc == LG_OK:
        return
    msg = f"{what}: {ERROR_NAMES.get(rc, rc)}: {last_error()}"
    if rc in (LG_ERR_INVALID_ARG, LG_ERR_UNSUPPORTED, LG_ERR_WORKSPACE):
        raise ContractError(msg)
    raise RuntimeError(msg)
