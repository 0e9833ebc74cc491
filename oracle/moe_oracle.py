"""CPU oracle of the GLM MoE block -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
import this module, and only as the checker; the product (livglm_b200) never
imports it.

It restates, in NumPy plus the small C library built from router_ref.c:

* TopKRouter.__call__            kg36/livglm src/glm53flash/moe.py:36-63
  (canonical fp32 order, see router_ref.c)
* MXFP4 decode implied by mx.gather_qmm(mode="mxfp4", group_size=32)
  on the byte-preserving U8 -> U32 view        expert_source.py:189-229
* ExpertSSD.__call__ (gate/up/SwiGLU/down)     expert_ssd.py:159-188
* limited_swiglu                               expert_ssd.py:103-107
* DenseMLP (bf16 shared expert)                layers.py:66-67,160-171
* the merge                                    moe.py:199-201

MLX rounds every op's result to the dtype of its inputs: with bf16 hidden
states gate, up, each SwiGLU op, the per-route down output and the shared
outputs are bf16; route weights are f32, so the merge is f32.  The oracle
rounds at exactly those points.  fp32 dot products use BLAS (order differs
from MLX and from the GPU; the tolerance covers it).

Pinning: the router is pinned by the reference's known-answer test
(tests/test_moe.py:10-23, restated in tests/test_oracle.py); the MXFP4 codec
is pinned against ml_dtypes' float4_e2m1fn / float8_e8m0fnu.  The expert
arithmetic has no golden vectors in the reference (its tests need MLX and a
170 GiB checkpoint): that part is "parity unpinned" beyond those pins.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import build_oracle

_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = build_oracle.OUT
        if not path.exists():
            build_oracle.build()
        _LIB = ctypes.CDLL(str(path))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C")
        _LIB.oracle_expf.argtypes = [f32p, f32p, ctypes.c_int64]
        _LIB.oracle_sigmoidf.argtypes = [f32p, f32p, ctypes.c_int64]
        _LIB.oracle_router.argtypes = [
            u16p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            ctypes.c_void_p, ctypes.c_void_p, f32p, u32p,
        ]
        _LIB.oracle_router.restype = ctypes.c_int
        _LIB.oracle_dispatch.argtypes = [u32p, ctypes.c_int64, ctypes.c_int, i32p, i32p, i32p]
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
        _LIB.oracle_moe_layer.argtypes = [
            u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, f32p, f32p,
            u8p, u8p, u8p, u8p, u8p, u8p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            f32p, f32p, u32p,
        ]
        _LIB.oracle_moe_layer.restype = ctypes.c_int
    return _LIB


# ---------------------------------------------------------------- bf16 ---

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit pattern (NaN stays NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------- MXFP4 ---

E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)


def e8m0_to_f32(s: np.ndarray) -> np.ndarray:
    s = np.asarray(s, dtype=np.uint8)
    e = np.where(s == 255, 0, s.astype(np.int32) - 127)
    out = np.ldexp(np.float64(1.0), e).astype(np.float32)
    out[s == 255] = np.nan
    return out


def e4m3fn_to_f32(codes: np.ndarray) -> np.ndarray:
    """E4M3FN bytes -> f32 (fp8.py:13-30): sign, 4-bit exponent (bias 7),
    3-bit mantissa, exponent 0 subnormal, 0x7F / 0xFF NaN, no infinities."""
    b = np.asarray(codes, np.uint8).astype(np.int64)
    e, m = (b >> 3) & 15, b & 7
    v = np.where(e == 0, np.ldexp(m / 8.0, -6), np.ldexp(1.0 + m / 8.0, e - 7))
    v = np.where((e == 15) & (m == 7), np.nan, v)
    return np.where(b & 0x80, -v, v).astype(np.float32)


def fp8_block_dequant_bf16(weight: np.ndarray, scale_inv: np.ndarray, block: int = 128) -> np.ndarray:
    """fp8.py:43-78 (decode, multiply the f32 block scale, f32 product), then
    the resident plan's bf16 destination (resident_plan.py:206-214): bf16 bits."""
    rows, cols = weight.shape
    dec = e4m3fn_to_f32(weight).reshape(rows // block, block, cols // block, block)
    prod = (dec * np.asarray(scale_inv, np.float32)[:, None, :, None]).astype(np.float32)
    return f32_to_bf16_bits(prod.reshape(rows, cols))


def mx_requantize_bf16(w_bits: np.ndarray, bits: int) -> np.ndarray:
    """Resident MXFP8 / MXFP4 quantisation of a bf16 matrix (layers.py:67-104,
    mx.quantize group 32) by the OCP MX rule -> bf16 bits of the quantised
    values: per 32-value group X = clamp(floor(log2 amax) - emax, -127, 127)
    (emax 8 for E4M3, 2 for E2M1; -127 for an all-zero group); element =
    round-to-nearest-even of v * 2^-X (f32 product) saturated to the largest
    finite element; value = element * 2^X.  MLX's own quantiser is not
    available here, so this restates the published rule."""
    import ml_dtypes

    v = bf16_bits_to_f32(np.asarray(w_bits, np.uint16))
    rows, cols = v.shape
    g = v.reshape(rows, cols // 32, 32)
    amax = np.abs(g).max(axis=-1)
    _, ex = np.frexp(amax)
    emax = 8 if bits == 8 else 2
    X = np.where(amax > 0, ex.astype(np.int64) - 1 - emax, -127).clip(-127, 127)
    down = np.ldexp(np.float32(1.0), -X).astype(np.float32)[..., None]
    up = np.ldexp(np.float32(1.0), X).astype(np.float32)[..., None]
    q = (g * down).astype(np.float32)
    if bits == 8:
        el = np.clip(q, -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn).astype(np.float32)
    else:
        el = np.clip(q, -6.0, 6.0).astype(ml_dtypes.float4_e2m1fn).astype(np.float32)
    return f32_to_bf16_bits((el * up).astype(np.float32).reshape(rows, cols))


def mxfp4_dequant(packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """U8 [rows, cols/2] nibbles (low nibble = even column) and U8 [rows,
    cols/32] E8M0 scales -> f32 [rows, cols] (value = E2M1 * 2^(s-127))."""
    packed = np.asarray(packed, dtype=np.uint8)
    rows, half = packed.shape
    codes = np.empty((rows, half * 2), dtype=np.uint8)
    codes[:, 0::2] = packed & 0x0F
    codes[:, 1::2] = packed >> 4
    vals = E2M1_VALUES[codes]
    s = e8m0_to_f32(scale)
    return (vals.reshape(rows, -1, 32) * s[:, :, None]).reshape(rows, half * 2)


# -------------------------------------------------------------- config ---

@dataclass(frozen=True)
class Geometry:
    hidden_size: int
    moe_intermediate_size: int
    n_routed_experts: int
    num_experts_per_tok: int
    n_shared_experts: int
    n_group: int
    topk_group: int
    norm_topk_prob: bool
    routed_scaling_factor: float
    swiglu_limit: float


def geometry(cfg) -> Geometry:
    return Geometry(
        int(cfg.hidden_size), int(cfg.moe_intermediate_size), int(cfg.n_routed_experts),
        int(cfg.num_experts_per_tok), int(cfg.n_shared_experts), int(cfg.n_group),
        int(cfg.topk_group), bool(cfg.norm_topk_prob), float(cfg.routed_scaling_factor),
        float(cfg.swiglu_limit),
    )


# -------------------------------------------------------------- router ---

def sigmoid(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_sigmoidf(x.reshape(-1), y.reshape(-1), x.size)
    return y


def own_exp(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_expf(x.reshape(-1), y.reshape(-1), x.size)
    return y


def router(x_bits: np.ndarray, weight: np.ndarray, bias: np.ndarray, cfg):
    """moe.py:36-63 -> (logits f32 [M,E], weights f32 [M,k], indices u32 [M,k])."""
    g = geometry(cfg)
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1, g.hidden_size)
    M = x_bits.shape[0]
    weight = np.ascontiguousarray(weight, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    logits = np.zeros((M, g.n_routed_experts), np.float32)
    wts = np.zeros((M, g.num_experts_per_tok), np.float32)
    idx = np.zeros((M, g.num_experts_per_tok), np.uint32)
    if M:
        rc = lib().oracle_router(
            x_bits, weight, bias, M, g.hidden_size, g.n_routed_experts, g.n_group,
            g.topk_group, g.num_experts_per_tok, int(g.norm_topk_prob),
            g.routed_scaling_factor, logits.ctypes.data, None, wts, idx,
        )
        if rc:
            raise ValueError("oracle router rejected the geometry")
    return logits, wts, idx


def dispatch(indices: np.ndarray, n_experts: int):
    """Stable counting sort of route slots by expert -> counts, offsets, perm."""
    flat = np.ascontiguousarray(indices, dtype=np.uint32).reshape(-1)
    counts = np.bincount(flat.astype(np.int64), minlength=n_experts).astype(np.int32)
    offsets = np.zeros(n_experts + 1, np.int32)
    np.cumsum(counts, out=offsets[1:])
    perm = np.argsort(flat, kind="stable").astype(np.int32)
    return counts, offsets, perm


# ------------------------------------------------------------- experts ---

def limited_swiglu_bf16(gate: np.ndarray, up: np.ndarray, limit: float) -> np.ndarray:
    """expert_ssd.py:103-107 on bf16 values, each op rounded to bf16."""
    gate = np.asarray(gate, np.float32)
    up = np.asarray(up, np.float32)
    if limit > 0:
        lim = np.float32(limit)
        gate = np.minimum(gate, lim)
        up = np.clip(up, -lim, lim)
    s = round_bf16(sigmoid(gate))
    a = round_bf16(gate * s)
    return round_bf16(a * up)


def expert_outputs(x: np.ndarray, bank: dict, indices: np.ndarray, cfg,
                   tokens: np.ndarray | None = None) -> np.ndarray:
    """ExpertSSD.__call__ (expert_ssd.py:159-188) -> bf16-valued f32 [T, k, d].

    x: bf16 bit patterns [M, d]; bank: the layer's stacked expert tensors
    (gate_packed [E,F,d/2], gate_scale [E,F,d/32], up_*, down_packed
    [E,d,F/2], down_scale [E,d,F/32]); tokens: optional subset of rows.
    """
    g = geometry(cfg)
    xf = bf16_bits_to_f32(np.asarray(x).reshape(-1, g.hidden_size))
    idx = np.asarray(indices).reshape(-1, g.num_experts_per_tok)
    if tokens is not None:
        xf, idx = xf[tokens], idx[tokens]
    T, k = idx.shape
    out = np.zeros((T, k, g.hidden_size), np.float32)
    for e in np.unique(idx):
        sel = np.argwhere(idx == e)
        rows = xf[sel[:, 0]]
        wg = mxfp4_dequant(bank["gate_packed"][e], bank["gate_scale"][e])
        wu = mxfp4_dequant(bank["up_packed"][e], bank["up_scale"][e])
        wd = mxfp4_dequant(bank["down_packed"][e], bank["down_scale"][e])
        gate = round_bf16(rows @ wg.T)
        up = round_bf16(rows @ wu.T)
        act = limited_swiglu_bf16(gate, up, g.swiglu_limit)
        y = round_bf16(act @ wd.T)
        out[sel[:, 0], sel[:, 1]] = y
    return out


def shared_expert(x: np.ndarray, bank: dict, cfg, tokens: np.ndarray | None = None) -> np.ndarray:
    """DenseMLP with bf16 weights (layers.py:66-67,160-171) -> bf16-valued f32."""
    g = geometry(cfg)
    xf = bf16_bits_to_f32(np.asarray(x).reshape(-1, g.hidden_size))
    if tokens is not None:
        xf = xf[tokens]
    wg = bf16_bits_to_f32(bank["shared_gate"])
    wu = bf16_bits_to_f32(bank["shared_up"])
    wd = bf16_bits_to_f32(bank["shared_down"])
    gate = round_bf16(xf @ wg.T)
    up = round_bf16(xf @ wu.T)
    act = limited_swiglu_bf16(gate, up, g.swiglu_limit)
    return round_bf16(act @ wd.T)


def combine(y: np.ndarray, weights: np.ndarray, shared: np.ndarray | None) -> np.ndarray:
    """moe.py:199-201: f32 products, summed in route order, plus shared."""
    y = np.asarray(y, np.float32)
    w = np.asarray(weights, np.float32)
    acc = np.zeros(y.shape[0:1] + y.shape[2:], np.float32)
    for j in range(y.shape[1]):
        acc = acc + y[:, j, :] * w[:, j, None]
    if shared is not None:
        acc = acc + np.asarray(shared, np.float32)
    return acc


def moe_forward(x: np.ndarray, bank: dict, cfg, tokens: np.ndarray | None = None) -> dict:
    """ExpertSSDMoE.__call__ (moe.py:96-201) for bf16 hidden states.

    Returns a dict with logits, weights, indices (all tokens), and for the
    selected tokens: y (per-route outputs), shared, out (f32 merge).
    """
    g = geometry(cfg)
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1, g.hidden_size)
    if tokens is None:
        logits, wts, idx = router(x, bank["router_weight"], bank["router_bias"], cfg)
        sel = np.arange(x.shape[0])
    else:
        sel = np.asarray(tokens)
        logits, wts, idx = router(x[sel], bank["router_weight"], bank["router_bias"], cfg)
    xs = x[sel]
    y = expert_outputs(xs, bank, idx, cfg)
    sh = shared_expert(xs, bank, cfg) if g.n_shared_experts > 0 else None
    out = combine(y, wts, sh)
    return {"logits": logits, "weights": wts, "indices": idx, "y": y, "shared": sh, "out": out,
            "tokens": sel}


def moe_forward_c(x: np.ndarray, bank: dict, cfg) -> dict:
    """The whole block through the C restatement (experts_ref.c: MXFP4 decoded
    on the fly, OpenMP over weight rows) -> {"out", "weights", "indices"}.
    Routing is the canonical router's (bit-identical to router()); outputs
    agree with moe_forward() to within f32 summation order."""
    g = geometry(cfg)
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1, g.hidden_size)
    M = x.shape[0]
    d, F, E, k = g.hidden_size, g.moe_intermediate_size, g.n_routed_experts, g.num_experts_per_tok
    Fs = F * g.n_shared_experts
    out = np.zeros((M, d), np.float32)
    wts = np.zeros((M, k), np.float32)
    idx = np.zeros((M, k), np.uint32)
    if M == 0:
        return {"out": out, "weights": wts, "indices": idx}
    c = np.ascontiguousarray
    shared = [c(bank["shared_gate"], dtype=np.uint16), c(bank["shared_up"], dtype=np.uint16),
              c(bank["shared_down"], dtype=np.uint16)] if Fs else [None, None, None]
    rc = lib().oracle_moe_layer(
        x, M, d, F, Fs, E, g.n_group, g.topk_group, k, int(g.norm_topk_prob), g.routed_scaling_factor,
        g.swiglu_limit, c(bank["router_weight"], dtype=np.float32), c(bank["router_bias"], dtype=np.float32),
        c(bank["gate_packed"], dtype=np.uint8), c(bank["gate_scale"], dtype=np.uint8),
        c(bank["up_packed"], dtype=np.uint8), c(bank["up_scale"], dtype=np.uint8),
        c(bank["down_packed"], dtype=np.uint8), c(bank["down_scale"], dtype=np.uint8),
        *[a.ctypes.data if a is not None else None for a in shared], out, wts, idx)
    if rc:
        raise ValueError(f"C oracle rejected the call ({rc})")
    return {"out": out, "weights": wts, "indices": idx}
