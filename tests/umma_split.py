"""numpy restatement of the E2M1 activation split of livglm_b200/csrc/umma.cuh
(the checker for the tensor-core building blocks; test infrastructure).

A bf16 vector is written as T terms; term t holds, per 32-value block, one
UE8M0 scale byte 127 + e_t, e_t = max(s0 - 2t, -126) with s0 the smallest
integer such that 6 * 2^s0 >= the block's largest magnitude (at most 126),
and the round-to-nearest-even E2M1 codes (saturating at 6) of
residual / 2^e_t; the residual then loses the term's value.  Blocks whose
largest magnitude is below 2^-100 get code 0 and scale 127.  All arithmetic
in float32, as on the device.
"""

from __future__ import annotations

import numpy as np

GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def e2m1_rn(v: np.ndarray) -> np.ndarray:
    """float32 values -> 4-bit codes (sign in bit 3), nearest with ties to even, saturating at 6."""
    a = np.minimum(np.abs(v).astype(np.float32), np.float32(6))
    d = np.abs(a[..., None] - GRID)
    best = np.argmin(d, axis=-1)  # first of equal distances: the lower code
    nxt = np.minimum(best + 1, 7)
    tie = (np.take_along_axis(d, nxt[..., None], -1)[..., 0] == np.take_along_axis(d, best[..., None], -1)[..., 0])
    best = np.where(tie & (best % 2 == 1) & (nxt != best), nxt, best)
    return (best | (np.signbit(v).astype(np.int64) << 3)).astype(np.uint8)


def e2m1_value(code: np.ndarray) -> np.ndarray:
    v = GRID[code & 7]
    return np.where(code & 8, -v, v).astype(np.float32)


def split(x: np.ndarray, terms: int):
    """x float32 [K] (bf16 values) -> (codes u8 [T, K], scales u8 [T, K/32], residual f32 [K])."""
    K = x.shape[0]
    r = x.astype(np.float32).reshape(K // 32, 32).copy()
    codes = np.zeros((terms, K // 32, 32), np.uint8)
    scales = np.full((terms, K // 32), 127, np.uint8)
    a = np.max(np.abs(r), axis=1)
    live = a >= np.float32(2.0 ** -100)
    m, p = np.frexp(np.where(live, a, np.float32(1)))
    e0 = p.astype(np.int64) - 1
    s0 = np.minimum(np.where(2 * m <= 1.5, e0 - 2, e0 - 1), 126)
    for t in range(terms):
        e = np.maximum(s0 - 2 * t, -126)
        inv = np.ldexp(np.float32(1), -e).astype(np.float32)
        sc = np.ldexp(np.float32(1), e).astype(np.float32)
        c = e2m1_rn((r * inv[:, None]).astype(np.float32))
        c = np.where(live[:, None], c, 0).astype(np.uint8)
        q = e2m1_value(c)
        r = np.where(live[:, None], (r - (q * sc[:, None]).astype(np.float32)).astype(np.float32), r)
        codes[t] = c
        scales[t] = np.where(live, 127 + e, 127).astype(np.uint8)
    return codes.reshape(terms, K), scales, r.reshape(K)


def pack(codes: np.ndarray) -> np.ndarray:
    """[..., K] 4-bit codes -> [..., K/2] bytes, low nibble = even column."""
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def reconstruct(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Sum of the terms in float64 (exact: every term value is a short binary fraction)."""
    T, K = codes.shape
    v = e2m1_value(codes).astype(np.float64).reshape(T, K // 32, 32)
    s = np.ldexp(1.0, scales.astype(np.int64) - 127)[..., None]
    return (v * s).sum(axis=0).reshape(K)
