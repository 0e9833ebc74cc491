"""Tensor-core (tcgen05) building blocks against their checkers, on one
128-row tile (tests/csrc/umma_selftest.cu, built by tests/build_selftest.py
over the product's livglm_b200/csrc/umma.cuh):

* the E2M1 activation split equals its numpy restatement (tests/umma_split.py)
  byte for byte;
* the block-scaled kind::mxf4 MMA chain over those terms gives the MXFP4
  weights (the oracle's dequantisation) times the bf16 activations within
  f32 accumulation error;
* the kind::f16 MMA chain with bf16 weights does the same for the shared
  expert's format.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as mo
from tests import build_selftest
from tests.umma_split import pack, reconstruct, split

pytestmark = pytest.mark.gpu

_P = ctypes.c_void_p


@pytest.fixture(scope="module")
def umma_lib(cuda):
    lib = ctypes.CDLL(str(build_selftest.build()))
    fn = lib.lg_umma_selftest_tile
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, _P, _P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P, _P, _P]
    return lib


def bf16_vector(rng, n, scale=1.0):
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    return mo.f32_to_bf16_bits(x)


def run(lib, cuda, kind, w, wscale, x_bits, K, T):
    dw = torch.from_numpy(w).to(cuda)
    ds = torch.from_numpy(wscale).to(cuda) if wscale is not None else None
    dx = torch.from_numpy(x_bits.view(np.int16)).to(cuda)
    y = torch.full((128,), float("nan"), dtype=torch.float32, device=cuda)
    terms = torch.zeros(max(T, 1) * K // 2, dtype=torch.uint8, device=cuda)
    tsc = torch.zeros(max(T, 1) * K // 32, dtype=torch.uint8, device=cuda)
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = lib.lg_umma_selftest_tile(kind, dw.data_ptr(), ds.data_ptr() if ds is not None else None, dx.data_ptr(), K, T,
                                   y.data_ptr(), terms.data_ptr(), tsc.data_ptr(), st.data_ptr(),
                                   torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0 and int(st.item()) == 0
    return (y.cpu().numpy(), terms.cpu().numpy().reshape(max(T, 1), K // 2),
            tsc.cpu().numpy().reshape(max(T, 1), K // 32))


@pytest.mark.parametrize("K,T,xscale", [(4096, 16, 1.0), (256, 1, 1.0), (1536, 6, 1e-2), (512, 32, 40.0)])
def test_mxf4_tile_over_split_activations(umma_lib, cuda, K, T, xscale):
    rng = np.random.default_rng(K + T)
    w = rng.integers(0, 256, size=(128, K // 2), dtype=np.uint8)
    ws = rng.integers(118, 128, size=(128, K // 32), dtype=np.uint8)
    xb = bf16_vector(rng, K, xscale)
    x = mo.bf16_bits_to_f32(xb)
    y, terms, tsc = run(umma_lib, cuda, 0, w, ws, xb, K, T)
    codes, scales, _ = split(x, T)
    np.testing.assert_array_equal(terms, pack(codes))
    np.testing.assert_array_equal(tsc, scales)
    W = mo.mxfp4_dequant(w, ws).astype(np.float64)
    xt = reconstruct(codes, scales)  # the activations the MMAs see (== x once the split is exact)
    ref = W @ xt
    bound = 4e-6 * (np.abs(W) @ np.abs(xt)) + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
    if T >= 16:
        np.testing.assert_array_equal(xt, x.astype(np.float64))


def test_mxf4_tile_two_mmas_per_scale_column(umma_lib, cuda):
    """Scales of MMAs 2j and 2j+1 packed into one tensor-memory column and told
    apart by the instruction's scale-factor ids give the same bits as one
    column group per MMA."""
    K, T = 1024, 12
    rng = np.random.default_rng(7)
    w = rng.integers(0, 256, size=(128, K // 2), dtype=np.uint8)
    ws = rng.integers(118, 128, size=(128, K // 32), dtype=np.uint8)
    xb = bf16_vector(rng, K)
    y0, t0, s0 = run(umma_lib, cuda, 0, w, ws, xb, K, T)
    y2, t2, s2 = run(umma_lib, cuda, 2, w, ws, xb, K, T)
    np.testing.assert_array_equal(t2, t0)
    np.testing.assert_array_equal(s2, s0)
    np.testing.assert_array_equal(y2.view(np.uint32), y0.view(np.uint32))


@pytest.mark.parametrize("K", [64, 1536, 4096])
def test_bf16_tile(umma_lib, cuda, K):
    rng = np.random.default_rng(K)
    wb = mo.f32_to_bf16_bits((rng.standard_normal((128, K)) * 0.02).astype(np.float32))
    xb = bf16_vector(rng, K)
    y, _, _ = run(umma_lib, cuda, 1, wb.view(np.uint8).reshape(128, 2 * K), None, xb, K, 0)
    W = mo.bf16_bits_to_f32(wb).astype(np.float64)
    x = mo.bf16_bits_to_f32(xb).astype(np.float64)
    ref = W @ x
    bound = 4e-6 * (np.abs(W) @ np.abs(x)) + 1e-30
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))
