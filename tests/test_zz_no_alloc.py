"""lg_moe_forward_static_scratch: the MoE forward for callers that cannot
allocate device memory at call time (a framework that owns all device memory
and gives plugins no allocator, a decode loop where cudaMalloc could
synchronise the device, code holding a lock the allocator also takes).

Its scratch is a fixed 4 MiB device array inside the library, so the call
itself allocates nothing.  This test calls it through the C ABI twice in a row
and checks both results against lg_moe_forward with a caller workspace, using
the parity tolerance of the other tests; it also checks that a token count
whose scratch would exceed the fixed size is refused with a clear error.

The file name sorts last so a run that stops at the first failure has already
run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from livglm_b200 import _native, synthetic
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from tests.helpers import assert_close, to_numpy

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 4 << 20


def _forward_with_workspace(lib, c, w, x, M, dev):
    out = torch.empty(M, x.shape[1], dtype=torch.float32, device=dev)
    wts = torch.empty(M, c.num_experts_per_tok, dtype=torch.float32, device=dev)
    idx = torch.empty(M, c.num_experts_per_tok, dtype=torch.uint32, device=dev)
    ws = torch.zeros(lib.lg_moe_workspace_size(c, M), dtype=torch.uint8, device=dev)
    rc = lib.lg_moe_forward(c, ctypes.byref(w), x.data_ptr(), M, out.data_ptr(), wts.data_ptr(),
                            idx.data_ptr(), ws.data_ptr(), ws.numel(),
                            torch.cuda.current_stream(dev).cuda_stream)
    _native.check(rc, "lg_moe_forward")
    return out, wts, idx


def _forward_static(lib, c, w, x, M, dev):
    out = torch.full((M, x.shape[1]), float("nan"), dtype=torch.float32, device=dev)
    wts = torch.empty(M, c.num_experts_per_tok, dtype=torch.float32, device=dev)
    idx = torch.empty(M, c.num_experts_per_tok, dtype=torch.uint32, device=dev)
    rc = lib.lg_moe_forward_static_scratch(c, ctypes.byref(w), x.data_ptr(), M, out.data_ptr(),
                                           wts.data_ptr(), idx.data_ptr(),
                                           torch.cuda.current_stream(dev).cuda_stream)
    _native.check(rc, "lg_moe_forward_static_scratch")
    return out, wts, idx


@pytest.mark.parametrize("M", [1, 2, 33])
def test_static_scratch_forward_matches_workspace_forward(cuda, native_lib, M):
    cfg = CONFIGS["cfg1"]
    lib = native_lib
    c = _native.LgConfig.from_config(cfg)
    assert lib.lg_moe_workspace_size(c, M) <= STATIC_SCRATCH_BYTES
    moe = build_layer(cfg, synthetic.layer_weights(cfg, seed=7, device=cuda))
    w = moe.native_weights()
    x = synthetic.hidden_states(cfg, M, seed=11 + M, device=cuda)
    ref_out, ref_w, ref_idx = _forward_with_workspace(lib, c, w, x, M, cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    st = ctypes.c_int32(-1)
    _native.check(lib.lg_moe_static_scratch_status(1, ctypes.byref(st), stream), "status")  # start clean
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch
        out, wts, idx = _forward_static(lib, c, w, x, M, cuda)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(to_numpy(idx), to_numpy(ref_idx))
        np.testing.assert_array_equal(to_numpy(wts), to_numpy(ref_w))
        assert_close(to_numpy(out), to_numpy(ref_out))
        # the status word inside the fixed array: no device-side failure
        st.value = -1
        _native.check(lib.lg_moe_static_scratch_status(0, ctypes.byref(st), stream), "status")
        assert st.value == 0


def test_static_scratch_rejects_too_many_tokens(native_lib):
    cfg = CONFIGS["cfg1"]
    lib = native_lib
    c = _native.LgConfig.from_config(cfg)
    M = 64
    assert lib.lg_moe_workspace_size(c, M) > STATIC_SCRATCH_BYTES
    w = _native.LgWeights()
    rc = lib.lg_moe_forward_static_scratch(c, ctypes.byref(w), None, M, None, None, None, None)
    assert rc == _native.LG_ERR_UNSUPPORTED
    assert "more than the fixed" in _native.last_error()
