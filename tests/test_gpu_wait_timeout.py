"""Device-side failure reporting without a GPU fault.

Every wait inside the library's kernels is bounded: after a limit it records
LG_ERR_TIMEOUT and the waiting site in a status word and lets the kernel
return.  lg_moe_check_wait_timeout runs those same wait routines, with a
1 ms limit, against an mbarrier that never completes and a flag that nothing
sets; the test checks that each wait gave up with the documented status word
and that the context still runs the MoE block afterwards (config 0 against
the committed oracle record).
"""

import numpy as np
import pytest
import torch

from livglm_b200 import _native
from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from tests.helpers import assert_close, bank_to_device, to_device, to_numpy

pytestmark = pytest.mark.gpu

SITE_BARRIER = 30 << 8
SITE_FLAG = 31 << 8


def test_bounded_waits_give_up_and_report(cuda, native_lib, golden_cfg0):
    status = torch.full((4,), -1, dtype=torch.int32, device=cuda)
    rc = native_lib.lg_moe_check_wait_timeout(1_000_000, status.data_ptr(),
                                              torch.cuda.current_stream(cuda).cuda_stream)
    _native.check(rc, "lg_moe_check_wait_timeout")
    torch.cuda.synchronize()
    words = status.cpu().tolist()
    assert words == [_native.LG_ERR_TIMEOUT | SITE_BARRIER, _native.LG_ERR_TIMEOUT | SITE_BARRIER,
                     _native.LG_ERR_TIMEOUT | SITE_FLAG, 0], words
    # the context is intact: the block still runs and matches the oracle
    g = golden_cfg0
    moe = build_layer(CONFIGS["cfg0"], bank_to_device(g, cuda))
    out, _, idx = moe(to_device(g["x"], cuda, bf16=True), return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_numpy(idx), g["indices"])
    assert_close(to_numpy(out), g["out"])


def test_wait_check_rejects_bad_arguments(native_lib):
    assert native_lib.lg_moe_check_wait_timeout(1_000_000, None, None) == _native.LG_ERR_INVALID_ARG
    assert native_lib.lg_moe_check_wait_timeout(10, 16, None) == _native.LG_ERR_INVALID_ARG
