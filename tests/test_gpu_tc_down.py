"""The CUDA-core one-token down kernel (LIVGLM_TC_DOWN=0) against the oracle.

One-token calls use the tensor-core down kernel (livglm_b200/csrc/down_tc.cuh)
by default, which test_gpu_parity.py covers.  The library reads the switch
once per process, so the one-token parity tests run again in a child pytest
with the switch off: every M = 1 call then takes down1_stream_kernel, the
fallback for geometries the tensor-core plan does not cover.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

ONE_TOKEN_TESTS = " or ".join([
    "test_forward_cfg1_decode",
    "test_forward_deterministic_and_shape_preserving",
    "test_forward_host_tokens_and_output",
    "test_rebinding_weights_after_a_call",
])


def test_one_token_parity_through_cuda_core_down(cuda, native_lib):
    env = dict(os.environ, LIVGLM_TC_DOWN="0")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
         str(ROOT / "tests" / "test_gpu_parity.py"), "-k", ONE_TOKEN_TESTS],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
