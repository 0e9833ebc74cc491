"""The fused one-kernel decode layer (LIVGLM_FUSED_LAYER=1) against the oracle.

The library reads the switch once per process, so the decode-shaped parity
tests of test_gpu_parity.py run again in a child pytest with the switch on:
every M <= 4 call there then goes through the fused cooperative kernel
instead of the chain of stream kernels (the allocation-free entry point's
check included: its fixed scratch is shared by calls of different token
counts, whose grid counters must line up).
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

DECODE_TESTS = " or ".join([
    "test_forward_cfg1_decode",
    "test_forward_deterministic_and_shape_preserving",
    "test_forward_other_geometries",
    "test_forward_cfg0_small_batches",
    "test_forward_large_activations",
    "test_golden_cfg0_forward",
    "test_checkpoint_names_drop_in",
    "test_static_scratch_forward_matches_workspace_forward",
    "test_forward_host_tokens_and_output",
])


def test_decode_parity_through_fused_layer(cuda, native_lib):
    env = dict(os.environ, LIVGLM_FUSED_LAYER="1")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
         str(ROOT / "tests" / "test_gpu_parity.py"), str(ROOT / "tests" / "test_zz_no_alloc.py"),
         "-k", DECODE_TESTS],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
