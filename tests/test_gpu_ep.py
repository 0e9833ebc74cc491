"""Expert parallelism on two GPUs (NCCL) against the single-GPU block.

Runs tests/ep_gpu_worker.py under torchrun with two ranks; skipped on a
one-GPU machine.  The host logic is covered on CPU ranks by
tests/test_ep_exchange.py.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_expert_parallel_two_ranks_match_single_gpu(cuda, native_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(
        ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
         "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517",
         str(ROOT / "tests" / "ep_gpu_worker.py")],
        cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert r.stdout.count(" ok") == 10, r.stdout[-2000:]
