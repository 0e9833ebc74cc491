import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_cfg0():
    with np.load(GOLDEN / "cfg0.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def native_lib():
    """The in-tree CUDA library, built here if stale (nvcc cross-compiles)."""
    from livglm_b200 import _native, build

    if not _native.LIB_PATH.exists():
        build.build()
    return _native.load()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
