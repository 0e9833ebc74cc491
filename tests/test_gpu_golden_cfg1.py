"""The GPU block against the frozen config-1 records (tests/golden/cfg1.npz):
M = 1 and M = 2 run the decode chain, M = 256 the batched tensor-core path.
Routing bit-for-bit, outputs within the parity bar of the stored oracle
outputs (all tokens for M = 1, 2; the stored sample of 16 for M = 256)."""

import numpy as np
import pytest
import torch

from livglm_b200.config import CONFIGS
from livglm_b200.moe import build_layer
from tests.golden import make_golden_cfg1 as g1
from tests.helpers import assert_close, to_numpy

pytestmark = pytest.mark.gpu


def _torch_bank(bank: dict, device) -> dict:
    t = {}
    for k, v in bank.items():
        if k.startswith("shared_"):
            t[k] = torch.from_numpy(v.view(np.int16)).to(device).view(torch.bfloat16)
        else:
            t[k] = torch.from_numpy(v).to(device)
    return t


@pytest.fixture(scope="module")
def layer_and_records(cuda, native_lib):
    cfg = CONFIGS["cfg1"]
    with np.load(g1.OUT) as z:
        rec = {k: z[k] for k in z.files}
    return cfg, build_layer(cfg, _torch_bank(g1.weights(cfg), cuda)), rec


@pytest.mark.parametrize("M", [1, 2, 256])
def test_gpu_matches_cfg1_record(cuda, layer_and_records, M):
    cfg, moe, rec = layer_and_records
    x = torch.from_numpy(rec[f"x{M}"].view(np.int16)).to(cuda).view(torch.bfloat16)
    out, w, idx = moe(x, return_route=True)
    torch.cuda.synchronize()
    assert moe.device_status() == 0
    np.testing.assert_array_equal(to_numpy(idx), rec[f"indices{M}"])
    np.testing.assert_array_equal(to_numpy(w).view(np.uint32), rec[f"weights{M}"].view(np.uint32))
    assert_close(to_numpy(out)[rec[f"sel{M}"]], rec[f"out{M}"])
