"""The frozen config-1 records (tests/golden/cfg1.npz, made by
tests/golden/make_golden_cfg1.py) against the oracles on the CPU.

The layer's weights are redrawn from their seeds (a few seconds); the
canonical router must reproduce the stored routing bit-for-bit, the NumPy
oracle the stored M = 1 output exactly, and the C restatement (the timed CPU
baseline) every stored output within the parity bar.
"""

import numpy as np
import pytest

from livglm_b200.config import CONFIGS
from oracle import moe_oracle as mo
from tests.golden import make_golden_cfg1 as g1
from tests.helpers import assert_close


@pytest.fixture(scope="module")
def cfg1_records():
    cfg = CONFIGS["cfg1"]
    with np.load(g1.OUT) as z:
        rec = {k: z[k] for k in z.files}
    return cfg, g1.weights(cfg), rec


def test_cfg1_records_routing_reproduced(cfg1_records):
    cfg, bank, rec = cfg1_records
    for M in (1, 2, 256):
        np.testing.assert_array_equal(rec[f"x{M}"], g1.tokens(cfg, M))
        _, w, idx = mo.router(rec[f"x{M}"], bank["router_weight"], bank["router_bias"], cfg)
        np.testing.assert_array_equal(idx, rec[f"indices{M}"])
        np.testing.assert_array_equal(w.view(np.uint32), rec[f"weights{M}"].view(np.uint32))


def test_cfg1_record_m1_reproduced_by_numpy_oracle(cfg1_records):
    cfg, bank, rec = cfg1_records
    np.testing.assert_array_equal(mo.moe_forward(rec["x1"], bank, cfg)["out"], rec["out1"])


@pytest.mark.parametrize("M", [1, 2, 256])
def test_cfg1_records_c_restatement(cfg1_records, M):
    cfg, bank, rec = cfg1_records
    sel = rec[f"sel{M}"]
    got = mo.moe_forward_c(rec[f"x{M}"][sel], bank, cfg)
    np.testing.assert_array_equal(got["indices"], rec[f"indices{M}"][sel])
    assert_close(got["out"], rec[f"out{M}"])
