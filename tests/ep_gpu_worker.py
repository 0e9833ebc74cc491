"""One rank of the expert-parallel GPU check (launched by tests/test_gpu_ep.py).

Every rank builds the same seeded layer, keeps its E/W routed experts, runs
its own rows through ExpertParallelMoE over NCCL and compares with the
single-GPU ExpertSSDMoE on the same rows (full weights on this GPU): routing
bit-exact, outputs within the parity bar, and a few rows against the CPU
checker.  Exit status 0 on success.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from livglm_b200 import synthetic  # noqa: E402
from livglm_b200.config import CONFIGS  # noqa: E402
from livglm_b200.ep import ExpertParallelMoE  # noqa: E402
from livglm_b200.moe import build_layer  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402
from tests.helpers import assert_close, bank_to_numpy, to_numpy  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        for name, per_rank_rows in (("cfg0", [8, 5]), ("cfg1", [64, 40])):
            cfg = CONFIGS[name]
            t = synthetic.layer_weights(cfg, seed=7, device=dev)
            M = per_rank_rows[rank % len(per_rank_rows)]
            x = synthetic.hidden_states(cfg, M, seed=100 + rank, device=dev)
            ep = ExpertParallelMoE(cfg, 0, t)
            out, w, idx = ep(x, return_route=True)
            ref_out, ref_w, ref_idx = build_layer(cfg, t)(x, return_route=True)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(to_numpy(idx), to_numpy(ref_idx))
            np.testing.assert_array_equal(to_numpy(w).view(np.uint32), to_numpy(ref_w).view(np.uint32))
            assert_close(to_numpy(out), to_numpy(ref_out))
            tn = bank_to_numpy(t)
            sample = np.arange(min(M, 4))
            ref = mo.moe_forward(to_numpy(x), tn, cfg, tokens=sample)
            assert_close(to_numpy(out)[sample], ref["out"])
            print(f"rank {rank}: {name} M={M} ok", flush=True)
            del ep, t
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
