"""One rank of the expert-parallel GPU check (launched by tests/test_gpu_ep.py).

Every rank builds the same seeded layer, keeps its E/W routed experts, runs
its own rows through ExpertParallelMoE over NCCL and compares with the
single-GPU ExpertSSDMoE on the same rows (full weights on this GPU): routing
bit-exact, outputs within the parity bar, and a few rows against the CPU
checker.  The same layer through the C call lg_moe_ep_forward (an
EpCommunicator) must give bit-identical routing and output; a rank with no
rows and a rank whose row count exceeds the communicator's bound (every rank
then gets the error, and the communicator stays usable) are checked too.
Exit status 0 on success.
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
from livglm_b200.config import ContractError  # noqa: E402
from livglm_b200.ep import EpCommunicator, ExpertParallelMoE  # noqa: E402
from livglm_b200.moe import build_layer  # noqa: E402
from oracle import moe_oracle as mo  # noqa: E402
from tests.helpers import assert_close, bank_to_numpy, to_numpy  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    comm = EpCommunicator(max_tokens=64)
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
            native = ExpertParallelMoE(cfg, 0, t, comm=comm)
            n_out, n_w, n_idx = native(x, return_route=True)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(to_numpy(n_idx), to_numpy(idx))
            np.testing.assert_array_equal(to_numpy(n_w).view(np.uint32), to_numpy(w).view(np.uint32))
            np.testing.assert_array_equal(to_numpy(n_out).view(np.uint32), to_numpy(out).view(np.uint32))
            assert native.status() == 0
            print(f"rank {rank}: {name} M={M} native ok", flush=True)
            del ep, t
        # rank 1 brings no rows; then rank 1 brings too many (every rank fails
        # the same call); then a normal call on the same communicator
        cfg = CONFIGS["cfg0"]
        t = synthetic.layer_weights(cfg, seed=7, device=dev)
        native = ExpertParallelMoE(cfg, 0, t, comm=comm)
        single = build_layer(cfg, t)
        for M_rank1, expect_error in ((0, False), (65, True), (3, False)):
            M = 6 if rank == 0 else M_rank1
            x = synthetic.hidden_states(cfg, M, seed=300 + rank, device=dev)
            try:
                got = native(x)
                err = None
            except ContractError as exc:
                got, err = None, str(exc)
            if expect_error:
                assert err is not None and ("M=65" in err or "rank 1" in err), err
            else:
                assert err is None, err
                torch.cuda.synchronize()
                if M:
                    assert_close(to_numpy(got), to_numpy(single(x)))
                else:
                    assert got.shape == (0, cfg.hidden_size)
        print(f"rank {rank}: edge cases ok", flush=True)
        dist.barrier()
    finally:
        comm.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
