"""Host logic of the expert-parallel exchange (livglm_b200/ep.py) on CPU ranks.

Two gloo ranks route their own rows of the cfg0 golden batch with the CPU
checker, ship every route slot to the rank that owns its expert, run the
received rows through the checker's expert arithmetic there (standing in for
the CUDA experts), and ship the outputs back.  Each rank's per-slot outputs
must equal the checker's single-process expert outputs for its rows exactly,
for even, uneven and empty token shares.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from livglm_b200.config import CONFIGS
from livglm_b200.ep import exchange_ids, exchange_routes, expert_owner
from oracle import moe_oracle as mo
from tests.conftest import GOLDEN


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, shares: list, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = CONFIGS["cfg0"]
        with np.load(GOLDEN / "cfg0.npz") as z:
            bank = {key: z[key] for key in z.files}
        E, k, d = cfg.n_routed_experts, cfg.num_experts_per_tok, cfg.hidden_size
        lo = sum(shares[:rank])
        x_bits = bank["x"][lo:lo + shares[rank]]
        M = x_bits.shape[0]
        if M:
            _, _, idx = mo.router(x_bits, bank["router_weight"], bank["router_bias"], cfg)
        else:
            idx = np.zeros((0, k), np.uint32)
        slot_expert = torch.from_numpy(idx.reshape(-1).astype(np.int64))
        slot_xid = exchange_ids(E, world)[slot_expert].to(torch.int64)
        perm = torch.from_numpy(np.argsort(slot_xid.numpy(), kind="stable").astype(np.int64))
        owner = expert_owner(slot_expert, E, world)
        send_counts = torch.bincount(owner, minlength=world).to(torch.int64)
        rows = torch.from_numpy(mo.bf16_bits_to_f32(x_bits.astype(np.uint16)).reshape(M, d))
        cfg1 = cfg.replace(num_experts_per_tok=1)

        def compute_local(x: torch.Tensor, local_expert: torch.Tensor) -> torch.Tensor:
            bits = mo.f32_to_bf16_bits(x.numpy())
            glob = (local_expert.numpy() * world + rank).astype(np.uint32).reshape(-1, 1)
            y = mo.expert_outputs(bits, bank, glob, cfg1)
            return torch.from_numpy(y.reshape(-1, d))

        y_slots = exchange_routes(rows, slot_xid, perm, send_counts, E, compute_local)
        ref = mo.expert_outputs(x_bits, bank, idx, cfg).reshape(-1, d) if M else np.zeros((0, d), np.float32)
        result_q.put((rank, bool(np.array_equal(y_slots.numpy(), ref)), int(M)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shares", [[4, 4], [3, 5], [0, 8]])
def test_exchange_matches_single_process_experts(shares):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shares, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    assert codes == [0, 0], codes
    got = sorted(q.get() for _ in range(2))
    assert [g[1] for g in got] == [True, True], got
    assert [g[2] for g in got] == shares


def test_expert_owner_ranges():
    e = torch.arange(16)
    assert expert_owner(e, 16, 4).tolist() == [0, 1, 2, 3] * 4
    xid = exchange_ids(16, 4)
    # sorted by exchange id = grouped by owner, then by local index e // W
    assert torch.argsort(xid).tolist() == [0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15]
    assert (xid // 4).tolist() == expert_owner(e, 16, 4).tolist()
    assert (xid % 4).tolist() == (e // 4).tolist()
