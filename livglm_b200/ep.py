"""Expert-parallel MoE block: routed experts sharded over ranks, NCCL exchange.

No counterpart in the reference (its experts stream from SSD on one device);
this is the multi-GPU form of ExpertSSDMoE.__call__ (moe.py:96-201) for
batched work.  Rank r of a W-rank process group holds the routed experts
r, r + W, r + 2W, ... and a replica of the router and the shared expert; tokens
are data-parallel (each rank brings its own rows).  One call:

1. route the local rows (lg_moe_router), renumber the chosen experts to
   exchange ids (expert e lives on rank e mod W, as local expert e // W;
   exchange id = owner * E/W + local index) and sort the route slots t*k + j
   by exchange id (lg_moe_dispatch, a stable counting sort): that order groups
   the slots by destination rank and, within it, by local expert;
2. exchange the per-destination route counts (all-to-all of W integers; the
   split sizes go to the host once per call);
3. send one bf16 row per route slot and its expert id local to the
   destination by all-to-all, and run the local tokens' shared expert while
   the exchange is in flight;
4. run the received rows through the local experts (lg_moe_experts with
   top-k 1 over the E/W local experts);
5. send the bf16 outputs back by the reverse all-to-all and merge them, read
   through the inverse of the dispatch permutation, with the local shared
   expert (lg_moe_combine_gather).

The send buffers of step 3 (rows in destination order, local expert ids, the
inverse permutation) come from one kernel, lg_moe_ep_pack.

The per-route arithmetic is the single-GPU kernels' own, so the result equals
ExpertSSDMoE on the same rows up to the batched kernels' rounding order.
Collectives run on the caller's process group (NCCL for CUDA tensors).

The same layer is one C call in liblivglm_moe_ep.so (lg_moe_ep_forward,
include/livglm_moe_ep.h): give ExpertParallelMoE an EpCommunicator and it
runs that call instead of the steps above (same kernels, same order, its own
NCCL communicator and exchange stream).
"""

from __future__ import annotations

import ctypes
from dataclasses import replace
from typing import Callable

import torch
import torch.distributed as dist

from . import _native
from .config import ContractError, MoEConfig
from .moe import (DenseMLP, ResidentExperts, TopKRouter, Workspace, _rows_bf16, _stream_ptr,
                  require_weight)

LocalCompute = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def expert_owner(expert: torch.Tensor, n_experts: int, world: int) -> torch.Tensor:
    """Rank that holds each expert id: round-robin, expert e on rank e mod W
    (popular experts -- low ids under the Zipf workload -- spread over the
    ranks instead of piling onto rank 0)."""
    return torch.remainder(expert, world)


def exchange_ids(n_experts: int, world: int, device=None) -> torch.Tensor:
    """Expert id -> exchange id (int32 [E]): owner * (E/W) + local index, so
    that sorting routes by exchange id groups them by owning rank, and the
    exchange id mod E/W is the expert's index in its owner's bank (expert e is
    local expert e // W of rank e mod W)."""
    e = torch.arange(n_experts, dtype=torch.int64, device=device)
    return ((e % world) * (n_experts // world) + e // world).to(torch.int32)


def exchange_rows(x_send: torch.Tensor, e_send: torch.Tensor, send_counts: torch.Tensor,
                  compute_local: LocalCompute, group=None,
                  overlap: Callable[[], None] | None = None) -> torch.Tensor:
    """Steps 2-5 above on packed send buffers: ship route rows to the experts'
    owners, run them there, ship the outputs back.

    x_send [N, d] route rows grouped by destination rank (rank order);
    e_send [N] int32 expert id local to the destination; send_counts [W]
    int64 rows bound for each rank.  compute_local(x [n, d], local_expert
    [n] int32) -> [n, d] runs on the received rows.  overlap(), if given, runs
    after the dispatch exchange is issued and before it is waited for (the
    shared expert overlaps the transfer that way).  Returns [N, d]: the
    output of every sent row, in send order.

    One all-to-all of W counts (whose values reach the host once: NCCL's
    variable-size exchange takes host split sizes), one of the rows and one of
    their expert ids (both issued before overlap() runs), and one of the
    outputs.
    """
    d = x_send.shape[1]
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.stack([send_counts, recv_counts]).cpu()  # the split sizes, one host copy
    send_split, recv_split = counts[0].tolist(), counts[1].tolist()
    n_send, n_recv = sum(send_split), sum(recv_split)
    if n_send != x_send.shape[0] or e_send.shape[0] != n_send:
        raise ContractError("route counts do not cover every route slot")
    x_recv = x_send.new_empty((n_recv, d))
    e_recv = torch.empty(n_recv, dtype=torch.int32, device=x_send.device)
    w_x = dist.all_to_all_single(x_recv, x_send, recv_split, send_split, group=group, async_op=True)
    w_e = dist.all_to_all_single(e_recv, e_send, recv_split, send_split, group=group, async_op=True)
    if overlap is not None:
        overlap()
    w_x.wait()
    w_e.wait()
    if n_recv:
        y_recv = compute_local(x_recv, e_recv).reshape(n_recv, d).to(x_send.dtype)
    else:
        y_recv = x_send.new_empty((0, d))
    y_back = x_send.new_empty((n_send, d))
    dist.all_to_all_single(y_back, y_recv.contiguous(), send_split, recv_split, group=group)
    return y_back


def exchange_routes(rows: torch.Tensor, slot_expert: torch.Tensor, perm: torch.Tensor,
                    send_counts: torch.Tensor, n_experts: int, compute_local: LocalCompute,
                    group=None, overlap: Callable[[], None] | None = None) -> torch.Tensor:
    """exchange_rows with the packing done by torch ops (any device): rows
    [M, d] one per token, slot_expert [M*k] int64 exchange id of each route
    slot (exchange_ids), perm [M*k] int64 route slots sorted by it (stable),
    send_counts [W] int64.  Returns [M*k, d], the output of every route slot
    in slot order.  ExpertParallelMoE does the same packing and unpacking
    with lg_moe_ep_pack and lg_moe_combine_gather."""
    world = dist.get_world_size(group)
    per_rank = n_experts // world
    k = slot_expert.numel() // max(1, rows.shape[0])
    token = torch.div(perm, max(1, k), rounding_mode="floor")
    x_send = rows.index_select(0, token)
    e_send = (slot_expert.index_select(0, perm) % per_rank).to(torch.int32)
    y_back = exchange_rows(x_send, e_send, send_counts, compute_local, group, overlap)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), dtype=perm.dtype, device=perm.device)
    return y_back.index_select(0, inv)


class EpCommunicator:
    """The C library's NCCL communicator over the ranks of a torch.distributed
    group (lg_ep_comm_init): rank 0 makes the id, the group broadcasts it.
    max_tokens bounds the rows any rank passes to one layer call.  Call on the
    device the layers run on (torch.cuda.set_device first)."""

    def __init__(self, max_tokens: int, group=None):
        if not dist.is_initialized():
            raise ContractError("EpCommunicator needs an initialised torch.distributed group")
        lib = _native.load_ep()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens = int(max_tokens)
        n = lib.lg_ep_unique_id_bytes()
        uid = (ctypes.c_uint8 * n)()
        if self.rank == 0:
            _native.ep_check(lib.lg_ep_get_unique_id(uid), "lg_ep_get_unique_id")
        box = [bytes(uid)]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(box, src=src, group=group)
        ctypes.memmove(uid, box[0], n)
        handle = ctypes.c_void_p()
        _native.ep_check(lib.lg_ep_comm_init(uid, self.world, self.rank, self.max_tokens, ctypes.byref(handle)),
                         "lg_ep_comm_init")
        self.handle = handle
        self._ws: torch.Tensor | None = None

    def workspace(self, cfg: _native.LgConfig, device) -> torch.Tensor:
        """Scratch of lg_moe_ep_forward, shared by every layer that uses this
        communicator (their calls are ordered on one stream), grown to the
        largest geometry asked for.  Zero-filled: the status word starts at 0."""
        need = _native.load_ep().lg_moe_ep_workspace_size(cfg, self.max_tokens, self.world)
        if need == 0:
            _native.ep_check(_native.LG_ERR_INVALID_ARG, "lg_moe_ep_workspace_size")
        if self._ws is None or self._ws.numel() < need or self._ws.device != torch.device(device):
            self._ws = torch.zeros(need, dtype=torch.uint8, device=device)
        return self._ws

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            _native.load_ep().lg_ep_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertParallelMoE:
    """ExpertSSDMoE with its routed experts sharded over a process group.

    tensors: the layer's stacked tensors as built by synthetic.layer_weights
    (router_weight, router_bias, shared_*, and either the full expert banks,
    of which this rank keeps experts rank, rank + W, ..., or banks already
    holding only the E/W local experts in that order).

    comm: an EpCommunicator over the same group runs the layer as one C call
    (lg_moe_ep_forward); without one the steps run from Python over
    torch.distributed.
    """

    def __init__(self, config: MoEConfig, layer_idx: int, tensors: dict, *, group=None,
                 comm: EpCommunicator | None = None):
        if not dist.is_initialized():
            raise ContractError("expert parallelism needs an initialised torch.distributed group")
        self.config = config
        self.layer_idx = layer_idx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E = config.n_routed_experts
        if E % self.world:
            raise ContractError(f"{E} routed experts do not split evenly over {self.world} ranks")
        self.per_rank = E // self.world
        self.gate = TopKRouter(config)
        self.gate.weight = require_weight(tensors.get("router_weight"), "router.weight")
        self.gate.e_score_correction_bias = require_weight(tensors.get("router_bias"),
                                                           "router.e_score_correction_bias")
        self.shared_experts = DenseMLP(config.hidden_size, config.shared_intermediate_size,
                                       config.swiglu_limit, config)
        if config.n_shared_experts > 0:
            self.shared_experts.gate_proj.weight = tensors["shared_gate"]
            self.shared_experts.up_proj.weight = tensors["shared_up"]
            self.shared_experts.down_proj.weight = tensors["shared_down"]
        # local experts: top-1 over E/W experts, no routing or shared part of their own
        self.local_config = replace(config, n_routed_experts=self.per_rank, num_experts_per_tok=1,
                                    n_group=1, topk_group=1, n_shared_experts=0)
        self.experts = ResidentExperts(self.local_config, layer=layer_idx)
        banks = []
        for name in ("gate_packed", "gate_scale", "up_packed", "up_scale", "down_packed", "down_scale"):
            t = tensors[name]
            if t.shape[0] == E:
                t = t[self.rank::self.world]
            if t.shape[0] != self.per_rank:
                raise ContractError(f"{name} holds {t.shape[0]} experts, expected {E} or {self.per_rank}")
            banks.append(t.contiguous())
        self.experts.set_banks(*banks)
        self._cfg = _native.LgConfig.from_config(config)
        self._ws = Workspace()
        self._xid = exchange_ids(E, self.world, self.gate.weight.device)
        self.comm = comm
        if comm is not None and comm.world != self.world:
            raise ContractError("communicator and process group differ in size")
        self._ep_ws: torch.Tensor | None = None
        self._native_w: _native.LgWeights | None = None
        self._native_key: tuple = ()

    def _native_weights(self) -> _native.LgWeights:
        """The C call's weight table, rebuilt whenever a bound tensor changed
        (the expert banks' own table, the router, the shared expert)."""
        local = self.experts.native_weights()
        tensors = [require_weight(self.gate.weight, "router.weight"),
                   require_weight(self.gate.e_score_correction_bias, "router.e_score_correction_bias")]
        if self.config.n_shared_experts > 0:
            tensors += [self.shared_experts.gate_proj.weight, self.shared_experts.up_proj.weight,
                        self.shared_experts.down_proj.weight]
        key = (id(local),) + tuple(t.data_ptr() if t is not None else 0 for t in tensors)
        if self._native_w is None or self._native_key != key:
            w = _native.LgWeights()
            for name, _ in _native.LgWeights._fields_:
                setattr(w, name, getattr(local, name))
            w.router_weight = tensors[0].data_ptr()
            w.router_bias = tensors[1].data_ptr()
            if self.config.n_shared_experts > 0:
                self.shared_experts.native_into(w)
            self._native_w, self._native_key, self._native_refs = w, key, (local, tensors)
        return self._native_w

    def _forward_native(self, rows: torch.Tensor):
        """lg_moe_ep_forward: the whole layer in one C call."""
        c, comm = self.config, self.comm
        M, dev, k, d = rows.shape[0], rows.device, c.num_experts_per_tok, c.hidden_size
        lib = _native.load_ep()
        self._ep_ws = comm.workspace(self._cfg, dev)
        out = torch.empty(M, d, dtype=torch.float32, device=dev)
        weights = torch.empty(M, k, dtype=torch.float32, device=dev)
        indices = torch.empty(M, k, dtype=torch.uint32, device=dev)
        _native.ep_check(lib.lg_moe_ep_forward(comm.handle, self._cfg, self._native_weights(), rows.data_ptr(), M,
                                               out.data_ptr(), weights.data_ptr(), indices.data_ptr(),
                                               self._ep_ws.data_ptr(), self._ep_ws.numel(), _stream_ptr(dev)),
                         "lg_moe_ep_forward")
        return out, weights, indices

    def status(self) -> int:
        """Device status word of the C call's workspace (0 = ok)."""
        if self._ep_ws is None:
            return self._ws.status()
        return int(self._ep_ws[:4].view(torch.int32).item())

    def use_workspace(self, ws: Workspace) -> None:
        """Share one scratch area with other layers run in order on one stream
        (this layer's router, local experts, shared expert and dispatch all
        use it, one call after another)."""
        self._ws = ws
        for part in (self.gate, self.experts, self.shared_experts):
            if hasattr(part, "_ws"):
                part._ws = ws

    def _local(self, x: torch.Tensor, local_expert: torch.Tensor) -> torch.Tensor:
        idx = local_expert.to(torch.int32).view(torch.uint32).reshape(-1, 1)
        return self.experts(x, idx).reshape(x.shape[0], self.config.hidden_size)

    def __call__(self, hidden_states: torch.Tensor, *, return_route: bool = False):
        """Local bf16 rows [..., d] -> f32 [..., d], as ExpertSSDMoE.__call__."""
        c = self.config
        rows = _rows_bf16(hidden_states, c.hidden_size)
        if self.comm is not None:
            out, weights, indices = self._forward_native(rows)
            result = out.reshape(*hidden_states.shape[:-1], c.hidden_size)
            return (result, weights, indices) if return_route else result
        M, dev, k, E, d = rows.shape[0], rows.device, c.num_experts_per_tok, c.n_routed_experts, c.hidden_size
        lib = _native.load()
        stream = _stream_ptr(dev)
        R = M * k
        x_send = torch.empty(R, d, dtype=torch.bfloat16, device=dev)
        e_send = torch.empty(R, dtype=torch.int32, device=dev)
        inv = torch.empty(R, dtype=torch.int32, device=dev)
        if M:
            _, weights, indices = self.gate(rows)
            xidx = self._xid[indices.view(torch.int32).long()].view(torch.uint32)  # exchange ids
            counts = torch.empty(E, dtype=torch.int32, device=dev)
            offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
            perm = torch.empty(R, dtype=torch.int32, device=dev)
            ws, nbytes = self._ws.get(self._cfg, M, dev)
            _native.check(lib.lg_moe_dispatch(self._cfg, xidx.data_ptr(), M, counts.data_ptr(),
                                              offsets.data_ptr(), perm.data_ptr(), ws, nbytes, stream),
                          "lg_moe_dispatch")
            _native.check(lib.lg_moe_ep_pack(self._cfg, rows.data_ptr(), M, xidx.data_ptr(), perm.data_ptr(),
                                             self.world, x_send.data_ptr(), e_send.data_ptr(), inv.data_ptr(),
                                             stream), "lg_moe_ep_pack")
            bounds = offsets[::self.per_rank].to(torch.int64)  # [W + 1] dispatch ranges per owner
            send_counts = bounds[1:] - bounds[:-1]
        else:
            weights = torch.empty(0, k, dtype=torch.float32, device=dev)
            indices = torch.empty(0, k, dtype=torch.uint32, device=dev)
            send_counts = torch.zeros(self.world, dtype=torch.int64, device=dev)
        shared = None

        def run_shared() -> None:  # overlaps the dispatch exchange
            nonlocal shared
            if M and c.n_shared_experts > 0:
                shared = self.shared_experts(rows)

        y_disp = exchange_rows(x_send, e_send, send_counts, self._local, self.group, overlap=run_shared)
        out = torch.empty(M, d, dtype=torch.float32, device=dev)
        if M:
            _native.check(lib.lg_moe_combine_gather(self._cfg, y_disp.data_ptr(), inv.data_ptr(), weights.data_ptr(),
                                                    shared.data_ptr() if shared is not None else None, M,
                                                    out.data_ptr(), stream), "lg_moe_combine_gather")
        result = out.reshape(*hidden_states.shape[:-1], d)
        if return_route:
            return result, weights, indices
        return result
