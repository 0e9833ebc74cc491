"""B200-native drop-in for the GLM MoE block of kg36/livglm.

Same module structure, constructor and call signatures as the reference
(src/glm53flash/moe.py:19-201): ExpertSSDMoE(config, layer_idx,
expert_factory) holds `gate` (TopKRouter), `experts` (the routed-expert
backend built by expert_factory(layer_idx)) and `shared_experts` (DenseMLP);
calling it on bf16 hidden states returns the f32 merge.  Torch tensors only
carry device memory and the current stream; all arithmetic runs in the CUDA
library through the C ABI of include/livglm_moe.h.

Differences from the reference, by design:
* Experts are resident in HBM as banks (all E experts of a layer, stacked,
  byte-identical to the checkpoint records) instead of an SSD-backed slot
  cache; the backend is ResidentExperts, not ExpertSSD/NativeExpertSSD.
* Hidden states must be bf16 (as in the native QMV path,
  native_expert_ssd.py:612-620).  Other dtypes raise ContractError.
"""

from __future__ import annotations

import re
from dataclasses import asdict, dataclass
from typing import Callable, Mapping

import torch

from . import _native
from .config import ContractError, MoEConfig

ROUTED_EXPERT_RE = re.compile(
    r"^model\.language_model\.layers\.(\d+)\.mlp\.experts\.(\d+)\."
    r"(down_proj|gate_proj|up_proj)\.(weight_packed|weight_scale)$"
)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device: torch.device) -> int:
    """Raw handle of the current stream of `device` (an int; no Stream object
    where the torch build offers the raw query)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _rows_bf16(hidden_states: torch.Tensor, hidden: int, *, allow_host: bool = False) -> torch.Tensor:
    """[..., d] bf16 -> contiguous [M, d].  With allow_host, a contiguous
    tensor in page-locked host memory is accepted as it is."""
    if not isinstance(hidden_states, torch.Tensor):
        raise ContractError("hidden states must be a torch tensor")
    if hidden_states.dtype != torch.bfloat16:
        raise ContractError(f"hidden states must be bf16, got {hidden_states.dtype}")
    if hidden_states.shape[-1] != hidden:
        raise ContractError(f"hidden size {hidden_states.shape[-1]} != {hidden}")
    if hidden_states.is_cuda:
        return hidden_states.reshape(-1, hidden).contiguous()
    if not allow_host:
        raise ContractError("hidden states must be on a CUDA device")
    if not hidden_states.is_pinned() or not hidden_states.is_contiguous():
        raise ContractError("host hidden states must be a contiguous tensor in page-locked memory")
    return hidden_states.reshape(-1, hidden)


def _out_f32(out: torch.Tensor, M: int, hidden: int) -> torch.Tensor:
    if (not isinstance(out, torch.Tensor) or out.dtype != torch.float32 or out.numel() != M * hidden
            or not out.is_contiguous() or not (out.is_cuda or out.is_pinned())):
        raise ContractError(f"out must be a contiguous f32 tensor of {M}x{hidden} elements on the "
                            "device or in page-locked host memory")
    return out


class Workspace:
    """Caller-owned scratch for the C ABI, grown outside the hot calls.

    Allocated zero-filled: its first 4 bytes are the library's device status
    word (0 = ok; set when a bounded device wait gives up)."""

    def __init__(self) -> None:
        self.buf: torch.Tensor | None = None
        self._ptr = 0
        self._device: torch.device | None = None
        self._need: dict[tuple[int, int], tuple[_native.LgConfig, int]] = {}

    def get(self, cfg: _native.LgConfig, tokens: int, device: torch.device) -> tuple[int, int]:
        tokens = max(int(tokens), 1)
        hit = self._need.get((id(cfg), tokens))
        if hit is not None and hit[0] is cfg:
            need = hit[1]
        else:
            need = _native.load().lg_moe_workspace_size(cfg, tokens)
            if need == 0:
                _native.check(_native.LG_ERR_INVALID_ARG, "workspace size")
            self._need[(id(cfg), tokens)] = (cfg, need)  # holds cfg, so its id stays unique
        if self.buf is None or self.buf.numel() < need or self._device != device:
            self.buf = torch.zeros(need, dtype=torch.uint8, device=device)
            self._ptr, self._device = self.buf.data_ptr(), device
        return self._ptr, self.buf.numel()

    def status(self) -> int:
        """The device status word (synchronises with the device)."""
        if self.buf is None:
            return 0
        return int(self.buf[:4].view(torch.int32).item())


FP8_BLOCK = 128  # block size of the checkpoint's block-FP8 weights (resident_plan.py:189-205)


def widen_block_fp8(weight: torch.Tensor, scale_inv: torch.Tensor, block: int = FP8_BLOCK) -> torch.Tensor:
    """Block-FP8 weight (float8_e4m3fn [rows, cols]) and its f32 block scales
    ([rows/block, cols/block]) -> bf16 [rows, cols] on the weight's CUDA device
    (lg_fp8_block_dequant; fp8.py:43-78).  Non-finite results are refused, as
    the reference refuses them."""
    if weight.dim() != 2 or weight.dtype != torch.float8_e4m3fn:
        raise ContractError(f"block-FP8 weight must be a 2-D float8_e4m3fn tensor, got {weight.dtype}")
    rows, cols = weight.shape
    if rows % block or cols % block:
        raise ContractError(f"block-FP8 shape must be divisible by {block}: {tuple(weight.shape)}")
    if tuple(scale_inv.shape) != (rows // block, cols // block):
        raise ContractError(f"block-FP8 scale shape mismatch: {tuple(scale_inv.shape)} != "
                            f"{(rows // block, cols // block)}")
    if weight.device.type != "cuda":
        raise ContractError("block-FP8 weights are widened on the GPU: move them to a CUDA device first")
    dev = weight.device
    w = weight.contiguous().view(torch.uint8)
    sc = scale_inv.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty(rows, cols, dtype=torch.bfloat16, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _native.load()
    _native.check(lib.lg_fp8_block_dequant(w.data_ptr(), sc.data_ptr(), rows, cols, block, out.data_ptr(),
                                           bad.data_ptr(), _stream_ptr(dev)), "lg_fp8_block_dequant")
    if int(bad.item()):
        raise ContractError("block-FP8 dequantization produced a non-finite weight")
    return out


def require_weight(value, name: str):
    """layers.py:12-15."""
    if value is None:
        raise ContractError(f"resident parameter was not loaded: {name}")
    return value


class TopKRouter:
    """Sigmoid router with correction bias and group-limited top-k (moe.py:19-63)."""

    def __init__(self, config: MoEConfig):
        self.config = config
        self.top_k = config.num_experts_per_tok
        self.num_experts = config.n_routed_experts
        self.hidden_dim = config.hidden_size
        self.routed_scaling_factor = config.routed_scaling_factor
        self.num_group = config.n_group
        self.topk_group = config.topk_group
        self.norm_topk_prob = config.norm_topk_prob
        self.weight: torch.Tensor | None = None
        self.e_score_correction_bias: torch.Tensor | None = None
        self._cfg = _native.LgConfig.from_config(config)
        self._ws = Workspace()

    def __call__(self, hidden_states: torch.Tensor):
        """-> (logits f32 [M,E], weights f32 [M,k], indices u32 [M,k]); indices
        ascend in choice score, best expert last (moe.py:58)."""
        rows = _rows_bf16(hidden_states, self.hidden_dim)
        w = require_weight(self.weight, "router.weight")
        b = require_weight(self.e_score_correction_bias, "router.e_score_correction_bias")
        M, dev = rows.shape[0], rows.device
        logits = torch.empty(M, self.num_experts, dtype=torch.float32, device=dev)
        weights = torch.empty(M, self.top_k, dtype=torch.float32, device=dev)
        indices = torch.empty(M, self.top_k, dtype=torch.uint32, device=dev)
        ws, nbytes = self._ws.get(self._cfg, M, dev)
        rc = _native.load().lg_moe_router(
            self._cfg, rows.data_ptr(), M, w.data_ptr(), b.data_ptr(), logits.data_ptr(),
            weights.data_ptr(), indices.data_ptr(), ws, nbytes, _stream_ptr(dev))
        _native.check(rc, "lg_moe_router")
        return logits, weights, indices


@dataclass(frozen=True)
class ExpertCacheStats:
    """Field-compatible with expert_ssd.py:16-29.  Everything is resident, so
    there are no misses or evictions; hits count routes served."""

    layer: int
    capacity: int
    resident: int
    hits: int
    misses: int
    evictions: int
    route_sync_seconds: float = 0.0
    slot_plan_seconds: float = 0.0
    policy: str = "hbm-resident"

    def as_dict(self):
        return asdict(self)


class _Projection:
    def __init__(self):
        self.weight_packed: torch.Tensor | None = None  # U8 [E, rows, cols/2]
        self.weight_scale: torch.Tensor | None = None   # U8 [E, rows, cols/32]


class ResidentExperts:
    """All routed experts of one layer resident in HBM.

    Replaces the ExpertSSD backend interface (expert_ssd.py:130-194):
    __call__(x, indices) -> [M, k, d], stats(), capacity, last_expert_ids.
    Banks: gate_proj / up_proj / down_proj each hold weight_packed and
    weight_scale stacked over experts, byte-identical to the checkpoint's
    per-expert U8 tensors.
    """

    def __init__(self, config: MoEConfig, *, layer: int):
        self.config = config
        self.layer = layer
        self.capacity = config.n_routed_experts
        self.swiglu_limit = config.swiglu_limit
        self.gate_proj = _Projection()
        self.up_proj = _Projection()
        self.down_proj = _Projection()
        self._routes = 0
        self._last_indices: torch.Tensor | None = None
        self._cfg = _native.LgConfig.from_config(config)
        self._ws = Workspace()
        self._w: _native.LgWeights | None = None
        self._w_key: tuple = ()
        self._w_refs: tuple = ()

    # -- loading -----------------------------------------------------------
    def set_banks(self, gate_packed, gate_scale, up_packed, up_scale, down_packed, down_scale) -> None:
        c = self.config
        d, F, E = c.hidden_size, c.moe_intermediate_size, c.n_routed_experts
        expect = {
            "gate_packed": (gate_packed, (E, F, d // 2)), "gate_scale": (gate_scale, (E, F, d // 32)),
            "up_packed": (up_packed, (E, F, d // 2)), "up_scale": (up_scale, (E, F, d // 32)),
            "down_packed": (down_packed, (E, d, F // 2)), "down_scale": (down_scale, (E, d, F // 32)),
        }
        for name, (t, shape) in expect.items():
            if t.dtype != torch.uint8:
                raise ContractError(f"native MXFP4 tensor must use U8 storage: {name}")
            if tuple(t.shape) != shape:
                raise ContractError(f"{name} has shape {tuple(t.shape)}, expected {shape}")
            if not t.is_cuda or not t.is_contiguous():
                raise ContractError(f"{name} must be a contiguous CUDA tensor")
        self.gate_proj.weight_packed, self.gate_proj.weight_scale = gate_packed, gate_scale
        self.up_proj.weight_packed, self.up_proj.weight_scale = up_packed, up_scale
        self.down_proj.weight_packed, self.down_proj.weight_scale = down_packed, down_scale
        self._w = None

    def load_checkpoint(self, tensors: Mapping[str, torch.Tensor], device="cuda") -> None:
        """Bind `model.language_model.layers.{L}.mlp.experts.{e}.{proj}.{part}`
        tensors (contract.py:47-50) of this layer into HBM banks."""
        c = self.config
        d, F, E = c.hidden_size, c.moe_intermediate_size, c.n_routed_experts
        shapes = {
            ("gate_proj", "weight_packed"): (F, d // 2), ("gate_proj", "weight_scale"): (F, d // 32),
            ("up_proj", "weight_packed"): (F, d // 2), ("up_proj", "weight_scale"): (F, d // 32),
            ("down_proj", "weight_packed"): (d, F // 2), ("down_proj", "weight_scale"): (d, F // 32),
        }
        banks = {key: torch.empty((E, *shp), dtype=torch.uint8, device=device) for key, shp in shapes.items()}
        seen = set()
        for name, t in tensors.items():
            m = ROUTED_EXPERT_RE.match(name)
            if not m or int(m.group(1)) != self.layer:
                continue
            e, proj, part = int(m.group(2)), m.group(3), m.group(4)
            if not 0 <= e < E:
                raise ContractError(f"routed expert ids are out of range: {e}")
            if t.dtype != torch.uint8 or tuple(t.shape) != shapes[(proj, part)]:
                raise ContractError(f"unexpected expert tensor {name}: {t.dtype} {tuple(t.shape)}")
            banks[(proj, part)][e].copy_(t)
            seen.add((e, proj, part))
        if len(seen) != E * 6:
            raise ContractError(f"layer {self.layer}: {E * 6 - len(seen)} routed expert tensors missing")
        self.set_banks(banks[("gate_proj", "weight_packed")], banks[("gate_proj", "weight_scale")],
                       banks[("up_proj", "weight_packed")], banks[("up_proj", "weight_scale")],
                       banks[("down_proj", "weight_packed")], banks[("down_proj", "weight_scale")])

    # -- native view -------------------------------------------------------
    def _bank_key(self) -> tuple:
        """Identity and address of the six bank tensors: the cached native table
        is rebuilt when a bank is rebound or its storage replaced."""
        banks = (self.gate_proj.weight_packed, self.gate_proj.weight_scale, self.up_proj.weight_packed,
                 self.up_proj.weight_scale, self.down_proj.weight_packed, self.down_proj.weight_scale)
        return tuple(id(t) for t in banks) + tuple(_ptr(t) for t in banks), banks

    def native_weights(self) -> _native.LgWeights:
        key, banks = self._bank_key()
        if self._w is None or self._w_key != key:
            g, u, dn = self.gate_proj, self.up_proj, self.down_proj
            for name, t in (("gate_proj", g.weight_packed), ("up_proj", u.weight_packed),
                            ("down_proj", dn.weight_packed)):
                require_weight(t, f"experts.{name}")
            w = _native.LgWeights()
            w.gate_packed, w.gate_scale = g.weight_packed.data_ptr(), g.weight_scale.data_ptr()
            w.up_packed, w.up_scale = u.weight_packed.data_ptr(), u.weight_scale.data_ptr()
            w.down_packed, w.down_scale = dn.weight_packed.data_ptr(), dn.weight_scale.data_ptr()
            w.gate_packed_stride = g.weight_packed[0].numel()
            w.gate_scale_stride = g.weight_scale[0].numel()
            w.up_packed_stride = u.weight_packed[0].numel()
            w.up_scale_stride = u.weight_scale[0].numel()
            w.down_packed_stride = dn.weight_packed[0].numel()
            w.down_scale_stride = dn.weight_scale[0].numel()
            self._w, self._w_key, self._w_refs = w, key, banks  # refs keep the ids unique
        return self._w

    # -- reference interface -------------------------------------------------
    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """expert_ssd.py:159-188: per-route down(limited_swiglu(gate, up)) -> [M, k, d] bf16."""
        c = self.config
        rows = _rows_bf16(x, c.hidden_size)
        if indices.ndim < 1 or indices.shape[-1] != c.num_experts_per_tok:
            raise ContractError("routed expert indices must have a top-k dimension")
        idx = indices.reshape(-1, c.num_experts_per_tok)
        if idx.shape[0] != rows.shape[0]:
            raise ContractError("token and routed-index counts differ")
        idx = idx.to(device=rows.device).contiguous()
        if idx.dtype != torch.uint32:
            idx = idx.to(torch.int64).to(torch.int32).view(torch.uint32)
        M, dev = rows.shape[0], rows.device
        y = torch.empty(M, c.num_experts_per_tok, c.hidden_size, dtype=torch.bfloat16, device=dev)
        ws, nbytes = self._ws.get(self._cfg, M, dev)
        rc = _native.load().lg_moe_experts(self._cfg, self.native_weights(), rows.data_ptr(),
                                           idx.data_ptr(), M, y.data_ptr(), ws, nbytes,
                                           _stream_ptr(dev))
        _native.check(rc, "lg_moe_experts")
        self._record(idx, M)
        return y

    def _record(self, idx: torch.Tensor, M: int) -> None:
        self._routes += M * self.config.num_experts_per_tok
        self._last_indices = idx

    @property
    def last_expert_ids(self) -> tuple[int, ...]:
        """Routed expert ids of the last call, flattened (expert_ssd.py:165).
        Reading it synchronises with the device."""
        if self._last_indices is None:
            return ()
        return tuple(int(v) for v in self._last_indices.view(torch.int32).reshape(-1).cpu().tolist())

    def stats(self) -> ExpertCacheStats:
        E = self.config.n_routed_experts
        return ExpertCacheStats(self.layer, E, E, self._routes, 0, 0)

    def clear(self) -> None:
        """Nothing to evict: experts stay resident."""


class _Linear:
    def __init__(self, input_dims: int, output_dims: int):
        self.input_dims = input_dims
        self.output_dims = output_dims
        self.weight: torch.Tensor | None = None  # bf16 [out, in]


class DenseMLP:
    """Shared expert with bf16 weights (layers.py:160-171, bf16 branch 66-67)."""

    def __init__(self, hidden_size: int, intermediate_size: int, swiglu_limit: float,
                 config: MoEConfig | None = None):
        self.gate_proj = _Linear(hidden_size, intermediate_size)
        self.up_proj = _Linear(hidden_size, intermediate_size)
        self.down_proj = _Linear(intermediate_size, hidden_size)
        self.swiglu_limit = swiglu_limit
        if config is None:
            config = MoEConfig(hidden_size=hidden_size, moe_intermediate_size=intermediate_size,
                               n_routed_experts=2, num_experts_per_tok=1, n_shared_experts=1,
                               swiglu_limit=swiglu_limit)
        self.config = config
        self._cfg = _native.LgConfig.from_config(config)
        self._ws = Workspace()

    quantization_mode: str | None = None

    def quantize_to_mxfp(self, bits: int) -> tuple[int, int]:
        """The reference runtime's resident quantisation of the three linears
        (layers.py:67-104, DeferredLinear.quantize_to_mxfp: mx.quantize with
        group size 32, mode mxfp8 / mxfp4), done on the GPU by lg_mx_requantize.
        The quantised values are kept as bf16 (bf16 holds every MXFP8 / MXFP4
        value exactly), so the shared-expert kernels compute the quantised
        products.  Returns (source bytes, bytes of the MX encoding) as the
        reference does."""
        if bits not in (4, 8):
            raise ContractError(f"unsupported resident quantization: mxfp{bits}")
        if self.quantization_mode is not None:
            raise ContractError("deferred linear was already quantized")
        source = dest = 0
        for name, lin in (("gate_proj", self.gate_proj), ("up_proj", self.up_proj), ("down_proj", self.down_proj)):
            t = require_weight(lin.weight, f"shared_experts.{name}.weight")
            if t.dim() != 2 or t.shape[-1] % 32 or t.dtype != torch.bfloat16 or not t.is_cuda:
                raise ContractError(f"resident MXFP{bits} requires a group-32 bf16 CUDA matrix: {tuple(t.shape)}")
            t = t.contiguous()
            out = torch.empty_like(t)
            _native.check(_native.load().lg_mx_requantize(t.data_ptr(), t.shape[0], t.shape[1], bits,
                                                          out.data_ptr(), _stream_ptr(t.device)),
                          "lg_mx_requantize")
            lin.weight = out
            source += t.numel() * 2
            dest += t.numel() * bits // 8 + t.numel() // 32
        self.quantization_mode = f"mxfp{bits}"
        return source, dest

    def quantize_to_mxfp8(self) -> tuple[int, int]:
        return self.quantize_to_mxfp(8)

    def quantize_to_mxfp4(self) -> tuple[int, int]:
        return self.quantize_to_mxfp(4)

    def native_into(self, w: _native.LgWeights) -> None:
        for name, lin in (("gate_proj", self.gate_proj), ("up_proj", self.up_proj),
                          ("down_proj", self.down_proj)):
            t = require_weight(lin.weight, f"shared_experts.{name}.weight")
            if t.dtype != torch.bfloat16 or tuple(t.shape) != (lin.output_dims, lin.input_dims):
                raise ContractError(f"shared_experts.{name}.weight must be bf16 "
                                    f"[{lin.output_dims}, {lin.input_dims}]")
            if not t.is_cuda or not t.is_contiguous():
                raise ContractError(f"shared_experts.{name}.weight must be a contiguous CUDA tensor")
        w.shared_gate = self.gate_proj.weight.data_ptr()
        w.shared_up = self.up_proj.weight.data_ptr()
        w.shared_down = self.down_proj.weight.data_ptr()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        c = self.config
        rows = _rows_bf16(x, c.hidden_size)
        w = _native.LgWeights()
        self.native_into(w)
        M, dev = rows.shape[0], rows.device
        out = torch.empty(M, c.hidden_size, dtype=torch.bfloat16, device=dev)
        ws, nbytes = self._ws.get(self._cfg, M, dev)
        rc = _native.load().lg_moe_shared(self._cfg, w, rows.data_ptr(), M, out.data_ptr(), ws,
                                          nbytes, _stream_ptr(dev))
        _native.check(rc, "lg_moe_shared")
        return out.reshape(*x.shape[:-1], c.hidden_size)


ExpertFactory = Callable[[int], ResidentExperts]


class ExpertSSDMoE:
    """Shared bf16 MLP plus HBM-resident MXFP4 routed experts (moe.py:70-201)."""

    def __init__(self, config: MoEConfig, layer_idx: int, expert_factory: ExpertFactory):
        self.config = config
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.gate = TopKRouter(config)
        self.experts = expert_factory(layer_idx)
        if not isinstance(self.experts, ResidentExperts):
            raise ContractError(
                f"sparse layer {layer_idx} must be backed by ResidentExperts, got "
                f"{type(self.experts).__name__}"
            )
        self.shared_experts = DenseMLP(config.hidden_size, config.shared_intermediate_size,
                                       config.swiglu_limit, config)
        self.last_route: tuple[int, ...] = ()
        self._last_indices: torch.Tensor | None = None
        self._cfg = _native.LgConfig.from_config(config)
        self._ws = Workspace()
        self._w_cache: tuple | None = None

    def _weight_key(self) -> tuple:
        """Identity and address of every tensor the native weight table points
        at; the table is rebuilt (and re-validated) when any of them changes."""
        g, s = self.gate, self.shared_experts
        refs = (g.weight, g.e_score_correction_bias, s.gate_proj.weight, s.up_proj.weight,
                s.down_proj.weight, self.experts.native_weights())
        ptrs = tuple(_ptr(t) for t in refs[:5])
        return refs, ptrs

    def native_weights(self) -> _native.LgWeights:
        refs, ptrs = self._weight_key()
        c = self._w_cache
        if c is not None and c[1] == ptrs and all(a is b for a, b in zip(c[0], refs)):
            return c[2]
        w = self._build_native_weights()
        self._w_cache = (refs, ptrs, w)
        return w

    def _build_native_weights(self) -> _native.LgWeights:
        w = _native.LgWeights()
        ctypes_copy = self.experts.native_weights()
        for name, _ in _native.LgWeights._fields_:
            setattr(w, name, getattr(ctypes_copy, name))
        w.router_weight = require_weight(self.gate.weight, "router.weight").data_ptr()
        w.router_bias = require_weight(self.gate.e_score_correction_bias,
                                       "router.e_score_correction_bias").data_ptr()
        if self.config.n_shared_experts > 0:
            self.shared_experts.native_into(w)
        return w

    def __call__(self, hidden_states: torch.Tensor, *, return_route: bool = False,
                 out: torch.Tensor | None = None):
        """bf16 hidden states [..., d] -> f32 [..., d] (moe.py:96-201).

        The hidden states may be on the device or, as the reference's unified
        memory allows, in page-locked host memory (read once by the GPU).
        `out`, when given, receives the result (device or page-locked host
        memory) and is returned reshaped; like a non-blocking copy, a host
        `out` holds the result once the current stream reaches this point."""
        rows = _rows_bf16(hidden_states, self.hidden_size, allow_host=True)
        w = self.native_weights()
        M = rows.shape[0]
        dev = rows.device if rows.is_cuda else self.gate.weight.device
        k = self.config.num_experts_per_tok
        if out is None:
            out = torch.empty(M, self.hidden_size, dtype=torch.float32, device=dev)
        else:
            out = _out_f32(out, M, self.hidden_size)
        weights = torch.empty(M, k, dtype=torch.float32, device=dev)
        indices = torch.empty(M, k, dtype=torch.uint32, device=dev)
        ws, nbytes = self._ws.get(self._cfg, M, dev)
        rc = _native.load().lg_moe_forward(self._cfg, w, rows.data_ptr(), M,
                                           out.data_ptr(), weights.data_ptr(), indices.data_ptr(),
                                           ws, nbytes, _stream_ptr(dev))
        _native.check(rc, "lg_moe_forward")
        self._last_indices = indices
        self.experts._record(indices, M)
        result = out.reshape(*hidden_states.shape[:-1], self.hidden_size)
        if return_route:
            return result, weights, indices
        return result

    def device_status(self) -> int:
        """Status word of this layer's workspace: 0, or LG_ERR_TIMEOUT | site << 8
        if a bounded device wait gave up."""
        return self._ws.status()

    def use_workspace(self, ws: Workspace) -> None:
        """Run on a workspace shared with other layers.  Calls that share one
        must not overlap on the GPU: layers called in order on one stream."""
        self._ws = ws

    @property
    def last_route_ids(self) -> tuple[int, ...]:
        """The reference's last_route (moe.py:179,200); synchronises."""
        return self.experts.last_expert_ids

    # -- loading -------------------------------------------------------------
    def load_checkpoint(self, tensors: Mapping[str, torch.Tensor], device="cuda") -> None:
        """Bind this layer's tensors by checkpoint name: router
        (`mlp.gate.weight`, `mlp.gate.e_score_correction_bias`), shared expert
        (`mlp.shared_experts.{gate,up,down}_proj.weight`, bf16) and routed
        experts (see ResidentExperts.load_checkpoint)."""
        p = f"model.language_model.layers.{self.layer_idx}.mlp."
        try:
            self.gate.weight = tensors[p + "gate.weight"].to(device=device, dtype=torch.float32).contiguous()
            self.gate.e_score_correction_bias = tensors[p + "gate.e_score_correction_bias"].to(
                device=device, dtype=torch.float32).contiguous()
            for name in ("gate_proj", "up_proj", "down_proj") if self.config.n_shared_experts > 0 else ():
                key = p + f"shared_experts.{name}.weight"
                w = tensors[key]
                if w.dtype == torch.float8_e4m3fn:  # block-FP8 with f32 block scales, widened on the GPU
                    w = widen_block_fp8(w.to(device), tensors[key + "_scale_inv"])
                getattr(self.shared_experts, name).weight = w.to(device=device, dtype=torch.bfloat16).contiguous()
        except KeyError as exc:
            raise ContractError(f"resident parameter was not loaded: {exc.args[0]}") from None
        self.experts.load_checkpoint(tensors, device=device)

    def quantize_resident_linears_mxfp(self, bits: int = 8) -> dict:
        """The block's part of the reference runtime's resident quantisation
        (model.py:240-262: every resident 2-D linear except the router gate,
        resident_plan.py:77-86): the shared expert's linears to MXFP8 (the
        runtime default) or MXFP4.  The routed experts are MXFP4 already."""
        if self.config.n_shared_experts < 1:
            return {"mode": f"mxfp{bits}", "linears": 0, "source_bytes": 0, "destination_bytes": 0}
        source, dest = self.shared_experts.quantize_to_mxfp(bits)
        return {"mode": f"mxfp{bits}", "linears": 3, "source_bytes": source, "destination_bytes": dest}

    @classmethod
    def from_checkpoint(cls, path, config: MoEConfig, layer_idx: int, device="cuda") -> "ExpertSSDMoE":
        """Construct layer `layer_idx` from a safetensors checkpoint directory
        (index + shards) or file: routed experts bound byte for byte into HBM
        banks, router in f32, shared expert in bf16 (block-FP8 widened)."""
        from .safetensors import SafetensorsCheckpoint

        ckpt = path if isinstance(path, SafetensorsCheckpoint) else SafetensorsCheckpoint(path)
        moe = cls(config, layer_idx, lambda layer: ResidentExperts(config, layer=layer))
        moe.load_checkpoint(ckpt.layer_tensors(layer_idx), device=device)
        return moe


def build_layer(config: MoEConfig, tensors: dict, layer_idx: int = 0) -> ExpertSSDMoE:
    """Construct a layer from stacked bank tensors (the synthetic.layer_weights
    layout) without going through checkpoint names."""
    def factory(layer: int) -> ResidentExperts:
        ex = ResidentExperts(config, layer=layer)
        ex.set_banks(tensors["gate_packed"], tensors["gate_scale"], tensors["up_packed"],
                     tensors["up_scale"], tensors["down_packed"], tensors["down_scale"])
        return ex

    moe = ExpertSSDMoE(config, layer_idx, factory)
    moe.gate.weight = tensors["router_weight"]
    moe.gate.e_score_correction_bias = tensors["router_bias"]
    if config.n_shared_experts > 0:
        moe.shared_experts.gate_proj.weight = tensors["shared_gate"]
        moe.shared_experts.up_proj.weight = tensors["shared_up"]
        moe.shared_experts.down_proj.weight = tensors["shared_down"]
    return moe
