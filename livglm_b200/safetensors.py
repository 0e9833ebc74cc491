"""Read tensors by name from a (composite) safetensors checkpoint.

The GLM-5.3-Flash checkpoint the reference loads (kg36/livglm
src/glm53flash/contract.py:47-50, resident_plan.py:177-279,
expert_source.py:270-381) is a directory of safetensors shards with a
`model.safetensors.index.json` weight map.  A shard is an 8-byte
little-endian header length N, N bytes of JSON {name: {"dtype", "shape",
"data_offsets": [begin, end]}, "__metadata__": {...}}, then the data;
offsets are relative to the end of the header.

SafetensorsCheckpoint maps names to shards, checks every header against its
file, and returns a tensor as a torch tensor over a read-only memory map of
the shard (copied to the device when one is given).  F8_E4M3 comes back as
torch.float8_e4m3fn (the raw bytes), U8 as uint8: the MoE block binds the
expert banks byte for byte and widens block-FP8 weights on the GPU
(ExpertSSDMoE.load_checkpoint).
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .config import ContractError

INDEX_NAME = "model.safetensors.index.json"
_DTYPES = {
    "U8": (np.uint8, torch.uint8, 1), "I8": (np.int8, torch.int8, 1),
    "BF16": (np.uint16, torch.bfloat16, 2), "F16": (np.float16, torch.float16, 2),
    "F32": (np.float32, torch.float32, 4), "I32": (np.int32, torch.int32, 4),
    "I64": (np.int64, torch.int64, 8), "F8_E4M3": (np.uint8, torch.float8_e4m3fn, 1),
}
_MAX_HEADER = 100 << 20


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple[int, ...]
    shard: Path
    offset: int  # absolute byte offset in the shard
    nbytes: int


def read_header(path: Path) -> dict[str, TensorInfo]:
    """The tensors of one shard, each checked to lie inside the file."""
    size = path.stat().st_size
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ContractError(f"safetensors shard too short: {path}")
        (n,) = struct.unpack("<Q", raw)
        if n > _MAX_HEADER or 8 + n > size:
            raise ContractError(f"safetensors header length {n} invalid: {path}")
        try:
            header = json.loads(f.read(n))
        except ValueError as exc:
            raise ContractError(f"safetensors header is not JSON: {path}") from exc
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        try:
            dtype, shape, (begin, end) = meta["dtype"], tuple(int(s) for s in meta["shape"]), meta["data_offsets"]
        except (KeyError, TypeError, ValueError) as exc:
            raise ContractError(f"safetensors entry malformed: {name} in {path}") from exc
        if dtype not in _DTYPES:
            raise ContractError(f"unsupported safetensors dtype {dtype}: {name}")
        count = int(np.prod(shape, dtype=np.int64)) if shape else 1
        if end - begin != count * _DTYPES[dtype][2] or begin < 0 or 8 + n + end > size:
            raise ContractError(f"safetensors byte range of {name} does not match its shape or file")
        out[name] = TensorInfo(name, dtype, shape, path, 8 + n + begin, end - begin)
    return out


class SafetensorsCheckpoint:
    """Name -> tensor over a checkpoint directory (index + shards) or one file."""

    def __init__(self, path: str | Path):
        path = Path(path)
        self.tensors: dict[str, TensorInfo] = {}
        if path.is_file():
            self.tensors = read_header(path)
            return
        index = path / INDEX_NAME
        if index.exists():
            weight_map = json.loads(index.read_text()).get("weight_map")
            if not isinstance(weight_map, dict):
                raise ContractError(f"{index} has no weight_map")
            headers = {s: read_header(path / s) for s in sorted(set(weight_map.values()))}
            for name, shard in weight_map.items():
                info = headers[shard].get(name)
                if info is None:
                    raise ContractError(f"{name} is mapped to {shard} but not stored there")
                self.tensors[name] = info
        else:
            for shard in sorted(path.glob("*.safetensors")):
                for name, info in read_header(shard).items():
                    if name in self.tensors:
                        raise ContractError(f"{name} is stored in two shards")
                    self.tensors[name] = info
        if not self.tensors:
            raise ContractError(f"no safetensors tensors under {path}")

    def names(self, prefix: str = "") -> list[str]:
        return sorted(n for n in self.tensors if n.startswith(prefix))

    def info(self, name: str) -> TensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise ContractError(f"checkpoint has no tensor {name}") from None

    def tensor(self, name: str, device=None) -> torch.Tensor:
        t = self.info(name)
        np_dtype, torch_dtype, _ = _DTYPES[t.dtype]
        arr = np.memmap(t.shard, dtype=np_dtype, mode="r", offset=t.offset, shape=t.shape or (1,))
        host = torch.from_numpy(np.array(arr, copy=True))
        if t.dtype in ("BF16", "F8_E4M3"):
            host = host.view(torch_dtype)
        host = host.reshape(t.shape)
        return host if device is None else host.to(device)

    def layer_tensors(self, layer: int, device=None) -> dict[str, torch.Tensor]:
        """Every tensor of layer `layer`'s MLP (router, shared and routed experts)."""
        prefix = f"model.language_model.layers.{layer}.mlp."
        names = self.names(prefix)
        if not names:
            raise ContractError(f"checkpoint has no tensors under {prefix}")
        return {n: self.tensor(n, device) for n in names}
