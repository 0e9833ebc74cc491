"""Write safetensors files for test fixtures (test infrastructure): an 8-byte
little-endian header length, the JSON header, then the tensors' bytes."""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

SIZES = {"U8": 1, "I8": 1, "BF16": 2, "F16": 2, "F32": 4, "I32": 4, "I64": 8, "F8_E4M3": 1}


def write(path: Path, tensors: dict[str, tuple[str, np.ndarray]], *, pad_header: int = 8) -> None:
    """tensors: name -> (safetensors dtype, array whose bytes are stored as is)."""
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, (dtype, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        assert len(raw) == int(np.prod(arr.shape, dtype=np.int64)) * SIZES[dtype], name
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % pad_header)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_checkpoint(directory: Path, shards: dict[str, dict[str, tuple[str, np.ndarray]]]) -> None:
    """A checkpoint directory: shards plus model.safetensors.index.json."""
    directory.mkdir(parents=True, exist_ok=True)
    weight_map = {}
    for shard, tensors in shards.items():
        write(directory / shard, tensors)
        weight_map.update({name: shard for name in tensors})
    (directory / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
