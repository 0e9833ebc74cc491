"""Build the CUDA library in-tree for sm_100a.

    python -m livglm_b200.build

Produces livglm_b200/_lib/liblivglm_moe.so from livglm_b200/csrc/*.cu with
nvcc (cross-compiles without a GPU), and liblivglm_moe_ep.so (the
expert-parallel layer, csrc/moe_ep.cu) linked against it and against the NCCL
that PyTorch ships (the same libnccl.so.2 torch.distributed loads, so a
process holds one NCCL).  The .so files are git-ignored but ship with the
source tree to GPU hosts.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "_lib" / "liblivglm_moe.so"
SOURCES = ["moe_capi.cu", "moe_noalloc.cu", "ffn_site.cu"]
EP_OUT = PKG / "_lib" / "liblivglm_moe_ep.so"
EP_SOURCES = ["moe_ep.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, sources: list[Path]) -> bool:
    if not out.exists():
        return True
    deps = list(CSRC.glob("*.cu*")) + list((ROOT / "include").glob("*.h")) + list(sources)
    return max(p.stat().st_mtime for p in deps) > out.stat().st_mtime


def nccl_dir() -> Path:
    """The nvidia-nccl wheel PyTorch depends on (include/nccl.h, lib/libnccl.so.2)."""
    import torch

    site = Path(torch.__file__).resolve().parents[1]
    cand = site / "nvidia" / "nccl"
    if not (cand / "include" / "nccl.h").exists() or not (cand / "lib" / "libnccl.so.2").exists():
        raise RuntimeError(f"NCCL headers/library not found under {cand}")
    return cand


def build_library(out: Path, sources: list[Path], force: bool = False, verbose: bool = False,
                  extra: list[str] | None = None) -> Path:
    """nvcc -shared for sm_100a with the package's headers on the include path."""
    if not force and not _stale(out, sources):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(f".{os.getpid()}.tmp")
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           f"-Xlinker=-soname={out.name}", f"-I{ROOT / 'include'}", f"-I{CSRC}",
           *[str(s) for s in sources], *(extra or []), "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def build_ep(force: bool = False, verbose: bool = False) -> Path:
    """liblivglm_moe_ep.so: needs liblivglm_moe.so (found next to it at run
    time) and NCCL (the libnccl.so.2 already loaded by torch, else the wheel's)."""
    nccl = nccl_dir()
    extra = [f"-I{nccl / 'include'}", f"-L{OUT.parent}", "-llivglm_moe", f"-L{nccl / 'lib'}", "-l:libnccl.so.2",
             "-Xlinker=-rpath=$ORIGIN", f"-Xlinker=-rpath={nccl / 'lib'}"]
    sources = [CSRC / s for s in EP_SOURCES]
    if not force and EP_OUT.exists() and OUT.exists() and OUT.stat().st_mtime > EP_OUT.stat().st_mtime:
        force = True  # relink after the main library changed
    return build_library(EP_OUT, sources, force, verbose, extra)


def build(force: bool = False, verbose: bool = False) -> Path:
    out = build_library(OUT, [CSRC / s for s in SOURCES], force, verbose)
    build_ep(force, verbose)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
