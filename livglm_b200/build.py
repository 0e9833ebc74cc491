"""Build the CUDA library in-tree for sm_100a.

    python -m livglm_b200.build

Produces livglm_b200/_lib/liblivglm_moe.so from livglm_b200/csrc/*.cu with
nvcc (cross-compiles without a GPU).  The .so is git-ignored but ships with
the source tree to GPU hosts.
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
SOURCES = ["moe_capi.cu", "moe_noalloc.cu"]
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


def build_library(out: Path, sources: list[Path], force: bool = False, verbose: bool = False) -> Path:
    """nvcc -shared for sm_100a with the package's headers on the include path."""
    if not force and not _stale(out, sources):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(f".{os.getpid()}.tmp")
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           f"-I{ROOT / 'include'}", f"-I{CSRC}", *[str(s) for s in sources], "-o", str(tmp)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def build(force: bool = False, verbose: bool = False) -> Path:
    return build_library(OUT, [CSRC / s for s in SOURCES], force, verbose)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
