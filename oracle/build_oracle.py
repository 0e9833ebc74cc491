"""Build recipe for the CPU oracle's C part -- TEST INFRASTRUCTURE ONLY.

Compiles oracle/router_ref.c (router) and oracle/experts_ref.c (routed and
shared experts, merge) into oracle/_build/liboracle.so with gcc, with
floating-point contraction off so every fmaf/add/mul rounds exactly where the
source says, and OpenMP across tokens and weight rows.  The reference itself (kg36/livglm) is Python + MLX and has no
C/C++ sources for this path, so there is nothing to build under oracle/_ref.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRCS = [HERE / "router_ref.c", HERE / "experts_ref.c"]
OUT = HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    if not force and OUT.exists() and all(OUT.stat().st_mtime >= s.stat().st_mtime for s in SRCS):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(f".{os.getpid()}.tmp")
    cmd = [
        "gcc", "-O3", "-std=c11", "-shared", "-fPIC",
        "-ffp-contract=off", "-fno-fast-math", "-fno-builtin", "-fopenmp",
        *[str(s) for s in SRCS], "-o", str(tmp), "-lm",
    ]
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
