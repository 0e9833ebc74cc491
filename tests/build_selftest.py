"""Build the tcgen05 building-block self-test library (test infrastructure).

    python -m tests.build_selftest

Compiles tests/csrc/umma_selftest.cu against the product's tensor-core
primitives (livglm_b200/csrc/umma.cuh) into tests/_build/liblivglm_umma_selftest.so
for sm_100a.  Only tests/test_gpu_umma.py loads it; it is not part of the
MoE library.
"""

from __future__ import annotations

import sys
from pathlib import Path

from livglm_b200 import build as lib_build

TESTS = Path(__file__).resolve().parent
OUT = TESTS / "_build" / "liblivglm_umma_selftest.so"
SOURCES = [TESTS / "csrc" / "umma_selftest.cu"]


def build(force: bool = False, verbose: bool = False) -> Path:
    return lib_build.build_library(OUT, SOURCES, force=force, verbose=verbose)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
