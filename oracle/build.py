"""Builds the CPU oracle (test infrastructure only).

libmc_oracle.so: the bit-careful restatement (mc_oracle.c), compiled with
-ffp-contract=off so only the fmaf calls it names are fused. Output goes to
oracle/_build/ (git-ignored; it travels to the GPU box with the tree, and the
box rebuilds it if missing -- gcc is in the image).

-march=x86-64-v3 (AVX2 + FMA) rather than -march=native so a library built
here also runs on the GPU box's host CPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build"
EXACT = OUT / "libmc_oracle.so"
FAST = OUT / "libmc_oracle_fast.so"

COMMON = ["-shared", "-fPIC", "-march=x86-64-v3", "-std=c11"]


def _stale(lib: Path, src: Path) -> bool:
    return not lib.exists() or lib.stat().st_mtime < max(src.stat().st_mtime,
                                                          Path(__file__).stat().st_mtime)


def build(force: bool = False) -> tuple[Path, Path | None]:
    OUT.mkdir(exist_ok=True)
    src = HERE / "mc_oracle.c"
    if force or _stale(EXACT, src):
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", *COMMON, "-o",
               str(EXACT) + ".tmp", str(src), "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(str(EXACT) + ".tmp", EXACT)
    fast_src = HERE / "mc_oracle_fast.c"
    if fast_src.exists() and (force or _stale(FAST, fast_src)):
        cmd = ["gcc", "-O3", "-fopenmp", "-ffast-math", *COMMON, "-o", str(FAST) + ".tmp",
               str(fast_src), "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(str(FAST) + ".tmp", FAST)
    return EXACT, FAST if FAST.exists() else None


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
