"""Builds the CPU oracle (test infrastructure only).

libmc_oracle.so: the bit-careful restatement (mc_oracle.c), compiled with
-ffp-contract=off so only the fmaf calls it names are fused (-O3 and OpenMP
change no result: without -ffast-math nothing is reassociated, and the
parallel loops split independent outputs). Output goes to
oracle/_build/ (git-ignored; it travels to the GPU box with the tree, and the
box rebuilds it if missing -- gcc is in the image).

-march=x86-64-v3 (AVX2 + FMA) rather than -march=native so a library built
here also runs on the GPU box's host CPU.
"""
from __future__ import annotations

import fcntl
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


def _compile(cmd_head: list[str], lib: Path, src: Path, tail: list[str]) -> None:
    tmp = f"{lib}.{os.getpid()}.tmp"
    subprocess.run([*cmd_head, "-o", tmp, str(src), *tail], check=True)
    os.replace(tmp, lib)


def build(force: bool = False) -> tuple[Path, Path | None]:
    """Compiles what is stale. Several processes (the spawned ranks of the
    multi-process tests) may call this at once: an exclusive lock on
    _build/.lock serialises them, and each re-checks staleness under it."""
    OUT.mkdir(exist_ok=True)
    with open(OUT / ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        src = HERE / "mc_oracle.c"
        if force or _stale(EXACT, src):
            _compile(["gcc", "-O3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", *COMMON],
                     EXACT, src, ["-lm"])
        fast_src = HERE / "mc_oracle_fast.c"
        if fast_src.exists() and (force or _stale(FAST, fast_src)):
            _compile(["gcc", "-O3", "-fopenmp", "-ffast-math", *COMMON], FAST, fast_src, ["-lm"])
    return EXACT, FAST if FAST.exists() else None


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
