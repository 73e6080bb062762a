"""Builds the sm_100a C-ABI library ``molten_b200/libmolten_cuda.so`` in-tree.

nvcc compiles every ``csrc/*.cu`` for ``sm_100a`` (it cross-compiles; no GPU
is needed), one object per file in parallel, and links them. ``--fmad=false`` keeps nvcc from fusing
multiply-adds on its own: every fused multiply-add in the kernels is written
out explicitly, because the decode path's reduction order is part of its
contract (bit-identical ids and tokens).
"""
from __future__ import annotations

import fcntl
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libmolten_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + [HERE.parent / "include" / "molten_cuda.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library if a source is newer: one object per csrc/*.cu,
    compiled in parallel (no device symbol crosses files), then one link.
    Concurrent callers (the spawned ranks of multi-process tests) are
    serialised by an exclusive lock next to the library; each re-checks
    staleness under it."""
    if not force and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    with open(HERE / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not needs_build():
            return LIB
        objdir = HERE / "_build"
        objdir.mkdir(exist_ok=True)
        tag = os.getpid()
        objs = [objdir / f"{src.stem}.{tag}.o" for src in sources()]
        jobs = [[NVCC, *NVCC_FLAGS, "-c", "-o", str(o), str(src)]
                for src, o in zip(sources(), objs)]
        try:
            with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
                list(ex.map(lambda c: _run(c, verbose), jobs))
            tmp = LIB.with_suffix(f".so.{tag}.tmp")
            _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
                  *map(str, objs), "-ldl"], verbose)
            os.replace(tmp, LIB)
        finally:
            for o in objs:
                if o.exists():
                    o.unlink()
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
