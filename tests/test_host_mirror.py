"""The C++ host mirror (include/molten_b200.hpp) compiles against the C ABI
and its reference-style argument checks fire before the ABI is reached
(tests/cpp/test_host_mirror.cpp, no GPU needed)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_cpp_host_mirror_checks(tmp_path):
    from molten_b200 import build
    lib = build.build()
    exe = tmp_path / "test_host_mirror"
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cpp" / "test_host_mirror.cpp"), "-L", str(lib.parent),
           "-lmolten_cuda", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok (0 failures)")
