"""The C++ host mirror (include/molten_b200.hpp) driving the kernels on the
GPU, checked bit for bit against the CPU oracle (tests/cpp/test_host_mirror_gpu.cpp)."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from molten_b200 import synth

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")

pytestmark = pytest.mark.gpu


def test_cpp_host_mirror_on_gpu(tmp_path):
    assert shutil.which("g++") is not None, "needs g++"
    from molten_b200 import build
    lib = build.build()
    g = synth.rng(77)
    for name, n, bits, b in (("q4", 2048, 4, 3), ("q6", 65536, 6, 2)):
        codes, s, bi = synth.quant_weights_np(g, n, 2048, bits)
        x = synth.activations_np(g, b, 2048)
        for part, arr in (("codes", codes), ("scales", s), ("biases", bi), ("x", x)):
            np.ascontiguousarray(arr).tofile(tmp_path / f"{name}_{part}.bin")
        if bits == 4:
            np.ascontiguousarray(oracle.gemv_quant(codes, s, bi, 4, x)).tofile(tmp_path / "q4_want.bin")
        else:
            keys, _ = oracle.head_argmax(codes, s, bi, 6, x)
            np.ascontiguousarray(keys.astype(np.uint64)).tofile(tmp_path / "q6_keys.bin")
    exe = tmp_path / "test_host_mirror_gpu"
    cmd = ["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"),
           str(ROOT / "tests" / "cpp" / "test_host_mirror_gpu.cpp"), "-L", str(lib.parent),
           "-lmolten_cuda", f"-Wl,-rpath,{lib.parent}", "-L", str(CUDA / "lib64"), "-lcudart",
           f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok (0 failures)")
