"""CPU tests of the C ABI boundary: the library loads without a GPU, exports
every symbol include/molten_cuda.h declares, and validates arguments (no
compute call is made)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "molten_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mc_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from molten_b200 import build, _lib
    build.build()
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_signatures_cover_header(lib):
    from molten_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES), (
        set(declared_symbols()) ^ set(_lib.SIGNATURES))


def test_version_and_error_channel(lib):
    assert b"sm_100a" in lib.mc_version()
    from molten_b200 import _lib
    rc = lib.mc_check_quant(None)
    assert rc == _lib.MC_EINVAL
    assert b"null" in lib.mc_last_error()


def _qw(codes=0x1000, bits=4, group=64, out=2048, inp=2048):
    from molten_b200 import _lib
    return _lib.QW(codes, 0x2000, 0x3000, out, inp, group, bits)


def test_check_quant_rules(lib):
    """check_quant (quant.rs:42-66): bit width, block-packable groups and the
    16-byte code alignment -- evaluated on descriptors, no device memory."""
    from molten_b200 import _lib
    assert lib.mc_check_quant(C.byref(_qw())) == 0
    assert lib.mc_check_quant(C.byref(_qw(bits=3))) == _lib.MC_EINVAL
    assert b"bit width" in lib.mc_last_error()
    assert lib.mc_check_quant(C.byref(_qw(codes=0x1008))) == _lib.MC_EINVAL
    assert b"16-aligned" in lib.mc_last_error()
    assert lib.mc_check_quant(C.byref(_qw(inp=2000))) == _lib.MC_EINVAL
    assert lib.mc_check_quant(C.byref(_qw(group=16))) == _lib.MC_EINVAL  # 16 < 32 codes/block
    assert lib.mc_check_quant(C.byref(_qw(bits=6, group=64))) == 0


def test_entry_points_reject_null_context(lib):
    from molten_b200 import _lib
    q = _qw()
    assert lib.mc_gemv_quant(None, C.byref(q), 0x100, 0x200, 1) == _lib.MC_EINVAL
    assert b"null context" in lib.mc_last_error()
    assert lib.mc_moe_sort_map(None, 0x1, 16, 64, 128, 1, 1, 1, 1, 1, 1, 100) == _lib.MC_EINVAL


def test_python_mirror_raises_on_bad_shapes():
    import torch
    from molten_b200 import quant
    w = quant.QuantWeights(torch.zeros((8, 256), dtype=torch.int32),
                           torch.zeros((8, 31), dtype=torch.bfloat16),
                           torch.zeros((8, 32), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="scales/biases shape"):
        quant.check_quant(w)


def test_product_does_not_import_oracle():
    """The product path never routes through the CPU oracle."""
    for p in (ROOT / "molten_b200").rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p
    for p in (ROOT / "molten_b200" / "csrc").glob("*"):
        for line in p.read_text().splitlines():
            if line.lstrip().startswith("#include") or "dlopen" in line:
                assert "oracle" not in line, (p, line)
