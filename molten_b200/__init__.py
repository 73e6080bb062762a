"""molten_b200: B200 (sm_100a) CUDA implementation of Molten's quantized MoE
matmul path behind a C ABI (include/molten_cuda.h).

Modules:
  _lib   ctypes binding of libmolten_cuda.so (fails loudly if not built)
  quant  QuantWeights / check_quant (weights.rs, quant.rs)
  lfm    op-level mirror of src/kernels/lfm.rs and elementwise.rs
  synth  seeded synthetic inputs with BASELINE.json's shapes and distributions
  build  nvcc build of the library
"""
from . import _lib  # noqa: F401

__all__ = ["_lib", "quant", "lfm", "synth", "build"]
