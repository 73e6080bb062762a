"""Quantized weights in MLX affine form (weights.rs:7-30) and their check
(``check_quant``, quant.rs:42-66)."""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class QuantWeights:
    """One linear layer in MLX affine form.

    codes: int32 [out, in * bits / 32] (u32 bit patterns, 32/bits codes per
    word for Q4, low code first; Q6 rows are a little-endian 6-bit stream);
    scales, biases: bf16 [out, in / group_size]; w = scale * q + bias.
    """

    codes: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int = 64
    bits: int = 4

    @property
    def out_features(self) -> int:
        return self.codes.shape[0]

    @property
    def in_features(self) -> int:
        return self.codes.shape[1] * 32 // self.bits

    def qw(self) -> _lib.QW:
        return _lib.QW(self.codes.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                       self.out_features, self.in_features, self.group_size, self.bits)

    def to(self, device) -> "QuantWeights":
        return QuantWeights(self.codes.to(device), self.scales.to(device),
                            self.biases.to(device), self.group_size, self.bits)

    def rows(self, start: int, stop: int) -> "QuantWeights":
        """View of output rows [start, stop) (a stacked expert's slice)."""
        return QuantWeights(self.codes[start:stop], self.scales[start:stop],
                            self.biases[start:stop], self.group_size, self.bits)


def check_quant(w: QuantWeights) -> tuple[int, int]:
    """check_quant (quant.rs:42-66): returns (out, in) or raises ValueError."""
    n, k = w.out_features, w.in_features
    if w.codes.dtype != torch.int32:
        raise ValueError("codes must be U32 (stored as int32)")
    if w.scales.dtype != torch.bfloat16 or w.biases.dtype != torch.bfloat16:
        raise ValueError("scales/biases must be BF16")
    if tuple(w.scales.shape) != (n, k // w.group_size) or \
            tuple(w.biases.shape) != (n, k // w.group_size):
        raise ValueError(f"scales/biases shape mismatch for [{n}, {k}] gs={w.group_size}")
    for t in (w.codes, w.scales, w.biases):
        if not t.is_contiguous():
            raise ValueError("weights must be contiguous")
    rc = _lib.lib().mc_check_quant(w.qw())
    if rc != _lib.MC_OK:
        raise ValueError(_lib.lib().mc_last_error().decode())
    return n, k
