"""Helpers shared by the GPU tests: numpy <-> CUDA tensor plumbing."""
import numpy as np
import torch

from molten_b200 import synth
from molten_b200.quant import QuantWeights


def dev_bf16(bits: np.ndarray) -> torch.Tensor:
    return synth.bf16_tensor(np.ascontiguousarray(bits)).cuda()


def dev_u32(a: np.ndarray) -> torch.Tensor:
    return synth.u32_tensor(np.ascontiguousarray(a, dtype=np.uint32)).cuda()


def dev_f32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def dev_qw(codes, s, b, bits=4) -> QuantWeights:
    return QuantWeights(dev_u32(codes), dev_bf16(s), dev_bf16(b), 64, bits)


def host_bits(t: torch.Tensor) -> np.ndarray:
    return synth.tensor_bits(t)


def host_u32(t: torch.Tensor) -> np.ndarray:
    return synth.tensor_u32(t)


def empty_bf16(*shape) -> torch.Tensor:
    return torch.empty(shape, dtype=torch.bfloat16, device="cuda")


def zeros_u32(*shape) -> torch.Tensor:
    return torch.zeros(shape, dtype=torch.int32, device="cuda")


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str = ""):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
    assert bad.size == 0, f"{what}: {bad.size} of {got.size} differ, first at {bad[:8]}"
