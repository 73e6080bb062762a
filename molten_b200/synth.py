"""Seeded synthetic inputs with BASELINE.json's shapes and value distributions.

The reference benchmarks this path on a real checkpoint; no checkpoint or
dataset is available here, so every config uses seeded synthetic tensors:

  Q4/Q6 codes   uniform random words (each code uniform over its range)
  scales        bf16(U(0.002, 0.02))
  biases        bf16(-8 * scale + N(0, 1e-3))
  activations   bf16(N(0, 1))
  RMSNorm gain  bf16(1 + N(0, 0.02))
  router        bf16(N(0, 0.02))   [E, H]
  cfg3 logits   log(Zipf_1(rank(pi(e)))) + Gumbel(0, 1), pi a seeded
                permutation of the experts, so top-4 is a Plackett-Luce draw
                proportional to a Zipf(s=1) popularity

Generation runs on the host with numpy's Philox (the oracle and the GPU see
identical bytes) or, for the multi-GB bench configs, on the GPU with
torch.Generator (seeded; the CPU baseline then copies a bounded sample).
"""
from __future__ import annotations

import numpy as np
import torch

from .quant import QuantWeights

HIDDEN = 2048
MOE_INTER = 1536
N_EXPERTS = 64
VOCAB = 65536


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(seed))


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def tensor_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u32_tensor(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32))


def tensor_u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.uint32)


def quant_weights_np(g: np.random.Generator, out: int, inp: int, bits: int = 4,
                     centre: float = 8.0):
    """(codes u32 [out, in*bits/32], scales bf16 bits, biases bf16 bits);
    bias = -centre * scale + N(0, 1e-3) (BASELINE: centre 8)."""
    words = inp * bits // 32
    codes = g.integers(0, 2**32, size=(out, words), dtype=np.uint64).astype(np.uint32)
    s = g.uniform(0.002, 0.02, size=(out, inp // 64)).astype(np.float32)
    sb = f32_to_bf16_bits(s)
    b = -centre * bf16_bits_to_f32(sb) + g.normal(0.0, 1e-3, size=s.shape).astype(np.float32)
    bb = f32_to_bf16_bits(b.astype(np.float32))
    return codes, sb, bb


def to_qw(codes, sb, bb, bits=4, device="cpu") -> QuantWeights:
    return QuantWeights(u32_tensor(codes).to(device), bf16_tensor(sb).to(device),
                        bf16_tensor(bb).to(device), 64, bits)


def activations_np(g: np.random.Generator, *shape) -> np.ndarray:
    return f32_to_bf16_bits(g.normal(0.0, 1.0, size=shape).astype(np.float32))


def norm_weight_np(g: np.random.Generator, n: int = HIDDEN) -> np.ndarray:
    return f32_to_bf16_bits((1.0 + g.normal(0.0, 0.02, size=n)).astype(np.float32))


def router_np(g: np.random.Generator, e: int = N_EXPERTS, h: int = HIDDEN) -> np.ndarray:
    return f32_to_bf16_bits(g.normal(0.0, 0.02, size=(e, h)).astype(np.float32))


def zipf_logits_np(g: np.random.Generator, m: int, e: int = N_EXPERTS, s: float = 1.0):
    """Router logits whose top-4 is a Plackett-Luce draw from Zipf(s) popularity."""
    perm = g.permutation(e)
    rank = perm.astype(np.float64) + 1.0
    base = -s * np.log(rank)
    gumbel = g.gumbel(0.0, 1.0, size=(m, e))
    return (base[None, :] + gumbel).astype(np.float32)


# ----------------------------------------------------------- device-side gen

def quant_weights_torch(gen: torch.Generator, out: int, inp: int, bits: int = 4,
                        device="cuda", centre: float = 8.0) -> QuantWeights:
    """Same distributions as quant_weights_np, generated on the device. `centre`
    sets bias = -centre * scale + N(0, 1e-3): 8 as BASELINE states for every
    config; 31.5 centres 6-bit codes (0..63) on zero."""
    words = inp * bits // 32
    codes = torch.randint(-2**31, 2**31 - 1, (out, words), generator=gen, device=device,
                          dtype=torch.int64).to(torch.int32)
    s = torch.empty((out, inp // 64), device=device).uniform_(0.002, 0.02, generator=gen)
    s = s.to(torch.bfloat16)
    b = (-centre * s.float() + torch.randn(s.shape, generator=gen, device=device) * 1e-3)
    return QuantWeights(codes, s, b.to(torch.bfloat16), 64, bits)


def moe_layer_torch(gen: torch.Generator, device="cuda", e: int = N_EXPERTS, h: int = HIDDEN,
                    i: int = MOE_INTER, centre: float = 8.0) -> dict:
    """One cfg1 MoE layer: norm gain, bf16 router, stacked gate/up/down
    (`centre` as in quant_weights_torch)."""
    return {
        "norm_w": (1.0 + 0.02 * torch.randn(h, generator=gen, device=device)).to(torch.bfloat16),
        "router": (0.02 * torch.randn((e, h), generator=gen, device=device)).to(torch.bfloat16),
        "gate": quant_weights_torch(gen, e * i, h, 4, device, centre),
        "up": quant_weights_torch(gen, e * i, h, 4, device, centre),
        "down": quant_weights_torch(gen, e * h, i, 4, device, centre),
    }
