"""Random sampling of the decode step (lfm/sample.rs mirrored over the C ABI).

``Sampling`` holds one request's validated parameters
(lfm/sample.rs:87-170: temperature 0 or >= 1e-6, top_k >= 0 with k >= vocab
meaning off, top_p in (0, 1], repetition_penalty in [1e-6, 1e6], a 64-bit
seed; absent / null / temperature 0 means greedy). ``SampleScratch`` owns the
device buffers of the draw -- the workspace (zeroed once, left zero by every
call) and the sequence's seen-token bitmap -- and encodes the draw of one
token into the zeroed 64-bit argmax key that ``lfm.token_tail`` reads, as
``SampleScratch::encode_draw`` does (lfm/sample.rs:248-338). Tokens never
leave the device between steps.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from .lfm import Context, _p, ensure

MIN_TEMPERATURE = 1e-6
PENALTY_RANGE = (1e-6, 1e6)
_FIELDS = {"temperature", "top_k", "top_p", "repetition_penalty", "seed"}


@dataclass(frozen=True)
class Sampling:
    temperature: float = 1.0
    top_k: int = 0            # 0 = off (values >= the vocabulary are off too)
    top_p: float = 1.0        # 1 = off
    repetition_penalty: float = 1.0
    seed: int = 0

    @staticmethod
    def from_request(value, vocab: int) -> "Sampling | None":
        """Parses a request's ``sampling`` object; None means greedy decoding."""
        if value is None:
            return None
        ensure(isinstance(value, dict), "generate.sampling must be an object")
        for k in value:
            ensure(k in _FIELDS, f"unknown sampling field {k!r}")

        def number(key, default):
            x = value.get(key, default)
            ensure(isinstance(x, (int, float)) and not isinstance(x, bool),
                   f"sampling.{key} must be a number")
            ensure(math.isfinite(x), f"sampling.{key} must be finite")
            return float(x)

        temperature = number("temperature", 1.0)
        ensure(temperature >= 0.0, "sampling.temperature must be >= 0")
        top_p = number("top_p", 1.0)
        ensure(0.0 < top_p <= 1.0, "sampling.top_p must be in (0, 1]")
        pen = number("repetition_penalty", 1.0)
        ensure(PENALTY_RANGE[0] <= pen <= PENALTY_RANGE[1],
               f"sampling.repetition_penalty must be in [{PENALTY_RANGE[0]}, {PENALTY_RANGE[1]}]")
        top_k = value.get("top_k", 0)
        ensure(isinstance(top_k, int) and not isinstance(top_k, bool) and top_k >= 0,
               "sampling.top_k must be a non-negative integer")
        seed = value.get("seed", 0)
        ensure(isinstance(seed, int) and not isinstance(seed, bool) and 0 <= seed < 2 ** 64,
               "sampling.seed must be an integer in [0, 2^64)")
        if temperature == 0.0:
            return None
        ensure(temperature >= MIN_TEMPERATURE,
               f"sampling.temperature must be 0 (greedy) or at least {MIN_TEMPERATURE}")
        return Sampling(temperature, 0 if top_k >= vocab else top_k, top_p, pen, seed)

    def uses_penalty(self) -> bool:
        return self.repetition_penalty != 1.0

    def c(self) -> _lib.Sampling:
        return _lib.Sampling(self.temperature, self.top_k, self.top_p, self.repetition_penalty,
                             self.seed)


class SampleScratch:
    """Device buffers of the sampled step for one sequence."""

    def __init__(self, ctx: Context, vocab: int, device=None):
        ensure(vocab % 4 == 0 and vocab >= 4, "vocab must be a multiple of 4")
        dev = device or ctx.device
        self.ctx, self.vocab = ctx, vocab
        n = int(_lib.lib().mc_sample_workspace_bytes(vocab))
        self.ws = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.seen = torch.zeros((vocab + 31) // 32, dtype=torch.int32, device=dev)

    def upload_seen(self, tokens) -> None:
        """Sets the seen set to the given token ids (the sequence so far)."""
        import numpy as np
        bits = np.zeros(self.seen.numel(), np.uint32)
        for t in tokens:
            t = int(t)
            if 0 <= t < self.vocab:
                bits[t // 32] |= np.uint32(1 << (t % 32))
        self.seen.copy_(torch.from_numpy(bits.view(np.int32)))

    def encode_draw(self, logits: torch.Tensor, best: torch.Tensor, s: Sampling,
                    pos: int | torch.Tensor) -> None:
        """Draws the token at absolute position ``pos`` from bf16 ``logits``
        [vocab] into ``best`` (int64 [1], zero on entry). ``pos`` may be a
        device int32 [1] tensor (read on the device: a captured step draws at
        the position ``encode_mark`` advanced)."""
        ensure(logits.numel() == self.vocab and logits.dtype == torch.bfloat16,
               "sampling logits row")
        ensure(best.dtype == torch.int64 and best.numel() >= 1, "sampling key")
        dev_pos = isinstance(pos, torch.Tensor)
        ensure(dev_pos or 0 <= pos < 2 ** 32, "position exceeds u32")
        sp = s.c()
        _lib.call("mc_sample_draw", self.ctx.handle, _p(logits), self.vocab,
                  _p(self.seen) if s.uses_penalty() else None, _lib.C.byref(sp),
                  0 if dev_pos else pos, _p(pos) if dev_pos else None, _p(best),
                  _p(self.ws), self.ws.numel())

    def encode_mark(self, tok: torch.Tensor, pos: torch.Tensor | None = None) -> None:
        """After the token tail wrote ``tok`` (int32 [1]): adds it to the seen
        set, and advances the device position ``pos`` (int32 [1]) when given."""
        ensure(tok.numel() == 1 and tok.dtype == torch.int32, "sampled token slot")
        _lib.call("mc_sample_mark", self.ctx.handle, _p(tok), _p(self.seen), self.vocab, _p(pos))
