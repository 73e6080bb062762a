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


def bf16_err_stats(got_bits, want_bits) -> dict:
    """How far bf16 outputs are from the oracle's: share bit-identical, the
    largest distance in bf16 ulps (of max(|want|, 1e-2 rms)), the largest relative error
    over outputs with |want| >= 1e-2 rms(want) (below that the value is a
    near-cancellation, whose relative error no summation order controls),
    and the largest absolute error as a fraction of rms(want)."""
    g = synth.bf16_bits_to_f32(np.asarray(got_bits)).astype(np.float64).ravel()
    w = synth.bf16_bits_to_f32(np.asarray(want_bits)).astype(np.float64).ravel()
    if w.size == 0:
        return {"n": 0}
    rms = float(np.sqrt(np.mean(w ** 2)))
    err = np.abs(g - w)
    # ulps of max(|want|, 1e-2 rms): an exact zero has no ulp of its own
    e = np.floor(np.log2(np.maximum(np.abs(w), max(1e-2 * rms, 2.0 ** -126))))
    ulps = err / 2.0 ** (e - 7)
    big = np.abs(w) >= 1e-2 * rms
    return {"n": int(w.size),
            "bit_identical": float(np.mean(np.asarray(got_bits).ravel() ==
                                           np.asarray(want_bits).ravel())),
            "max_ulps": float(ulps.max()),
            "max_rel_err": float((err[big] / np.abs(w[big])).max()) if big.any() else 0.0,
            "max_abs_err_over_rms": float(err.max() / rms) if rms else 0.0}


def record_stats(name: str, stats: dict) -> None:
    """Prints the stats (pytest -s) and appends them to $MC_ERR_STATS (a
    JSON-lines file) when that is set."""
    import json
    import os
    line = json.dumps({"case": name, **stats})
    print(line)
    path = os.environ.get("MC_ERR_STATS")
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")
