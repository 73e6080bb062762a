"""MLX safetensors checkpoints for the quantized MoE path: the shard / index
reader (Checkpoint, safetensors.rs:1-160), load_tensor (lfm.rs:261-281) and
load_quant (lfm.rs:283-316), so real weights can replace the synthetic ones at
the same layout (QuantWeights: codes U32 [rows][K*bits/32], scales and biases
BF16 [rows][K/64]).

Format. A shard is an 8-byte little-endian header length, a JSON header that
maps each tensor name to {dtype, shape, data_offsets: [start, end)} relative
to the data section right after the header (an optional "__metadata__" object
is not a tensor), then the data section. A checkpoint directory holds either
model.safetensors.index.json, whose weight_map names each tensor's shard, or
one model.safetensors.

Errors are ValueError (the reference's `ensure!` / `bail!`), raised before
anything is read to the device. Beyond the reference's checks, every tensor's
byte range must lie inside its shard and match its shape and dtype.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .quant import QuantWeights

INDEX_NAME = "model.safetensors.index.json"
SINGLE_NAME = "model.safetensors"

# dtypes the path loads (safetensors.rs:19-45); others stay listed but cannot be read
_DTYPES = {"BF16": (np.uint16, 2), "F32": (np.float32, 4), "U32": (np.uint32, 4)}
_TORCH = {"BF16": (torch.int16, torch.bfloat16), "F32": (torch.float32, torch.float32),
          "U32": (torch.int32, torch.int32)}


def _ensure(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


@dataclass(frozen=True)
class TensorMeta:
    """Where one tensor lives: its shard and absolute byte range."""

    dtype: str
    shape: tuple
    shard: Path
    start: int
    end: int

    @property
    def byte_len(self) -> int:
        return self.end - self.start

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


def parse_shard_header(path: Path) -> dict[str, TensorMeta]:
    """One shard's tensors (safetensors.rs:128-160)."""
    path = Path(path)
    size = path.stat().st_size
    with open(path, "rb") as f:
        head = f.read(8)
        _ensure(len(head) == 8, f"{path}: no header length")
        (hlen,) = struct.unpack("<Q", head)
        _ensure(8 + hlen <= size, f"{path}: header length {hlen} past the end of the file")
        raw = json.loads(f.read(hlen))
    _ensure(isinstance(raw, dict), f"{path}: header is not a JSON object")
    data = 8 + hlen
    out: dict[str, TensorMeta] = {}
    for name, entry in raw.items():
        if name == "__metadata__":
            continue
        try:
            dtype, shape = str(entry["dtype"]), tuple(int(d) for d in entry["shape"])
            start, end = (int(v) for v in entry["data_offsets"])
        except (KeyError, TypeError, ValueError) as e:
            raise ValueError(f"{path}: bad header entry for {name}: {e}") from None
        _ensure(end >= start, f"tensor {name} has reversed data offsets")
        _ensure(data + end <= size, f"tensor {name} ends past the end of {path}")
        meta = TensorMeta(dtype, shape, path, data + start, data + end)
        if dtype in _DTYPES:
            _ensure(meta.byte_len == meta.numel * _DTYPES[dtype][1],
                    f"tensor {name}: {meta.byte_len} bytes for shape {shape} of {dtype}")
        out[name] = meta
    return out


class Checkpoint:
    """A checkpoint directory: every tensor name mapped to its location."""

    def __init__(self, tensors: dict[str, TensorMeta]):
        self.tensors = tensors

    @classmethod
    def open(cls, directory) -> "Checkpoint":
        """Via model.safetensors.index.json when present, else one
        model.safetensors (safetensors.rs:84-117)."""
        d = Path(directory)
        index = d / INDEX_NAME
        if index.exists():
            wm = json.loads(index.read_text()).get("weight_map", {})
            _ensure(isinstance(wm, dict), f"{index}: weight_map is not an object")
            shards = [d / n for n in sorted(set(wm.values()))]
        else:
            single = d / SINGLE_NAME
            _ensure(single.exists(), f"no {INDEX_NAME} or {SINGLE_NAME} under {d}")
            shards = [single]
        tensors: dict[str, TensorMeta] = {}
        for shard in shards:
            for name, meta in parse_shard_header(shard).items():
                _ensure(name not in tensors, f"tensor {name} appears in multiple shards")
                tensors[name] = meta
        return cls(tensors)

    def names(self):
        return self.tensors.keys()

    def meta(self, name: str) -> TensorMeta | None:
        return self.tensors.get(name)

    def read(self, name: str) -> np.ndarray:
        """The tensor's values on the host (BF16 as uint16 bit patterns)."""
        meta = self.tensors.get(name)
        _ensure(meta is not None, f"tensor {name} not in checkpoint")
        _ensure(meta.dtype in _DTYPES, f"tensor {name} has unsupported dtype {meta.dtype}")
        npdt, _ = _DTYPES[meta.dtype]
        with open(meta.shard, "rb") as f:
            f.seek(meta.start)
            buf = f.read(meta.byte_len)
        _ensure(len(buf) == meta.byte_len, f"short read of {name}")
        return np.frombuffer(bytearray(buf), dtype=npdt).reshape(meta.shape)


def load_tensor(ckpt: Checkpoint, name: str, device="cuda") -> torch.Tensor:
    """load_tensor (lfm.rs:261-281): BF16 -> torch.bfloat16, F32 -> float32,
    U32 -> int32 holding the u32 bit patterns."""
    meta = ckpt.meta(name)
    _ensure(meta is not None, f"tensor {name} not in checkpoint")
    _ensure(meta.dtype in _TORCH, f"unsupported dtype {meta.dtype} for {name}")
    store, view = _TORCH[meta.dtype]
    host = ckpt.read(name)
    t = torch.from_numpy(np.ascontiguousarray(host).view(
        {torch.int16: np.int16, torch.float32: np.float32, torch.int32: np.int32}[store]))
    return t.view(view).to(device)


def load_quant(ckpt: Checkpoint, base: str, expected_rows: int, expected_k: int,
               expected_bits: int, device="cuda") -> QuantWeights:
    """load_quant (lfm.rs:283-316): `{base}.weight` (U32 codes), `.scales` and
    `.biases` (BF16), group 64; rows counted over every leading dimension, so
    stacked experts [E][rows][cols] load as one [E*rows][cols] matrix."""
    wname, sname, bname = f"{base}.weight", f"{base}.scales", f"{base}.biases"
    smeta, bmeta, wmeta = ckpt.meta(sname), ckpt.meta(bname), ckpt.meta(wname)
    _ensure(smeta is not None, f"missing {sname}")
    _ensure(bmeta is not None, f"missing {bname}")
    _ensure(wmeta is not None, f"missing {wname}")
    _ensure(wmeta.dtype == "U32", f"{base} codes must be U32")
    _ensure(len(wmeta.shape) > 0 and wmeta.shape[-1] > 0, f"{base}: empty shape")
    cols = wmeta.shape[-1]
    groups = expected_k // 64
    _ensure(expected_k % 64 == 0 and len(smeta.shape) > 0 and smeta.shape[-1] == groups,
            f"{base}: scales group count mismatch")
    _ensure((32 * cols) % expected_k == 0, f"{base}: {cols} code words do not pack K={expected_k}")
    bits = 32 * cols // expected_k
    _ensure(bits == expected_bits, f"{base}: expected {expected_bits}-bit, found {bits}")
    rows = wmeta.numel // cols
    _ensure(rows == expected_rows, f"{base}: rows {rows} != {expected_rows}")
    _ensure(smeta.numel // groups == rows and bmeta.numel // groups == rows,
            f"{base}: scale rows mismatch")
    _ensure(smeta.dtype == "BF16" and bmeta.dtype == "BF16", f"{base}: scales dtype")
    codes = load_tensor(ckpt, wname, device).reshape(rows, cols)
    scales = load_tensor(ckpt, sname, device).reshape(rows, groups)
    biases = load_tensor(ckpt, bname, device).reshape(rows, groups)
    return QuantWeights(codes, scales, biases, 64, bits)


def load_moe_layer(ckpt: Checkpoint, layer: int, n_experts: int = 64, hidden: int = 2048,
                   inter: int = 1536, device="cuda", allow_missing_bias: bool = False) -> dict:
    """One MoE layer's tensors under the reference's names (lfm.rs:326-366):
    ffn_norm, the router (`feed_forward.gate.weight`, [E][H], F32 or BF16),
    `expert_bias` and the stacked Q4 experts
    `feed_forward.switch_mlp.{gate,up,down}_proj`. The reference requires
    `expert_bias` (lfm.rs:359; its sigmoid routing selects on it), so a layer
    without it is an error unless `allow_missing_bias` (then "expert_bias" is
    None, for the BASELINE softmax routing, which has no bias)."""
    p = f"model.layers.{layer}"
    moe = f"{p}.feed_forward"
    norm = load_tensor(ckpt, f"{p}.ffn_norm.weight", device)
    _ensure(norm.numel() == hidden, f"{p}: ffn_norm shape")
    router = load_tensor(ckpt, f"{moe}.gate.weight", device)
    _ensure(router.numel() == n_experts * hidden, f"{moe}: router shape")
    bias = None
    if ckpt.meta(f"{moe}.expert_bias") is not None:
        bias = load_tensor(ckpt, f"{moe}.expert_bias", device)
        _ensure(bias.numel() == n_experts, f"{moe}: expert_bias shape")
        bias = bias.reshape(n_experts)
    else:
        _ensure(allow_missing_bias, f"missing {moe}.expert_bias")
    return {
        "norm_w": norm.reshape(hidden),
        "router": router.reshape(n_experts, hidden),
        "expert_bias": bias,
        "gate": load_quant(ckpt, f"{moe}.switch_mlp.gate_proj", n_experts * inter, hidden, 4,
                           device),
        "up": load_quant(ckpt, f"{moe}.switch_mlp.up_proj", n_experts * inter, hidden, 4, device),
        "down": load_quant(ckpt, f"{moe}.switch_mlp.down_proj", n_experts * hidden, inter, 4,
                           device),
    }


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Writes one shard. tensors: name -> (dtype, numpy array of its bits:
    uint16 for BF16, float32 for F32, uint32 for U32)."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs, off = [], 0
    for name in sorted(tensors):
        dtype, arr = tensors[name]
        _ensure(dtype in _DTYPES, f"cannot write dtype {dtype}")
        b = np.ascontiguousarray(arr, dtype=_DTYPES[dtype][0]).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(arr)),
                        "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
