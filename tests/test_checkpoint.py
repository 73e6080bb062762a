"""MLX safetensors loading (molten_b200/checkpoint.py) on the CPU: single-file
and sharded checkpoints, the quantized-layer checks of load_quant
(lfm.rs:283-316) and malformed files."""
import json
import struct

import numpy as np
import pytest
import torch

from molten_b200 import checkpoint as ck
from molten_b200 import synth


def _q4(g, rows, k):
    codes, s, b = synth.quant_weights_np(g, rows, k, 4)
    return codes, s, b


def _moe_tensors(g, layer, e, h, inter, router_dtype="F32"):
    p = f"model.layers.{layer}"
    t = {f"{p}.ffn_norm.weight": ("BF16", synth.norm_weight_np(g, h))}
    router = g.normal(0, 0.02, (e, h)).astype(np.float32)
    t[f"{p}.feed_forward.gate.weight"] = (router_dtype, router if router_dtype == "F32"
                                          else synth.f32_to_bf16_bits(router))
    t[f"{p}.feed_forward.expert_bias"] = ("F32", g.normal(0, 0.1, e).astype(np.float32))
    for name, rows, k in (("gate_proj", e * inter, h), ("up_proj", e * inter, h),
                          ("down_proj", e * h, inter)):
        codes, s, b = _q4(g, rows, k)
        base = f"{p}.feed_forward.switch_mlp.{name}"
        # stacked experts as the checkpoint stores them: [E][rows/E][cols]
        t[f"{base}.weight"] = ("U32", codes.reshape(e, rows // e, -1))
        t[f"{base}.scales"] = ("BF16", s.reshape(e, rows // e, -1))
        t[f"{base}.biases"] = ("BF16", b.reshape(e, rows // e, -1))
    return t


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def test_single_file_moe_layer_round_trip(tmp_path):
    g = synth.rng(5)
    e, h, inter = 4, 256, 128
    t = _moe_tensors(g, 3, e, h, inter)
    ck.write_safetensors(tmp_path / ck.SINGLE_NAME, t, metadata={"format": "mlx"})
    c = ck.Checkpoint.open(tmp_path)
    assert set(c.names()) == set(t)
    L = ck.load_moe_layer(c, 3, e, h, inter, device="cpu")
    p = "model.layers.3.feed_forward"
    assert np.array_equal(_bits(L["norm_w"]), t["model.layers.3.ffn_norm.weight"][1])
    assert np.array_equal(_bits(L["router"]), t[f"{p}.gate.weight"][1])
    assert np.array_equal(_bits(L["expert_bias"]), t[f"{p}.expert_bias"][1])
    for name in ("gate", "up", "down"):
        w = L[name]
        base = f"{p}.switch_mlp.{name}_proj"
        rows = (e * inter) if name != "down" else (e * h)
        assert w.bits == 4 and w.group_size == 64 and w.out_features == rows
        assert w.in_features == (h if name != "down" else inter)
        assert np.array_equal(_bits(w.codes), t[f"{base}.weight"][1].reshape(rows, -1))
        assert np.array_equal(_bits(w.scales), t[f"{base}.scales"][1].reshape(rows, -1))
        assert np.array_equal(_bits(w.biases), t[f"{base}.biases"][1].reshape(rows, -1))


def test_sharded_index_and_bf16_router(tmp_path):
    g = synth.rng(6)
    t = _moe_tensors(g, 0, 4, 128, 64, router_dtype="BF16")
    names = sorted(t)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half],
              "model-00002-of-00002.safetensors": names[half:]}
    wm = {}
    for fname, ns in shards.items():
        ck.write_safetensors(tmp_path / fname, {n: t[n] for n in ns})
        wm.update({n: fname for n in ns})
    (tmp_path / ck.INDEX_NAME).write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    c = ck.Checkpoint.open(tmp_path)
    L = ck.load_moe_layer(c, 0, 4, 128, 64, device="cpu")
    assert L["router"].dtype == torch.bfloat16
    assert np.array_equal(_bits(L["router"]), t["model.layers.0.feed_forward.gate.weight"][1])
    assert c.meta("model.layers.0.ffn_norm.weight").shard.name in shards


def test_q6_head_and_bit_width_checks(tmp_path):
    g = synth.rng(7)
    codes, s, b = synth.quant_weights_np(g, 96, 2048, 6)
    t = {"model.embed_tokens.weight": ("U32", codes), "model.embed_tokens.scales": ("BF16", s),
         "model.embed_tokens.biases": ("BF16", b)}
    ck.write_safetensors(tmp_path / ck.SINGLE_NAME, t)
    c = ck.Checkpoint.open(tmp_path)
    w = ck.load_quant(c, "model.embed_tokens", 96, 2048, 6, device="cpu")
    assert w.bits == 6 and w.in_features == 2048
    assert np.array_equal(_bits(w.codes), codes)
    with pytest.raises(ValueError, match="expected 4-bit, found 6"):
        ck.load_quant(c, "model.embed_tokens", 96, 2048, 4, device="cpu")
    with pytest.raises(ValueError, match="rows 96 != 97"):
        ck.load_quant(c, "model.embed_tokens", 97, 2048, 6, device="cpu")
    with pytest.raises(ValueError, match="group count"):
        ck.load_quant(c, "model.embed_tokens", 96, 1024, 6, device="cpu")
    with pytest.raises(ValueError, match="missing model.nope.scales"):
        ck.load_quant(c, "model.nope", 96, 2048, 6, device="cpu")


def test_rejects_malformed_checkpoints(tmp_path):
    g = synth.rng(8)
    codes, s, b = _q4(g, 8, 128)
    good = {"w.weight": ("U32", codes), "w.scales": ("BF16", s), "w.biases": ("BF16", b)}

    d = tmp_path / "dtype"
    d.mkdir()
    ck.write_safetensors(d / ck.SINGLE_NAME, {**good, "w.weight": ("F32", codes.astype(np.float32))})
    with pytest.raises(ValueError, match="codes must be U32"):
        ck.load_quant(ck.Checkpoint.open(d), "w", 8, 128, 4, device="cpu")

    d = tmp_path / "dup"
    d.mkdir()
    ck.write_safetensors(d / "a.safetensors", good)
    ck.write_safetensors(d / "b.safetensors", {"w.scales": good["w.scales"]})
    (d / ck.INDEX_NAME).write_text(json.dumps({"weight_map": {"w.weight": "a.safetensors",
                                                               "w.scales": "b.safetensors"}}))
    with pytest.raises(ValueError, match="multiple shards"):
        ck.Checkpoint.open(d)

    d = tmp_path / "none"
    d.mkdir()
    with pytest.raises(ValueError, match="no model.safetensors.index.json"):
        ck.Checkpoint.open(d)

    def raw_file(path, header, data=b""):
        h = json.dumps(header).encode()
        path.write_bytes(struct.pack("<Q", len(h)) + h + data)

    d = tmp_path / "reversed"
    d.mkdir()
    raw_file(d / ck.SINGLE_NAME, {"x": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}},
             b"\0" * 4)
    with pytest.raises(ValueError, match="reversed"):
        ck.Checkpoint.open(d)

    d = tmp_path / "truncated"
    d.mkdir()
    raw_file(d / ck.SINGLE_NAME, {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}},
             b"\0" * 8)
    with pytest.raises(ValueError, match="past the end"):
        ck.Checkpoint.open(d)

    d = tmp_path / "size"
    d.mkdir()
    raw_file(d / ck.SINGLE_NAME, {"x": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}},
             b"\0" * 16)
    with pytest.raises(ValueError, match="16 bytes for shape"):
        ck.Checkpoint.open(d)

    d = tmp_path / "other"
    d.mkdir()
    raw_file(d / ck.SINGLE_NAME, {"x": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]},
                                  "__metadata__": {"k": "v"}}, b"\0" * 4)
    c = ck.Checkpoint.open(d)
    assert list(c.names()) == ["x"]
    with pytest.raises(ValueError, match="unsupported dtype F16"):
        c.read("x")


def test_missing_expert_bias_is_an_error(tmp_path):
    """The reference requires feed_forward.expert_bias (lfm.rs:359): a layer
    without it fails to load unless the caller opts out for bias-free routing."""
    g = synth.rng(8)
    t = _moe_tensors(g, 1, 4, 128, 64)
    del t["model.layers.1.feed_forward.expert_bias"]
    ck.write_safetensors(tmp_path / ck.SINGLE_NAME, t)
    c = ck.Checkpoint.open(tmp_path)
    with pytest.raises(ValueError, match="missing model.layers.1.feed_forward.expert_bias"):
        ck.load_moe_layer(c, 1, 4, 128, 64, device="cpu")
    L = ck.load_moe_layer(c, 1, 4, 128, 64, device="cpu", allow_missing_bias=True)
    assert L["expert_bias"] is None
