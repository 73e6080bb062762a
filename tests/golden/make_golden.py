"""Writes the golden fixtures in tests/golden/*.npz from the CPU oracle.

The reference (Rust + Metal) cannot run on this machine and has no fixtures
of its own, so these vectors come from the oracle on seeded inputs; they pin
the oracle's (and through the GPU tests, the kernels') behaviour against
regressions. Small cases store their inputs; larger ones store the seed plus a
SHA-256 of the regenerated inputs, so a change of numpy's generator is
reported as such rather than as a parity failure.

Usage: python -m tests.golden.make_golden
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

import oracle
from molten_b200 import synth

HERE = Path(__file__).resolve().parent


def path(name: str) -> Path:
    return HERE / f"{name}.npz"


def _sha(*arrays) -> np.ndarray:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), np.uint8).copy()


def q4_gemv(inputs_only=False, data=None):
    if data is None:
        g = synth.rng(101)
        codes, s, b = synth.quant_weights_np(g, 32, 2048, 4)
        x = synth.activations_np(g, 2, 2048)
        d = dict(codes=codes, scales=s, biases=b, x=x)
    else:
        d = {k: data[k] for k in ("codes", "scales", "biases", "x")}
    if inputs_only:
        return d
    y, acc = oracle.gemv_quant(d["codes"], d["scales"], d["biases"], 4, d["x"], with_acc=True)
    out = dict(y=y, acc=acc)
    return out if data is not None else {**d, **out}


def q6_head(inputs_only=False, data=None):
    if data is None:
        g = synth.rng(102)
        codes, s, b = synth.quant_weights_np(g, 64, 2048, 6)
        x = synth.activations_np(g, 2048)
        d = dict(codes=codes, scales=s, biases=b, x=x)
    else:
        d = {k: data[k] for k in ("codes", "scales", "biases", "x")}
    if inputs_only:
        return d
    y = oracle.gemv_quant(d["codes"], d["scales"], d["biases"], 6, d["x"])
    key, tok = oracle.head_argmax(d["codes"], d["scales"], d["biases"], 6, d["x"])
    out = dict(y=y, key=key, tok=tok)
    return out if data is not None else {**d, **out}


def router(inputs_only=False, data=None):
    if data is None:
        g = synth.rng(103)
        d = dict(h=synth.activations_np(g, 2, 2048), b=synth.activations_np(g, 2, 2048),
                 norm_w=synth.norm_weight_np(g), w=synth.router_np(g),
                 ebias=g.normal(0, 0.1, 64).astype(np.float32))
    else:
        d = {k: data[k] for k in ("h", "b", "norm_w", "w", "ebias")}
    if inputs_only:
        return d
    out = {}
    for mode in (0, 1):
        hout, normed, logits, ids, wts = oracle.router_addnorm_route(
            d["h"], d["b"], d["norm_w"], d["w"], 0, d["ebias"], mode)
        out.update({f"hout{mode}": hout, f"normed{mode}": normed, f"logits{mode}": logits,
                    f"ids{mode}": ids, f"wts{mode}": wts})
    return out if data is not None else {**d, **out}


def _layer_inputs(seed, E, I):
    g = synth.rng(seed)
    gate = synth.quant_weights_np(g, E * I, 2048)
    up = synth.quant_weights_np(g, E * I, 2048)
    down = synth.quant_weights_np(g, E * 2048, I)
    x = synth.activations_np(g, 2, 2048)
    ids = np.stack([g.permutation(E)[:4] for _ in range(2)]).astype(np.uint32)
    wts = synth.f32_to_bf16_bits(g.dirichlet(np.ones(4), 2).astype(np.float32))
    return gate, up, down, x, ids, wts


def decode_experts(inputs_only=False, data=None):
    """gate/up/act + down/combine with 8 experts of width 128 (seed-regenerated)."""
    E, I = 8, 128
    gate, up, down, x, ids, wts = _layer_inputs(104, E, I)
    sha = _sha(*gate, *up, *down, x, ids, wts)
    if data is not None:
        assert np.array_equal(sha, data["sha"]), "generator changed: regenerate fixtures"
    if inputs_only:
        return dict(gate=gate, up=up, down=down, x=x, ids=ids, wts=wts, E=E, I=I)
    # oracle's gemv_gather_act wrapper assumes E=64 stacking; call the C entry directly
    act = np.zeros((2, 4, I), np.uint16)
    L = oracle.lib()
    P = oracle._ptr
    L.or_gemv_gather_act(P(gate[0]), P(gate[1]), P(gate[2]), P(up[0]), P(up[1]), P(up[2]), I,
                         2048, P(x), P(ids), 2, P(act))
    out = oracle.gemv_gather_down_combine4(down, act, ids, wts, n_experts=E)
    res = dict(act=act, out=out)
    return res if data is not None else {"sha": sha, **res}


def prefill(inputs_only=False, data=None):
    E, I, m = 8, 128, 48
    g = synth.rng(105)
    x = synth.activations_np(g, m, 2048)
    logits = synth.zipf_logits_np(g, m, E)
    gate = synth.quant_weights_np(g, E * I, 2048)
    up = synth.quant_weights_np(g, E * I, 2048)
    down = synth.quant_weights_np(g, E * 2048, I)
    sha = _sha(x, logits, *gate, *up, *down)
    if data is not None:
        assert np.array_equal(sha, data["sha"]), "generator changed: regenerate fixtures"
    if inputs_only:
        return dict(x=x, logits=logits, gate=gate, up=up, down=down, E=E, I=I, m=m)
    r = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
    r.pop("ed")  # large and implied by act; keeps the fixture small
    return r if data is not None else {"sha": sha, **r}


CASES = {"q4_gemv": q4_gemv, "q6_head": q6_head, "router": router,
         "decode_experts": decode_experts, "prefill": prefill}


def main():
    for name, fn in CASES.items():
        d = fn()
        np.savez_compressed(path(name), **d)
        print(name, path(name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
