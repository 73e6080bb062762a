"""The sampling draw's CPU restatement (oracle/, test infrastructure) on the
CPU: Philox4x32-10 against the known-answer vectors its authors publish
(Random123 kat_vectors), the log and Gumbel transforms against float64
mathematics, and the draw's kept set and distribution against a float64
statement of the contract (docs/PROTOCOL.md:48-75): top-k ties kept, the
smallest top-p prefix with its boundary tie group, repetition penalty,
Gumbel-max frequencies matching softmax."""
import math

import numpy as np
import pytest

import oracle
from molten_b200 import synth
from molten_b200.sample import Sampling


@pytest.mark.parametrize("counter,key,want", [
    ((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff,) * 4, (0xffffffff, 0xffffffff), (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
])
def test_philox_known_answers(counter, key, want):
    assert oracle.philox4x32_10(counter, key) == list(want)


def test_log_within_two_ulps():
    xs = np.exp(np.linspace(-87.0, 88.0, 4001)).astype(np.float32)
    xs = np.concatenate([xs, np.float32([1e-40, 1e-45, 0.70710677, 0.70710683, 1.4142135,
                                         1.4142137, 1.0, 2.0, 3.4e38])])
    for x in xs:
        got = np.float32(oracle.log(float(x)))
        want = math.log(float(x))
        ulp = np.spacing(np.float32(abs(want))) if want != 0 else np.float32(1e-45)
        assert abs(float(got) - want) <= 2 * float(ulp), (x, got, want)
    assert oracle.log(0.0) == -math.inf
    assert math.isnan(oracle.log(-1.0))


def test_gumbel_transform():
    # decreasing in the word (G = -log(-log(1 - V))), the largest words
    # clamped at 1 - V = 2^-25; the variates have the Gumbel mean and variance
    words = [0, 1, 1000, 1 << 20, 1 << 26, 1 << 30, 1 << 31, 0xfffffff0, 0xffffffff]
    vals = [oracle.gumbel(w) for w in words]
    assert all(a > b for a, b in zip(vals[:-2], vals[1:-1])) and vals[-1] == vals[-2]
    g = synth.rng(12)
    sample = np.array([oracle.gumbel(int(w)) for w in g.integers(0, 2**32, 20000)])
    assert abs(sample.mean() - 0.5772156649) < 0.03
    assert abs(sample.var() - math.pi ** 2 / 6) < 0.08


def _w(logits_bits, temperature=1.0, seen=None, penalty=1.0):
    v = synth.bf16_bits_to_f32(logits_bits).astype(np.float32)
    inv_t, inv_p = np.float32(1.0) / np.float32(temperature), np.float32(1.0) / np.float32(penalty)
    if seen is not None:
        mark = np.array([(seen[i >> 5] >> (i & 31)) & 1 for i in range(v.size)], bool)
        v = np.where(mark & (v > 0), v * inv_p, np.where(mark, v * np.float32(penalty), v))
    return (v * inv_t).astype(np.float32)


def _kept_f64(w, top_k, top_p):
    """The kept set by the contract, in float64: ids with w >= tau."""
    order = np.argsort(-w.astype(np.float64), kind="stable")
    tau = -np.inf
    if top_k and top_k < w.size:
        tau = w[order[top_k - 1]]
    if top_p < 1.0:
        keep = w >= tau
        e = np.exp(w.astype(np.float64) - w.max())
        z = e[keep].sum()
        vals = np.unique(w[keep])[::-1]
        cum = 0.0
        for v in vals:
            cum += e[w == v].sum()
            if cum >= top_p * z:
                tau = v
                break
    return set(np.nonzero(w >= tau)[0].tolist())


def _token(key):
    return (~key) & 0xffffffff


@pytest.mark.parametrize("top_k,top_p", [(1, 1.0), (5, 1.0), (0, 0.3), (0, 0.9), (20, 0.6),
                                         (0, 1e-7)])
def test_kept_set_matches_the_contract(top_k, top_p):
    g = synth.rng(40 + top_k)
    V = 4096
    logits = synth.f32_to_bf16_bits(g.normal(0, 2.5, V).astype(np.float32))
    w = _w(logits, 0.9)
    kept = _kept_f64(w, top_k, top_p)
    seen_tokens = set()
    for pos in range(60):
        key, tau = oracle.sample_draw(logits, temperature=0.9, top_k=top_k, top_p=top_p,
                                      seed=77, pos=pos)
        tok = _token(key)
        assert tok in kept
        seen_tokens.add(tok)
        # the oracle's threshold keeps exactly the contract's set
        got_kept = set(np.nonzero(w >= _kfloat(tau))[0].tolist())
        assert got_kept == kept
    if len(kept) > 1:
        assert len(seen_tokens) > 1, "different positions draw different tokens"


def _kfloat(k):
    u = np.uint32(k & 0x7fffffff) if k & 0x80000000 else np.uint32(~k & 0xffffffff)
    return np.float32(u.view(np.float32)) if k else -np.inf


def test_top_k_keeps_the_whole_tie_group():
    V = 64
    vals = np.zeros(V, np.float32) - 5.0
    vals[[3, 9, 17, 40]] = 2.0     # four tokens tie for the 2nd..5th place
    vals[11] = 3.0
    logits = synth.f32_to_bf16_bits(vals)
    drawn = set()
    for pos in range(400):
        key, _ = oracle.sample_draw(logits, top_k=2, seed=9, pos=pos)
        drawn.add(_token(key))
    assert drawn == {3, 9, 11, 17, 40}


def test_top_p_boundary():
    # probabilities 0.5, 0.3, 0.2 (temperature 1): top_p 0.79 keeps two tokens,
    # 0.81 keeps all three
    vals = np.full(8, -60.0, np.float32)
    vals[[1, 4, 6]] = np.log([0.5, 0.3, 0.2]).astype(np.float32)
    logits = synth.f32_to_bf16_bits(vals)
    for top_p, want in ((0.79, {1, 4}), (0.81, {1, 4, 6})):
        drawn = {_token(oracle.sample_draw(logits, top_p=top_p, seed=3, pos=p)[0])
                 for p in range(300)}
        assert drawn == want, (top_p, drawn)


def test_repetition_penalty_changes_the_winner():
    vals = np.full(32, -30.0, np.float32)
    vals[5], vals[7] = 4.0, 3.0
    logits = synth.f32_to_bf16_bits(vals)
    seen = np.zeros(1, np.uint32)
    seen[0] |= 1 << 5                       # token 5 already in the sequence
    key, _ = oracle.sample_draw(logits, top_k=1, seed=1, pos=0)
    assert _token(key) == 5
    key, _ = oracle.sample_draw(logits, seen=seen, top_k=1, penalty=2.0, seed=1, pos=0)
    assert _token(key) == 7                 # 4 / 2 < 3


def test_draw_frequencies_follow_softmax():
    vals = np.float32([2.0, 1.0, 0.5, 0.0, -0.5, -1.0, 1.5, 0.25])
    logits = synth.f32_to_bf16_bits(vals)
    n = 12000
    counts = np.zeros(vals.size)
    for pos in range(n):
        counts[_token(oracle.sample_draw(logits, temperature=1.0, seed=2024, pos=pos)[0])] += 1
    p = np.exp(vals.astype(np.float64))
    p /= p.sum()
    sd = np.sqrt(n * p * (1 - p))
    assert np.all(np.abs(counts - n * p) < 4.5 * sd), (counts, n * p)


def test_sampling_request_validation():
    assert Sampling.from_request(None, 65536) is None
    assert Sampling.from_request({"temperature": 0}, 65536) is None
    assert Sampling.from_request({"top_k": 70000}, 65536).top_k == 0
    for bad in ({"top_p": 0.0}, {"temperature": 1e-9}, {"repetition_penalty": 0.0},
                {"seed": -1}, {"foo": 1}, {"top_k": 1.5}):
        with pytest.raises(ValueError):
            Sampling.from_request(bad, 65536)
