"""CPU checks of the oracle itself (test infrastructure): known answers that can
be computed by hand or by an independent float64 numpy restatement, the
selection/tie rules the reference documents, and the committed fixtures.

The reference ships no tests or golden vectors for this path and cannot run
here (Rust + Metal), so these known answers are what pins the oracle."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import synth

G = synth.rng


def dequant_f64(codes, s, b, bits, k):
    """Independent restatement of MLX affine dequant (weights.rs:7-20;
    lfm.metal:185-199 for the 6-bit packing) in float64."""
    n = codes.shape[0]
    if bits == 4:
        q = np.zeros((n, k), np.float64)
        for j in range(8):
            q[:, j::8] = (codes >> (4 * j)) & 15
    else:
        by = codes.view(np.uint8).reshape(n, -1)
        b0, b1, b2 = by[:, 0::3].astype(np.int64), by[:, 1::3].astype(np.int64), by[:, 2::3].astype(np.int64)
        q = np.zeros((n, k), np.float64)
        q[:, 0::4] = b0 & 0x3F
        q[:, 1::4] = ((b0 >> 6) & 3) | ((b1 & 0x0F) << 2)
        q[:, 2::4] = ((b1 >> 4) & 0x0F) | ((b2 & 3) << 4)
        q[:, 3::4] = (b2 >> 2) & 0x3F
    sf = np.repeat(synth.bf16_bits_to_f32(s).astype(np.float64), 64, axis=1)
    bf = np.repeat(synth.bf16_bits_to_f32(b).astype(np.float64), 64, axis=1)
    return sf * q + bf


def f32(bits):
    return synth.bf16_bits_to_f32(bits)


def test_exp_within_one_ulp():
    xs = np.linspace(-87.0, 88.5, 40001).astype(np.float32)
    for x in xs[::13]:
        a = np.float32(oracle.exp(float(x)))
        ref = np.exp(np.float64(x))
        assert abs(float(a) - ref) <= 1.0 * float(np.spacing(np.float32(ref))), x
    assert oracle.exp(0.0) == 1.0
    assert oracle.exp(100.0) == float("inf")
    assert oracle.exp(-110.0) == 0.0


def test_bf16_rounding_matches_torch():
    g = G(1)
    v = np.concatenate([g.normal(0, 10, 20000).astype(np.float32),
                        # exact ties between two bf16 values
                        (np.arange(1, 2000, dtype=np.uint32) << 16 | 0x8000).view(np.float32)])
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = np.array([oracle.f32_to_bf16(float(x)) for x in v], np.uint16)
    assert np.array_equal(got, ref)
    assert np.array_equal(synth.f32_to_bf16_bits(v), ref)


@pytest.mark.parametrize("bits", [4, 6])
def test_gemv_matches_float64_dequant(bits):
    g = G(2)
    n, k = 96, 2048
    codes, s, b = synth.quant_weights_np(g, n, k, bits)
    x = synth.activations_np(g, k)
    y, acc = oracle.gemv_quant(codes, s, b, bits, x, with_acc=True)
    ref = dequant_f64(codes, s, b, bits, k) @ f32(x).astype(np.float64)
    np.testing.assert_allclose(acc[0], ref, rtol=1e-4, atol=1e-4)
    assert np.array_equal(y[0], synth.f32_to_bf16_bits(acc[0]))


def test_gemv_all_zero_codes_is_bias_times_sum():
    """All-zero codes: y = sum_g b_g * sum(x over g), exactly in canonical order
    (one group per lane at K=2048, then the 32-lane butterfly)."""
    g = G(3)
    k = 2048
    _, s, b = synth.quant_weights_np(g, 4, k, 4)
    codes = np.zeros((4, k // 8), np.uint32)
    x = synth.activations_np(g, k)
    _, acc = oracle.gemv_quant(codes, s, b, 4, x, with_acc=True)
    xf = f32(x).reshape(32, 64)
    xg = np.zeros(32, np.float32)
    for grp in range(32):
        t = xf[grp, 0]
        for i in range(1, 64):
            t = np.float32(t + xf[grp, i])
        xg[grp] = t
    for r in range(4):
        lane = (np.float32(0) + f32(b[r]) * xg).astype(np.float32)
        for m in (16, 8, 4, 2, 1):
            lane = (lane + lane[np.arange(32) ^ m]).astype(np.float32)
        assert acc[0, r] == lane[0]


def test_gemv_single_nibble_and_saturated_rows():
    g = G(4)
    k = 2048
    _, s, b = synth.quant_weights_np(g, 2, k, 4)
    b[:] = 0  # bias 0 so only the code term remains
    x = synth.activations_np(g, k)
    codes = np.zeros((2, k // 8), np.uint32)
    codes[0, 37] = 9 << (4 * 5)              # code k = 37*8 + 5 = 301, q = 9
    codes[1, :] = 0xFFFFFFFF                 # q = 15 everywhere
    _, acc = oracle.gemv_quant(codes, s, b, 4, x, with_acc=True)
    kk = 37 * 8 + 5
    assert acc[0, 0] == np.float32(f32(s[0, kk // 64]) * np.float32(9 * f32(x[kk])))
    ref = (15.0 * np.repeat(f32(s[1]).astype(np.float64), 64) * f32(x)).sum()
    assert abs(acc[0, 1] - ref) <= 1e-5 * max(1.0, abs(ref))


def test_head_argmax_ties_to_lowest_index():
    """lfm.metal:1196-1214: equal bf16 logits resolve to the lowest token id."""
    g = G(5)
    n, k = 64, 2048
    codes, s, b = synth.quant_weights_np(g, n, k, 6)
    x = synth.activations_np(g, k)
    y = oracle.gemv_quant(codes, s, b, 6, x)[0]
    win = int(np.argmax(f32(y)))
    # copy the winning row onto rows 3 and 40: ties at the max
    for r in (3, 40):
        codes[r], s[r], b[r] = codes[win], s[win], b[win]
    keys, toks = oracle.head_argmax(codes, s, b, 6, x)
    assert toks[0] == min(3, win)
    assert keys[0] == oracle.argmax_key(float(f32(y[win])), int(toks[0]))
    assert oracle.argmax_bf16(oracle.gemv_quant(codes, s, b, 6, x))[0] == toks[0]


def test_argmax_key_order():
    k = oracle.argmax_key
    assert k(1.0, 5) > k(1.0, 6)          # equal value: lower index wins
    assert k(2.0, 9) > k(1.0, 0)
    assert k(-1.0, 0) > k(-2.0, 0)
    assert k(0.0, 3) == k(-0.0, 3)         # -0 folds to +0
    assert k(float("-inf"), 0) > 0


@pytest.mark.parametrize("mode", [0, 1])
def test_route_topk_ties_and_weights(mode):
    z = np.zeros(64, np.float32)
    z[[7, 3, 50, 20, 9]] = [2.0, 2.0, 1.0, 1.0, 0.5]
    bias = np.zeros(64, np.float32)
    ids, w = oracle.route_topk(z, mode, bias)
    assert list(ids[0]) == [3, 7, 20, 50]   # ties to the lower id
    wf = f32(w[0])
    assert abs(wf.sum() - 1.0) < 2e-2
    if mode == 0:
        e = np.exp(np.array([2.0, 2.0, 1.0, 1.0]))
        np.testing.assert_allclose(wf, e / e.sum(), rtol=1e-2)
    else:
        sg = 1 / (1 + np.exp(-np.array([2.0, 2.0, 1.0, 1.0])))
        np.testing.assert_allclose(wf, sg / (sg.sum() + 1e-6), rtol=1e-2)
    # expert_bias changes selection but not the weights' source (lfm.metal:633-654)
    if mode == 1:
        bias[63] = 5.0
        ids, _ = oracle.route_topk(z, mode, bias)
        assert ids[0, 0] == 63


def test_rmsnorm_matches_float64():
    g = G(6)
    h = synth.activations_np(g, 2048)
    b = synth.activations_np(g, 2048)
    w = synth.norm_weight_np(g)
    hout, nout = oracle.add_rmsnorm(h, b, w, 1e-5)
    hp = f32(synth.f32_to_bf16_bits(f32(h) + f32(b))).astype(np.float64)
    assert np.array_equal(hout, synth.f32_to_bf16_bits(f32(h) + f32(b)))
    ref = hp / np.sqrt((hp ** 2).mean() + 1e-5) * f32(w)
    np.testing.assert_allclose(f32(nout), ref, rtol=1e-2, atol=1e-2)


def test_router_logits_match_float64():
    g = G(7)
    n = synth.activations_np(g, 2048)
    w = synth.router_np(g)
    z = oracle.router_logits(n, w, 0)[0]
    ref = f32(w).astype(np.float64) @ f32(n).astype(np.float64)
    np.testing.assert_allclose(z, ref, rtol=1e-4, atol=1e-4)
    wf = f32(w).astype(np.float32)
    z32 = oracle.router_logits(n, wf, 1)[0]
    assert np.array_equal(z32, z)  # a bf16 router widened to f32 is the same router


def test_sort_is_stable_token_major():
    """moe_sorted (lfm.metal:1643-1686): per expert, slots in (token, rank) order."""
    g = G(8)
    m = 300
    ids = np.stack([g.permutation(64)[:4] for _ in range(m)]).astype(np.uint32)
    counts, offsets, ids_sorted, slotpos = oracle.moe_sort(ids)
    assert counts.sum() == 4 * m and offsets[0] == 0
    assert np.array_equal(offsets[1:], np.cumsum(counts)[:-1])
    for t in range(m):
        for r in range(4):
            p = slotpos[4 * t + r]
            assert ids_sorted[p] == t
            e = ids[t, r]
            assert offsets[e] <= p < offsets[e] + counts[e]
    for e in range(64):
        seg = ids_sorted[offsets[e]:offsets[e] + counts[e]]
        assert np.all(np.diff(seg.astype(np.int64)) > 0)  # token-major


def test_dequant_known_answer():
    """quant_nax.metal:2947-2953: w = bf16(s*q + b)."""
    s = synth.f32_to_bf16_bits(np.full((1, 1), 0.01, np.float32))
    b = synth.f32_to_bf16_bits(np.full((1, 1), -0.08, np.float32))
    codes = np.array([[0x76543210, 0xFEDCBA98] * 4], np.uint32)
    out = oracle.dequant_q4(codes, s, b)
    q = np.arange(64) % 16
    ref = synth.f32_to_bf16_bits((np.float32(f32(s)[0, 0]) * q.astype(np.float32)
                                  + np.float32(f32(b)[0, 0])).astype(np.float32))
    assert np.array_equal(out[0], ref)


def test_prefill_chain_small():
    """The prefill chain against an independent float64 restatement."""
    g = G(9)
    m, E, H, I = 24, 64, 2048, 1536
    x = synth.activations_np(g, m, H)
    logits = synth.zipf_logits_np(g, m)
    gate = synth.quant_weights_np(g, E * I, H)
    up = synth.quant_weights_np(g, E * I, H)
    down = synth.quant_weights_np(g, E * H, I)
    r = oracle.moe_prefill(x, logits, gate, up, down)
    xf = f32(x).astype(np.float64)
    for t in range(3):
        acc = np.zeros(H)
        for rk in range(4):
            e = int(r["ids"][t, rk])
            wg = dequant_f64(gate[0][e * I:(e + 1) * I], gate[1][e * I:(e + 1) * I],
                             gate[2][e * I:(e + 1) * I], 4, H)
            wu = dequant_f64(up[0][e * I:(e + 1) * I], up[1][e * I:(e + 1) * I],
                             up[2][e * I:(e + 1) * I], 4, H)
            wd = dequant_f64(down[0][e * H:(e + 1) * H], down[1][e * H:(e + 1) * H],
                             down[2][e * H:(e + 1) * H], 4, I)
            gg, uu = wg @ xf[t], wu @ xf[t]
            a = gg / (1 + np.exp(-gg)) * uu
            acc += float(f32(r["gw"][t:t + 1, rk])[0]) * (wd @ a)
        got = f32(r["out"][t]).astype(np.float64)
        rel = np.abs(got - acc).max() / np.abs(acc).max()
        assert rel < 3e-2, (t, rel)


def test_golden_fixtures_reproduce():
    """The committed fixtures (tests/golden, written by make_golden.py) still
    come out bit for bit: a regression pin of the oracle."""
    from tests.golden import make_golden
    for name, case in make_golden.CASES.items():
        data = np.load(make_golden.path(name))
        got = case(inputs_only=False, data=data)
        for key, val in got.items():
            assert np.array_equal(val, data[key]), (name, key)


def test_dense_gemm_one_expert_matches_float64():
    """The oracle behind mc_gemm_q4 (dequant_q4_bf16_bulk + gemm_bf16_nt,
    quant.metal:69-114, gemm.rs:33-60): its one-expert grouped GEMM equals a
    float64 product of a and the bf16-dequantised weights, the fp32 sums within
    accumulation rounding and the bf16 outputs their rounding."""
    g = G(12)
    m, n, k = 37, 256, 1024
    a = synth.activations_np(g, m, k)
    codes, s, b = synth.quant_weights_np(g, n, k, 4)
    c, acc = oracle.gemm_q4_grouped(a, (codes, s, b), np.array([m], np.uint32),
                                    np.array([0], np.uint32), 1, with_acc=True)
    w = f32(oracle.dequant_q4(codes, s, b)).astype(np.float64)
    ref = f32(a).astype(np.float64) @ w.T
    np.testing.assert_allclose(acc, ref, rtol=1e-4, atol=1e-3)
    assert np.array_equal(c, synth.f32_to_bf16_bits(acc))
