"""GPU parity of the prefill grouped expert GEMMs (tcgen05) against the CPU
oracle. The tensor cores accumulate in fp32 in an unspecified order, so the
bf16 outputs are compared within the BASELINE tolerance: |got - want| <=
1e-2 * |want| + 1e-2 * rms(want); integer/index outputs stay bit-exact."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import lfm, synth
from tests.gpu_util import (assert_bits_equal, dev_bf16, dev_f32, dev_qw, empty_bf16, host_bits,
                            host_u32, zeros_u32)

pytestmark = pytest.mark.gpu

RTOL = 1e-2
ATOL_RMS = 1e-2
ACT_ULPS = 3


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (8 significant bits)."""
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -126)))
    return 2.0 ** (e - 7)


def assert_close_bf16(got_bits, want_bits, what, min_equal=0.5, ulps=0):
    """|got - want| <= 1e-2 |want| + 1e-2 rms(want) (+ `ulps` bf16 ulps of want
    for values that went through several bf16 roundings)."""
    got = synth.bf16_bits_to_f32(np.asarray(got_bits)).astype(np.float64)
    want = synth.bf16_bits_to_f32(np.asarray(want_bits)).astype(np.float64)
    assert got.shape == want.shape, what
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    rms = np.sqrt(np.mean(want ** 2)) if want.size else 0.0
    err = np.abs(got - want)
    bad = err > RTOL * np.abs(want) + ATOL_RMS * rms + ulps * bf16_ulp(want)
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance, "
                           f"max err {err.max():.3g}, rms {rms:.3g}")
    eq = np.mean(np.asarray(got_bits) == np.asarray(want_bits))
    assert eq >= min_equal, f"{what}: only {eq:.2%} bit-identical"


def assert_out_close(got_bits, want, what="out"):
    """out[t] is a sum of four bf16-rounded terms that can cancel, so the
    relative part of the tolerance is taken on sum_r |w_r * ed_r|, not on |out|."""
    f = lambda b: synth.bf16_bits_to_f32(np.asarray(b)).astype(np.float64)
    m = want["out"].shape[0]
    terms = np.abs(f(want["gw"]).reshape(m, 4, 1) * f(want["ed"])[want["slotpos"].reshape(m, 4)])
    got_o, want_o = f(got_bits), f(want["out"])
    rms = np.sqrt(np.mean(want_o ** 2))
    bad = np.abs(got_o - want_o) > RTOL * terms.sum(axis=1) + ATOL_RMS * rms
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"


def prefill_case(seed, m, E, H, I, hot=None):
    g = synth.rng(seed)
    x = synth.activations_np(g, m, H)
    logits = synth.zipf_logits_np(g, m, E)
    if hot is not None:  # concentrate routing on a few experts (keeps the oracle fast)
        logits[:, hot:] -= 30.0
    gate = synth.quant_weights_np(g, E * I, H)
    up = synth.quant_weights_np(g, E * I, H)
    down = synth.quant_weights_np(g, E * H, I)
    return x, logits, gate, up, down


def run_gpu_chain(ctx, x, logits, gate, up, down, E, bm=128):
    m, H = x.shape
    I = gate[0].shape[0] // E
    S = 4 * m
    ids, gw = zeros_u32(m, 4), empty_bf16(m, 4)
    lfm.moe_route_batch(ctx, dev_f32(logits), None, ids, gw, m)
    max_tiles = (S + bm - 1) // bm + E
    counts, offsets = zeros_u32(E), zeros_u32(E)
    ids_sorted, slotpos = zeros_u32(S), zeros_u32(S)
    tiles, n_tiles = zeros_u32(max_tiles, 4), zeros_u32(1)
    lfm.moe_sort_map(ctx, ids, counts, offsets, ids_sorted, slotpos, tiles, n_tiles, m, bm)
    gx = empty_bf16(S, H)
    lfm.gather_rows_bf16(ctx, dev_bf16(x), ids_sorted, gx)
    act = torch.zeros((S, I), dtype=torch.bfloat16, device="cuda")
    ed = torch.zeros((S, H), dtype=torch.bfloat16, device="cuda")
    status = zeros_u32(1)
    G, U, D = dev_qw(*gate), dev_qw(*up), dev_qw(*down)
    lfm.gemm_q4_grouped_gu(ctx, gx, G, U, act, tiles, n_tiles, E, status)
    lfm.gemm_q4_grouped(ctx, act, D, ed, tiles, n_tiles, E, status)
    out = empty_bf16(m, H)
    lfm.moe_combine_rows(ctx, ed, slotpos, gw, out)
    torch.cuda.synchronize()
    assert int(host_u32(status)[0]) == 0, f"kernel status {host_u32(status)[0]}"
    return dict(ids=host_u32(ids), gw=host_bits(gw), ids_sorted=host_u32(ids_sorted),
                slotpos=host_u32(slotpos), act=host_bits(act), ed=host_bits(ed),
                out=host_bits(out), gx=gx)


@pytest.mark.parametrize("seed,m,E,I,hot,bm", [(1, 96, 8, 256, None, 128),
                                               (2, 300, 8, 384, None, 256),
                                               (3, 64, 64, 1536, 8, 256),
                                               (4, 10, 8, 256, None, 256),
                                               (5, 200, 4, 128, None, 64),
                                               (6, 300, 8, 640, None, 112),
                                               (7, 700, 4, 256, None, 200)])
def test_grouped_ffn_matches_oracle(cuda_ctx, seed, m, E, I, hot, bm):
    """bm 256: chunks up to the MMA's largest N (one 256-row token box); m=10:
    fewer rows (40) than the smallest token box; bm 64/112/200: chunk heights
    that pick each token-box size and are not multiples of 16; I=384/640: down
    K not a multiple of 256."""
    H = 2048
    x, logits, gate, up, down = prefill_case(seed, m, E, H, I, hot)
    got = run_gpu_chain(cuda_ctx, x, logits, gate, up, down, E, bm)
    want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
    assert np.array_equal(got["ids"], want["ids"])
    assert_bits_equal(got["gw"], want["gw"], "gw")
    assert np.array_equal(got["ids_sorted"], want["ids_sorted"])
    assert np.array_equal(got["slotpos"], want["slotpos"])
    # act = bf16(bf16(silu(bf16 g)) * bf16 u): a one-ulp flip of g or u (their
    # fp32 sums run in another order on the tensor cores) and of silu(g) stack
    # to about three bf16 ulps of act
    assert_close_bf16(got["act"], want["act"], "act", ulps=ACT_ULPS)
    # the down GEMM on the GPU's own act isolates the GEMM from act rounding
    counts, offsets, _, _ = oracle.moe_sort(want["ids"], E)
    ed_ref = oracle.gemm_q4_grouped(got["act"], down, counts, offsets, E)
    assert_close_bf16(got["ed"], ed_ref, "ed (teacher-forced act)", min_equal=0.8)
    assert_bits_equal(got["out"], oracle.moe_combine(got["ed"], got["slotpos"], got["gw"], m, H),
                      "combine (teacher-forced ed)")
    assert_out_close(got["out"], want)


def test_grouped_gemm_single_matrix_exactness_structure(cuda_ctx):
    """One expert, one tile, all-zero codes: C = A . b-row, so every output
    column n is sum_k a_k * b_n -- checks the B layout/swizzle and the tile
    bookkeeping with a hand-computable answer."""
    E, H, N, rows = 1, 2048, 128, 100
    g = synth.rng(5)
    a = synth.activations_np(g, rows, H)
    codes = np.zeros((E * N, H // 8), np.uint32)
    s = synth.f32_to_bf16_bits(np.full((E * N, H // 64), 0.01, np.float32))
    b = synth.f32_to_bf16_bits(np.repeat(np.linspace(-1, 1, N, dtype=np.float32)[:, None],
                                         H // 64, axis=1))
    tiles = np.zeros((4, 4), np.uint32)
    tiles[0] = [0, rows, 0, 0]
    n_tiles = np.array([1], np.uint32)
    from tests.gpu_util import dev_u32
    c = torch.zeros((rows, N), dtype=torch.bfloat16, device="cuda")
    st = zeros_u32(1)
    lfm.gemm_q4_grouped(cuda_ctx, dev_bf16(a), dev_qw(codes, s, b), c, dev_u32(tiles),
                        dev_u32(n_tiles), E, st)
    torch.cuda.synchronize()
    assert int(host_u32(st)[0]) == 0
    want = oracle.gemm_q4_grouped(a, (codes, s, b), np.array([rows], np.uint32),
                                  np.array([0], np.uint32), E)
    assert_close_bf16(host_bits(c), want, "single tile", min_equal=0.8)


def test_moe_prefill_entry_point(cuda_ctx):
    """mc_moe_prefill (all seven launches behind one call) against the oracle."""
    E, H, I, m = 8, 2048, 256, 160
    x, logits, gate, up, down = prefill_case(11, m, E, H, I)
    ws = torch.zeros(lfm.moe_prefill_workspace_size(m, E, H, I), dtype=torch.uint8, device="cuda")
    out = empty_bf16(m, H)
    lfm.moe_prefill(cuda_ctx, dev_bf16(x), dev_f32(logits), dev_qw(*gate), dev_qw(*up),
                    dev_qw(*down), ws, out, n_experts=E)
    torch.cuda.synchronize()
    v = lfm.prefill_workspace_view(ws, m, E, H, I)
    assert int(host_u32(v["status"])[0]) == 0
    want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
    assert np.array_equal(host_u32(v["ids"]), want["ids"])
    assert_close_bf16(host_bits(v["act"]), want["act"], "act", ulps=ACT_ULPS)
    # combine is a fixed-order sum: bit-exact on the GPU's own expert rows
    ed = host_bits(v["ed"])
    gw = host_bits(v["gw"])
    slot = host_u32(v["slotpos"])
    assert_bits_equal(host_bits(out), oracle.moe_combine(ed, slot, gw, m, H), "combine")
    assert_out_close(host_bits(out), want)


def test_grouped_gemm_flags_malformed_tile(cuda_ctx):
    """A tile past the last row or taller than 256 rows is not computed into C:
    status bit 1 is set and the good tile's rows are still right."""
    E, H, N, rows = 2, 2048, 128, 100
    g = synth.rng(6)
    a = synth.activations_np(g, rows, H)
    w = synth.quant_weights_np(g, E * N, H)
    from tests.gpu_util import dev_u32
    tiles = np.zeros((4, 4), np.uint32)
    tiles[0] = [0, rows, 1, 0]
    tiles[1] = [0, 400, 0, 0]  # m_end past rows and taller than 256
    c = torch.zeros((rows, N), dtype=torch.bfloat16, device="cuda")
    st = zeros_u32(1)
    lfm.gemm_q4_grouped(cuda_ctx, dev_bf16(a), dev_qw(*w), c, dev_u32(tiles),
                        dev_u32(np.array([2], np.uint32)), E, st)
    torch.cuda.synchronize()
    assert int(host_u32(st)[0]) == 2
    want = oracle.gemm_q4_grouped(a, w, np.array([0, rows], np.uint32),
                                  np.array([0, 0], np.uint32), E)
    assert_close_bf16(host_bits(c), want, "good tile beside a malformed one", min_equal=0.8)


@pytest.mark.parametrize("m,n,k", [(700, 256, 2048), (256, 384, 1536), (40, 128, 256)])
def test_dense_gemm_q4_matches_oracle(cuda_ctx, m, n, k):
    """mc_gemm_q4 (prefill projections, dequant_q4_bf16_bulk + gemm_bf16_nt):
    the grouped kernel with one expert over 256-row chunks, the last one partial
    (700, 40 rows), against the oracle's one-expert grouped GEMM."""
    g = synth.rng(90 + m)
    a = synth.activations_np(g, m, k)
    codes, s, b = synth.quant_weights_np(g, n, k, 4)
    ws = torch.zeros(lfm.gemm_q4_workspace_words(m), dtype=torch.int32, device="cuda")
    c = empty_bf16(m, n)
    st = zeros_u32(1)
    lfm.gemm_q4(cuda_ctx, dev_bf16(a), dev_qw(codes, s, b), c, ws, st)
    torch.cuda.synchronize()
    assert int(host_u32(st)[0]) == 0
    want = oracle.gemm_q4_grouped(a, (codes, s, b), np.array([m], np.uint32),
                                  np.array([0], np.uint32), 1)
    assert_close_bf16(host_bits(c), want, f"dense {m}x{n}x{k}", min_equal=0.8)
