"""GPU parity of the prefill dispatch kernels (route, sort/tile map, gather,
SwiGLU, combine) against the CPU oracle. All integer/index outputs and the
elementwise bf16 outputs are bit-exact."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import lfm, synth
from tests.gpu_util import (assert_bits_equal, dev_bf16, dev_f32, dev_u32, empty_bf16, host_bits,
                            host_u32, zeros_u32)

pytestmark = pytest.mark.gpu


def route_and_sort(ctx, logits_np, bm=128, E=64):
    m = logits_np.shape[0]
    ids, gw = zeros_u32(m, 4), empty_bf16(m, 4)
    lfm.moe_route_batch(ctx, dev_f32(logits_np), None, ids, gw, m)
    max_tiles = (4 * m + bm - 1) // bm + E
    bufs = dict(counts=zeros_u32(E), offsets=zeros_u32(E), ids_sorted=zeros_u32(4 * m),
                slotpos=zeros_u32(4 * m), tiles=zeros_u32(max_tiles, 4), n_tiles=zeros_u32(1))
    lfm.moe_sort_map(ctx, ids, bufs["counts"], bufs["offsets"], bufs["ids_sorted"],
                     bufs["slotpos"], bufs["tiles"], bufs["n_tiles"], m, bm)
    torch.cuda.synchronize()
    return ids, gw, bufs


@pytest.mark.parametrize("m", [1, 7, 300, 4096])
def test_route_batch_and_sort_map(cuda_ctx, m):
    g = synth.rng(60 + m)
    logits = synth.zipf_logits_np(g, m)
    ids, gw, bufs = route_and_sort(cuda_ctx, logits)
    io, wo = oracle.moe_route_batch(logits)
    assert np.array_equal(host_u32(ids), io)
    assert_bits_equal(host_bits(gw), wo, "gw")
    counts, offsets, ids_sorted, slotpos = oracle.moe_sort(io)
    assert np.array_equal(host_u32(bufs["counts"]), counts)
    assert np.array_equal(host_u32(bufs["offsets"]), offsets)
    assert np.array_equal(host_u32(bufs["ids_sorted"]), ids_sorted)
    assert np.array_equal(host_u32(bufs["slotpos"]), slotpos)
    # tile list: every expert's rows covered once by <=128-row tiles; full
    # tiles first in expert order, then partial tiles by decreasing height
    nt = int(host_u32(bufs["n_tiles"])[0])
    tiles = host_u32(bufs["tiles"])[:nt]
    full, part = [], []
    for e in range(64):
        for j in range(0, int(counts[e]), 128):
            m0 = int(offsets[e]) + j
            t = (m0, min(m0 + 128, int(offsets[e] + counts[e])), e, 0)
            (full if t[1] - t[0] == 128 else part).append(t)
    part.sort(key=lambda t: (-(t[1] - t[0]), t[2]))
    assert [tuple(t) for t in tiles] == full + part


def test_route_batch_sigmoid_mode(cuda_ctx):
    g = synth.rng(70)
    logits = g.normal(0, 2, (513, 64)).astype(np.float32)
    bias = g.normal(0, 0.5, 64).astype(np.float32)
    ids, gw = zeros_u32(513, 4), empty_bf16(513, 4)
    lfm.moe_route_batch(cuda_ctx, dev_f32(logits), dev_f32(bias), ids, gw, 513,
                        route_mode=lfm.ROUTE_SIGMOID_BIAS)
    io, wo = oracle.moe_route_batch(logits, 1, bias)
    assert np.array_equal(host_u32(ids), io)
    assert_bits_equal(host_bits(gw), wo)


def test_gather_silu_combine(cuda_ctx):
    g = synth.rng(71)
    m, H, I = 257, 2048, 1536
    x = synth.activations_np(g, m, H)
    logits = synth.zipf_logits_np(g, m)
    ids, gw, bufs = route_and_sort(cuda_ctx, logits)
    io, wo = oracle.moe_route_batch(logits)
    _, _, ids_sorted, slotpos = oracle.moe_sort(io)
    gx = empty_bf16(4 * m, H)
    lfm.gather_rows_bf16(cuda_ctx, dev_bf16(x), bufs["ids_sorted"], gx)
    assert_bits_equal(host_bits(gx), oracle.gather_rows(x, ids_sorted), "gather")
    gg = synth.activations_np(g, 4 * m, I)
    uu = synth.activations_np(g, 4 * m, I)
    act = empty_bf16(4 * m, I)
    lfm.silu_mul_bf16(cuda_ctx, dev_bf16(gg), dev_bf16(uu), act)
    assert_bits_equal(host_bits(act), oracle.silu_mul(gg, uu), "silu_mul")
    ed = synth.activations_np(g, 4 * m, H)
    out = empty_bf16(m, H)
    lfm.moe_combine_rows(cuda_ctx, dev_bf16(ed), bufs["slotpos"], gw, out)
    assert_bits_equal(host_bits(out), oracle.moe_combine(ed, slotpos, wo, m, H), "combine")
