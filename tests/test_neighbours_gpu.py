"""Decode neighbours of the MoE block against the CPU oracle, bit for bit:
the Q/K/V GEMVs with the V-cache scatter (proj3_gemv_scatter), the short
conv's projection + conv (conv3_gemv), the dense FFN's gate/up + SwiGLU
(gemv_gu_act) and its K = 11776 down projection (gemv_quant on wide rows),
at the reference model's shapes (hidden 2048, 32 query heads and 8 KV heads
of 64, dense width 11776)."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import _lib, lfm, synth
from tests.gpu_util import assert_bits_equal, dev_bf16, dev_qw, empty_bf16, host_bits

pytestmark = pytest.mark.gpu

H = 2048


@pytest.mark.parametrize("nq,nk,nv,max_seq,pos", [(2048, 512, 512, 64, 5),
                                                  (2048, 512, 512, 4096, 4095),
                                                  (128, 64, 64, 3, 0)])
def test_proj3_gemv_scatter(cuda_ctx, nq, nk, nv, max_seq, pos):
    g = synth.rng(1000 + nq + pos)
    q, k, v = (synth.quant_weights_np(g, n, H) for n in (nq, nk, nv))
    x = synth.activations_np(g, 1, H)
    cache = synth.activations_np(g, nv // 64, max_seq, 64)  # earlier positions stay
    cache_d = dev_bf16(cache)
    qo, ko = empty_bf16(nq), empty_bf16(nk)
    lfm.proj3_gemv_scatter(cuda_ctx, dev_qw(*q), dev_qw(*k), dev_qw(*v), dev_bf16(x), qo, ko,
                           cache_d, pos)
    torch.cuda.synchronize()
    wq, wk, wc = oracle.proj3_gemv_scatter(q, k, v, x, cache, pos)
    assert_bits_equal(host_bits(qo), wq, "q")
    assert_bits_equal(host_bits(ko), wk, "k")
    assert_bits_equal(host_bits(cache_d), wc, "v cache (slot pos written, the rest unchanged)")


def test_proj3_rejects_position_outside_the_cache(cuda_ctx):
    g = synth.rng(1010)
    q, k, v = (dev_qw(*synth.quant_weights_np(g, n, H)) for n in (128, 64, 64))
    with pytest.raises(ValueError, match="KV cache"):
        lfm.proj3_gemv_scatter(cuda_ctx, q, k, v, empty_bf16(H), empty_bf16(128), empty_bf16(64),
                               empty_bf16(1, 8, 64), 8)


@pytest.mark.parametrize("channels", [2048, 96])
def test_conv3_gemv(cuda_ctx, channels):
    g = synth.rng(1100 + channels)
    w = synth.quant_weights_np(g, 3 * channels, H)
    x = synth.activations_np(g, 1, H)
    taps = synth.f32_to_bf16_bits(g.normal(0, 0.5, (channels, 3)).astype(np.float32))
    state = synth.activations_np(g, 2, channels)
    out, ns = empty_bf16(channels), empty_bf16(2, channels)
    lfm.conv3_gemv(cuda_ctx, dev_qw(*w), dev_bf16(x), dev_bf16(taps), dev_bf16(state), out, ns)
    torch.cuda.synchronize()
    wo, wns = oracle.conv3_gemv(w, x, taps, state)
    assert_bits_equal(host_bits(out), wo, "conv out")
    assert_bits_equal(host_bits(ns), wns, "conv new state")


@pytest.mark.parametrize("n,k,batch", [(11776, 2048, 1), (11776, 2048, 3), (512, 4096, 2)])
def test_gemv_gu_act(cuda_ctx, n, k, batch):
    g = synth.rng(1200 + n + k + batch)
    gate, up = synth.quant_weights_np(g, n, k), synth.quant_weights_np(g, n, k)
    x = synth.activations_np(g, batch, k)
    act = empty_bf16(batch, n)
    lfm.gemv_gu_act(cuda_ctx, dev_qw(*gate), dev_qw(*up), dev_bf16(x), act)
    torch.cuda.synchronize()
    assert_bits_equal(host_bits(act), oracle.gemv_gu_act(gate, up, x), "act")


@pytest.mark.parametrize("k,batch", [(11776, 1), (11776, 2), (4160, 1), (16384, 1)])
def test_wide_q4_gemv(cuda_ctx, k, batch):
    """The dense FFN's down projection (K = 11776, lfm_gemv_q4_bf16_k11776)
    and the edges of the wide-row kernel (4160 = just above 4096, 16384)."""
    g = synth.rng(1300 + k + batch)
    n = 2048
    codes, s, b = synth.quant_weights_np(g, n, k)
    x = synth.activations_np(g, batch, k)
    y = empty_bf16(batch, n)
    lfm.gemv_quant(cuda_ctx, dev_qw(codes, s, b), dev_bf16(x), y)
    torch.cuda.synchronize()
    assert_bits_equal(host_bits(y), oracle.gemv_quant(codes, s, b, 4, x), f"K={k}")


def test_wide_rows_beyond_the_built_width_are_rejected(cuda_ctx):
    g = synth.rng(1400)
    w = dev_qw(*synth.quant_weights_np(g, 64, 16448))
    with pytest.raises(_lib.McError, match="16384"):
        lfm.gemv_quant(cuda_ctx, w, empty_bf16(1, 16448), empty_bf16(1, 64))
