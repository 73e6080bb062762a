"""GPU parity of the decode path (C ABI via the lfm mirror) against the CPU
oracle. The decode kernels share the oracle's fixed fp32 operation order, so
every output is compared bit for bit: bf16 rows, fp32 router logits, top-4
ids/weights and argmax tokens."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import lfm, synth
from tests.golden import make_golden
from tests.gpu_util import (assert_bits_equal, dev_bf16, dev_f32, dev_qw, dev_u32, empty_bf16,
                            host_bits, host_u32, zeros_u32)

pytestmark = pytest.mark.gpu


def test_device_math_bit_exact(cuda_ctx):
    g = synth.rng(11)
    x = np.concatenate([g.normal(0, 8, 200000), g.uniform(-110, 95, 50000),
                        [0.0, -0.0, 1e-30, -1e-30, 88.7, 88.8, -103.9, -104.0]]).astype(np.float32)
    xd = dev_f32(x)
    y = torch.empty_like(xd)
    refs = {0: oracle.exp, 1: oracle.silu, 2: oracle.sigmoid}
    for op, fn in refs.items():
        lfm.eval_math(cuda_ctx, op, xd, y)
        got = y.cpu().numpy()
        want = np.array([fn(float(v)) for v in x[::17]], np.float32)
        assert np.array_equal(got[::17].view(np.uint32), want.view(np.uint32)), op


# (4, 8192, ...) and (6, 9999, ...) take the ring-streamed kernel (batch 1,
# K = 2048, at least 32 rows per SM; 9999 leaves partial stages)
@pytest.mark.parametrize("bits,n,k,batch", [(4, 2048, 2048, 1), (4, 2048, 1536, 1),
                                            (4, 1000, 2048, 3), (4, 512, 4096, 2),
                                            (6, 4096, 2048, 1), (6, 96, 2048, 2),
                                            (4, 8192, 2048, 1), (6, 9999, 2048, 1)])
def test_gemv_quant_bit_exact(cuda_ctx, bits, n, k, batch):
    g = synth.rng(20 + bits + n + k + batch)
    codes, s, b = synth.quant_weights_np(g, n, k, bits)
    x = synth.activations_np(g, batch, k)
    w = dev_qw(codes, s, b, bits)
    y = empty_bf16(batch, n)
    lfm.gemv_quant(cuda_ctx, w, dev_bf16(x), y)
    want = oracle.gemv_quant(codes, s, b, bits, x)
    assert_bits_equal(host_bits(y), want, f"gemv q{bits} {n}x{k} b{batch}")


# batch >= 2 on matrices of at least 256 rows per SM, and batch >= 8 on any,
# take the batched kernel (each code decoded once for up to 8 tokens, the
# butterfly replayed in-lane; short matrices split K over 2-8 warps): partial
# token groups (5, 9, 12), K < 2048 (groups 16..31 / 24..31 idle), a partial
# row block (1000 rows)
@pytest.mark.parametrize("bits,n,k,batch", [(6, 40000, 2048, 2), (4, 38000, 1536, 5),
                                            (6, 65536, 2048, 9), (4, 40000, 1024, 3),
                                            (4, 2048, 2048, 8), (4, 2048, 2048, 32),
                                            (6, 1000, 2048, 9), (4, 2048, 1536, 12)])
def test_gemv_batched_bit_exact(cuda_ctx, bits, n, k, batch):
    g = synth.rng(60 + bits + k + batch)
    codes, s, b = synth.quant_weights_np(g, n, k, bits)
    x = synth.activations_np(g, batch, k)
    w = dev_qw(codes, s, b, bits)
    y = empty_bf16(batch, n)
    lfm.gemv_quant(cuda_ctx, w, dev_bf16(x), y)
    want = oracle.gemv_quant(codes, s, b, bits, x)
    assert_bits_equal(host_bits(y), want, f"batched gemv q{bits} {n}x{k} b{batch}")


def test_head_argmax_batched(cuda_ctx):
    """Q6 65536 x 2048 head at batch 11 (two token groups, the second partial):
    keys bit-exact, including a forced tie resolved to the lower row."""
    g = synth.rng(43)
    n, k = 65536, 2048
    codes, s, b = synth.quant_weights_np(g, n, k, 6)
    x = synth.activations_np(g, 11, k)
    y = oracle.gemv_quant(codes, s, b, 6, x[9:10])[0]
    win = int(np.argmax(synth.bf16_bits_to_f32(y)))
    lo = win // 3
    codes[lo], s[lo], b[lo] = codes[win], s[win], b[win]
    keys_o, toks_o = oracle.head_argmax(codes, s, b, 6, x)
    assert toks_o[9] == lo
    w = dev_qw(codes, s, b, 6)
    key = torch.zeros(11, dtype=torch.int64, device="cuda")
    lfm.gemv_head_argmax(cuda_ctx, w, dev_bf16(x), key)
    assert np.array_equal(key.cpu().numpy().view(np.uint64), keys_o)


def test_golden_gemv_and_head(cuda_ctx):
    for name, bits in (("q4_gemv", 4), ("q6_head", 6)):
        d = np.load(make_golden.path(name))
        w = dev_qw(d["codes"], d["scales"], d["biases"], bits)
        x = d["x"].reshape(-1, 2048)
        y = empty_bf16(x.shape[0], d["codes"].shape[0])
        lfm.gemv_quant(cuda_ctx, w, dev_bf16(x), y)
        assert_bits_equal(host_bits(y), d["y"].reshape(y.shape), name)
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    lfm.gemv_head_argmax(cuda_ctx, w, dev_bf16(d["x"]), key)
    assert int(key.cpu().numpy().view(np.uint64)[0]) == int(d["key"][0])


def test_head_argmax_cfg2_and_tail(cuda_ctx):
    """BASELINE cfg2: Q6 65536 x 2048 head + argmax; the tail clears the key."""
    g = synth.rng(31)
    n, k = 65536, 2048
    codes, s, b = synth.quant_weights_np(g, n, k, 6)
    x = synth.activations_np(g, 2, k)
    # force a tie at the top between rows 70000-ish: copy the winner to a lower row
    y = oracle.gemv_quant(codes, s, b, 6, x[:1])[0]
    win = int(np.argmax(synth.bf16_bits_to_f32(y)))
    lo = win // 2
    codes[lo], s[lo], b[lo] = codes[win], s[win], b[win]
    keys_o, toks_o = oracle.head_argmax(codes, s, b, 6, x)
    assert toks_o[0] == lo
    w = dev_qw(codes, s, b, 6)
    key = torch.zeros(2, dtype=torch.int64, device="cuda")
    lfm.gemv_head_argmax(cuda_ctx, w, dev_bf16(x), key)
    assert np.array_equal(key.cpu().numpy().view(np.uint64), keys_o)
    # batch 1 takes the ring-streamed kernel: same key, tie included
    key1 = torch.zeros(1, dtype=torch.int64, device="cuda")
    lfm.gemv_head_argmax(cuda_ctx, w, dev_bf16(x[:1]), key1)
    assert int(key1.cpu().numpy().view(np.uint64)[0]) == int(keys_o[0])
    emb = synth.activations_np(g, 1024, 2048)
    nw = synth.norm_weight_np(g)
    tok = zeros_u32(2)
    xn, nn = empty_bf16(2, 2048), empty_bf16(2, 2048)
    # embedding table smaller than the vocab: tokens >= 1024 leave zeros
    lfm.token_tail(cuda_ctx, key, tok, (dev_bf16(emb), dev_bf16(nw), xn, nn))
    torch.cuda.synchronize()
    assert np.array_equal(host_u32(tok), toks_o)
    assert int(key.abs().sum()) == 0
    for r in range(2):
        t = int(toks_o[r])
        if t < 1024:
            _, want_n = oracle.add_rmsnorm(emb[t], None, nw)
            assert_bits_equal(host_bits(xn[r]), emb[t])
            assert_bits_equal(host_bits(nn[r]), want_n)
        else:
            assert int(xn[r].view(torch.int16).abs().sum()) == 0


def test_argmax_bf16_ties(cuda_ctx):
    g = synth.rng(32)
    logits = synth.activations_np(g, 3, 65536)
    logits[1, 100] = logits[1, 5000] = synth.f32_to_bf16_bits(np.float32([50.0]))[0]
    out = zeros_u32(3)
    lfm.argmax_bf16(cuda_ctx, dev_bf16(logits), out)
    assert np.array_equal(host_u32(out), oracle.argmax_bf16(logits))
    assert host_u32(out)[1] == 100


@pytest.mark.parametrize("with_b", [True, False])
def test_add_rmsnorm(cuda_ctx, with_b):
    g = synth.rng(33)
    h = synth.activations_np(g, 3, 2048)
    b = synth.activations_np(g, 3, 2048) if with_b else None
    w = synth.norm_weight_np(g)
    hout, nout = empty_bf16(3, 2048), empty_bf16(3, 2048)
    lfm.add_rmsnorm(cuda_ctx, dev_bf16(h), None if b is None else dev_bf16(b), dev_bf16(w), hout,
                    nout)
    ho, no = oracle.add_rmsnorm(h, b, w)
    assert_bits_equal(host_bits(hout), ho, "hout")
    assert_bits_equal(host_bits(nout), no, "normed")


@pytest.mark.parametrize("mode,wdt", [(0, "bf16"), (1, "bf16"), (1, "f32"), (0, "f32")])
def test_router_addnorm_route(cuda_ctx, mode, wdt):
    d = np.load(make_golden.path("router"))
    B = 2
    w = d["w"] if wdt == "bf16" else synth.bf16_bits_to_f32(d["w"]).copy()
    wdev = dev_bf16(w) if wdt == "bf16" else dev_f32(w)
    hout, normed = empty_bf16(B, 2048), empty_bf16(B, 2048)
    logits = torch.empty((B, 64), dtype=torch.float32, device="cuda")
    ids, wts = zeros_u32(B, 4), empty_bf16(B, 4)
    counter = zeros_u32(B)
    for _ in range(2):  # the counter must come back zeroed for the next call
        lfm.router_addnorm_route(cuda_ctx, dev_bf16(d["h"]), dev_bf16(d["b"]),
                                 dev_bf16(d["norm_w"]), hout, normed, wdev, logits,
                                 dev_f32(d["ebias"]), ids, wts, counter, route_mode=mode)
    torch.cuda.synchronize()
    assert int(counter.abs().sum()) == 0
    assert_bits_equal(host_bits(hout), d[f"hout{mode}"], "hout")
    assert_bits_equal(host_bits(normed), d[f"normed{mode}"], "normed")
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), d[f"logits{mode}"].view(np.uint32))
    assert np.array_equal(host_u32(ids), d[f"ids{mode}"])
    assert_bits_equal(host_bits(wts), d[f"wts{mode}"], "weights")


def test_unfused_router_and_route(cuda_ctx):
    d = np.load(make_golden.path("router"))
    normed = d["normed0"]
    logits = torch.empty((2, 64), dtype=torch.float32, device="cuda")
    lfm.gemv_f32(cuda_ctx, dev_bf16(d["w"]), dev_bf16(normed), logits)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), d["logits0"].view(np.uint32))
    ids, wts = zeros_u32(2, 4), empty_bf16(2, 4)
    lfm.route_token(cuda_ctx, logits, dev_f32(d["ebias"]), ids, wts, route_mode=1)
    io, wo = oracle.route_topk(d["logits0"], 1, d["ebias"])
    assert np.array_equal(host_u32(ids), io)
    assert_bits_equal(host_bits(wts), wo)


def test_golden_decode_experts(cuda_ctx):
    d = np.load(make_golden.path("decode_experts"))
    inp = make_golden.decode_experts(inputs_only=True, data=d)
    E, I = inp["E"], inp["I"]
    gate, up, down = (dev_qw(*inp[k]) for k in ("gate", "up", "down"))
    act = empty_bf16(2, 4, I)
    lfm.gemv_gather_act(cuda_ctx, gate, up, dev_bf16(inp["x"]), dev_u32(inp["ids"]), act, E)
    assert_bits_equal(host_bits(act), d["act"], "act")
    out = empty_bf16(2, 2048)
    lfm.gemv_gather_down_combine4(cuda_ctx, down, act, dev_u32(inp["ids"]), dev_bf16(inp["wts"]),
                                  out, E)
    assert_bits_equal(host_bits(out), d["out"], "out")


@pytest.fixture(scope="module")
def moe_layer():
    """BASELINE cfg1 weights (64 experts, 2048 -> 1536 -> 2048), seeded."""
    g = synth.rng(40)
    E, H, I = 64, 2048, 1536
    L = dict(gate=synth.quant_weights_np(g, E * I, H), up=synth.quant_weights_np(g, E * I, H),
             down=synth.quant_weights_np(g, E * H, I), router=synth.router_np(g),
             norm_w=synth.norm_weight_np(g))
    L["dev"] = {k: dev_qw(*L[k]) for k in ("gate", "up", "down")}
    L["dev"]["router"] = dev_bf16(L["router"])
    L["dev"]["norm_w"] = dev_bf16(L["norm_w"])
    return L


@pytest.mark.parametrize("batch,seed", [(1, 0), (1, 1), (1, 2), (1, 3), (4, 7), (8, 9)])
def test_moe_decode_layer_cfg1(cuda_ctx, moe_layer, batch, seed):
    """BASELINE cfg1: fused add+norm+router+top-4, gate/up/SiLU, down+combine
    (batch 4 and 8 take the two- and four-tile expert GEMV variants)."""
    g = synth.rng(1000 + seed)
    h = synth.activations_np(g, batch, 2048)
    badd = synth.activations_np(g, batch, 2048)
    D = moe_layer["dev"]
    hout, normed = empty_bf16(batch, 2048), empty_bf16(batch, 2048)
    logits = torch.empty((batch, 64), dtype=torch.float32, device="cuda")
    ids, wts, counter = zeros_u32(batch, 4), empty_bf16(batch, 4), zeros_u32(batch)
    act, out = empty_bf16(batch, 4, 1536), empty_bf16(batch, 2048)
    lfm.router_addnorm_route(cuda_ctx, dev_bf16(h), dev_bf16(badd), D["norm_w"], hout, normed,
                             D["router"], logits, None, ids, wts, counter)
    lfm.gemv_gather_act(cuda_ctx, D["gate"], D["up"], normed, ids, act)
    lfm.gemv_gather_down_combine4(cuda_ctx, D["down"], act, ids, wts, out)
    torch.cuda.synchronize()
    ho, no, lo, io, wo = oracle.router_addnorm_route(h, badd, moe_layer["norm_w"],
                                                     moe_layer["router"], 0, None, 0)
    assert np.array_equal(host_u32(ids), io), "top-4 ids"
    assert_bits_equal(host_bits(wts), wo, "route weights")
    assert_bits_equal(host_bits(normed), no, "normed")
    act_o = oracle.gemv_gather_act(moe_layer["gate"], moe_layer["up"], no, io)
    assert_bits_equal(host_bits(act), act_o, "act")
    out_o = oracle.gemv_gather_down_combine4(moe_layer["down"], act_o, io, wo)
    assert_bits_equal(host_bits(out), out_o, "layer out")


def test_rejects_bad_arguments(cuda_ctx):
    from molten_b200 import _lib
    g = synth.rng(50)
    codes, s, b = synth.quant_weights_np(g, 64, 2048, 4)
    w = dev_qw(codes, s, b)
    x = empty_bf16(2049)[1:]  # misaligned
    with pytest.raises(_lib.McError, match="aligned"):
        lfm.gemv_quant(cuda_ctx, w, x, empty_bf16(64))
    bad = dev_qw(codes, s, b)
    bad.bits = 3
    with pytest.raises(ValueError):
        lfm.gemv_quant(cuda_ctx, bad, empty_bf16(2048), empty_bf16(64))
    # fused decode layer: expert width 96 (not a multiple of 64) is refused
    # before any launch
    E, I = 8, 96
    gu = dev_qw(*synth.quant_weights_np(g, E * I, 2048))
    dn = dev_qw(*synth.quant_weights_np(g, E * 2048, I))
    ws = zeros_u32(lfm.moe_decode_workspace_words(I))
    o = lambda: empty_bf16(1, 2048)
    with pytest.raises((_lib.McError, ValueError)):
        lfm.moe_decode_layer(cuda_ctx, o(), None, o(), o(), o(), dev_bf16(synth.router_np(g, E)),
                             torch.empty((1, E), dtype=torch.float32, device="cuda"), None,
                             zeros_u32(1, 4), empty_bf16(1, 4), gu, gu, dn, o(), ws,
                             n_experts=E)


@pytest.mark.parametrize("mode,seed", [(0, 0), (0, 1), (0, 2), (1, 3), (0, 4)])
def test_fused_moe_decode_layer(cuda_ctx, moe_layer, mode, seed):
    """The one-launch layer equals the oracle (and so the three-kernel path)
    bit for bit on consecutive calls sharing one workspace, and reports no
    error status."""
    g = synth.rng(2000 + seed)
    D = moe_layer["dev"]
    ebias = g.normal(0, 0.1, 64).astype(np.float32)
    ws = zeros_u32(lfm.moe_decode_workspace_words())
    hout, normed = empty_bf16(1, 2048), empty_bf16(1, 2048)
    logits = torch.empty((1, 64), dtype=torch.float32, device="cuda")
    ids, wts = zeros_u32(1, 4), empty_bf16(1, 4)
    out = empty_bf16(1, 2048)
    for it in range(3):
        h = synth.activations_np(g, 1, 2048)
        badd = synth.activations_np(g, 1, 2048)
        lfm.moe_decode_layer(cuda_ctx, dev_bf16(h), dev_bf16(badd), D["norm_w"], hout, normed,
                             D["router"], logits, dev_f32(ebias), ids, wts, D["gate"], D["up"],
                             D["down"], out, ws, route_mode=mode)
        torch.cuda.synchronize()
        ctl = host_u32(ws[:4])
        assert ctl[0] == it + 1 and ctl[1] == 0 and ctl[2] == 0 and ctl[3] == 0, ctl
        ho, no, lo, io, wo = oracle.router_addnorm_route(h, badd, moe_layer["norm_w"],
                                                         moe_layer["router"], 0, ebias, mode)
        assert np.array_equal(host_u32(ids), io), "top-4 ids"
        assert_bits_equal(host_bits(wts), wo, "weights")
        assert_bits_equal(host_bits(hout), ho, "h_out")
        assert_bits_equal(host_bits(normed), no, "normed")
        assert np.array_equal(logits.cpu().numpy().view(np.uint32), lo.view(np.uint32))
        act_o = oracle.gemv_gather_act(moe_layer["gate"], moe_layer["up"], no, io)
        assert_bits_equal(host_bits(lfm.decode_workspace_act(ws)), act_o.reshape(4, 1536), "act")
        out_o = oracle.gemv_gather_down_combine4(moe_layer["down"], act_o, io, wo)
        assert_bits_equal(host_bits(out), out_o, "out")


@pytest.mark.parametrize("mode,seed", [(0, 0), (1, 1)])
def test_fused_proj_moe_decode_layer(cuda_ctx, moe_layer, mode, seed):
    """mc_moe_decode_layer_proj: b = bf16(proj . h), computed inside the
    launch and exchanged between the CTAs, equals the oracle's Q4 GEMV bit for
    bit, and every layer output equals the oracle's (so gemv_quant followed by
    moe_decode_layer) on consecutive calls sharing one workspace."""
    g = synth.rng(2100 + seed)
    D = moe_layer["dev"]
    pc, ps, pb = synth.quant_weights_np(g, 2048, 2048)
    proj = dev_qw(pc, ps, pb)
    ebias = g.normal(0, 0.1, 64).astype(np.float32)
    ws = zeros_u32(lfm.moe_decode_proj_workspace_words())
    hout, normed = empty_bf16(1, 2048), empty_bf16(1, 2048)
    logits = torch.empty((1, 64), dtype=torch.float32, device="cuda")
    ids, wts = zeros_u32(1, 4), empty_bf16(1, 4)
    out, p_out = empty_bf16(1, 2048), empty_bf16(1, 2048)
    for it in range(3):
        h = synth.activations_np(g, 1, 2048)
        lfm.moe_decode_layer_proj(cuda_ctx, dev_bf16(h), proj, D["norm_w"], hout, normed,
                                  D["router"], logits, dev_f32(ebias), ids, wts, D["gate"],
                                  D["up"], D["down"], out, ws, p_out=p_out, route_mode=mode)
        torch.cuda.synchronize()
        ctl = host_u32(ws[:4])
        assert ctl[0] == it + 1 and ctl[1] == 0 and ctl[2] == 0 and ctl[3] == 0, ctl
        p_o = oracle.gemv_quant(pc, ps, pb, 4, h)
        assert_bits_equal(host_bits(p_out), p_o, "projection b")
        ho, no, lo, io, wo = oracle.router_addnorm_route(h, p_o, moe_layer["norm_w"],
                                                         moe_layer["router"], 0, ebias, mode)
        assert np.array_equal(host_u32(ids), io), "top-4 ids"
        assert_bits_equal(host_bits(wts), wo, "weights")
        assert_bits_equal(host_bits(hout), ho, "h_out")
        assert_bits_equal(host_bits(normed), no, "normed")
        assert np.array_equal(logits.cpu().numpy().view(np.uint32), lo.view(np.uint32))
        act_o = oracle.gemv_gather_act(moe_layer["gate"], moe_layer["up"], no, io)
        out_o = oracle.gemv_gather_down_combine4(moe_layer["down"], act_o, io, wo)
        assert_bits_equal(host_bits(out), out_o, "out")


def test_copy_async_host_device(cuda_ctx):
    """mc_copy_async: pinned host -> device and back through the copy kernel
    (16-byte multiples), an odd byte count through the cudaMemcpyAsync path,
    and unpinned host memory refused by the wrapper."""
    src = torch.randn(3, 2048).to(torch.bfloat16).pin_memory()
    dev = torch.empty((3, 2048), dtype=torch.bfloat16, device="cuda")
    back = torch.empty((3, 2048), dtype=torch.bfloat16, pin_memory=True)
    lfm.copy_async(cuda_ctx, dev, src)
    lfm.copy_async(cuda_ctx, back, dev)
    cuda_ctx.commit_wait()
    assert torch.equal(back.view(torch.int16), src.view(torch.int16))
    assert torch.equal(dev.cpu().view(torch.int16), src.view(torch.int16))
    odd = torch.arange(7, dtype=torch.int16).pin_memory()
    d7 = torch.zeros(7, dtype=torch.int16, device="cuda")
    lfm.copy_async(cuda_ctx, d7, odd)
    cuda_ctx.commit_wait()
    assert torch.equal(d7.cpu(), odd)
    with pytest.raises(ValueError):
        lfm.copy_async(cuda_ctx, d7, torch.zeros(7, dtype=torch.int16))
