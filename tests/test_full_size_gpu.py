"""Parity at BASELINE.json's full sizes against the CPU oracle.

cfg3 exactly as BASELINE states it -- 4096 tokens x 2048, E = 64 experts of
width 1536, router logits Zipf(s=1) + Gumbel over all 64 experts, top-4 --
through the one-call prefill entry point (mc_moe_prefill) and through the
expert-parallel path with W = 2, 4, 8 ranks emulated on one GPU (the
tokens split over the ranks): ids, gate weights, the sorted order and slot
positions bit-exact, activations within the bf16 tolerance.

cfg4 at its full shapes (E = 64, I = 1536, vocab 65536, a 4-layer stack,
three steps) at batch 8 and 32: tokens bit-exact on the per-token GEMV path;
the grouped tensor-core path teacher-forced layer by layer (each layer fed
the oracle's input row) within the tolerance, its ids bit-exact.

Each case records how far the activations are from the oracle (share
bit-identical, max bf16 ulps, max relative error, max absolute error / rms)
with tests.gpu_util.record_stats.
"""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import ep, lfm, synth
from molten_b200.stack import DecodeStack
from tests.gpu_util import (bf16_err_stats, dev_bf16, dev_f32, dev_qw, empty_bf16, host_bits,
                            host_u32, record_stats, zeros_u32)
from tests.test_grouped_gemm_gpu import ACT_ULPS, assert_close_bf16

pytestmark = pytest.mark.gpu

E, H, I, M = 64, 2048, 1536, 4096
RTOL, ATOL_RMS = 1e-2, 1e-2


def _f(bits):
    return synth.bf16_bits_to_f32(np.asarray(bits)).astype(np.float64)


def assert_rows_close(got, want, rows, what):
    """out rows `rows` of the oracle's full prefill: |got - want| <= 1e-2 *
    sum_r |w_r ed_r| + 1e-2 rms(out) (the four terms can cancel)."""
    m = len(rows)
    slot = want["slotpos"].reshape(-1, 4)[rows]
    gw = _f(want["gw"]).reshape(-1, 4)[rows]
    terms = np.abs(gw[:, :, None] * _f(want["ed"])[slot]).sum(axis=1)
    w = _f(want["out"][rows])
    rms = np.sqrt(np.mean(_f(want["out"]) ** 2))
    bad = np.abs(_f(got) - w) > RTOL * terms + ATOL_RMS * rms
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance"
    assert m == got.shape[0]


@pytest.fixture(scope="module")
def cfg3():
    g = synth.rng(3003)
    x = synth.activations_np(g, M, H)
    logits = synth.zipf_logits_np(g, M, E)
    gate, up, down = (synth.quant_weights_np(g, E * I, H), synth.quant_weights_np(g, E * I, H),
                      synth.quant_weights_np(g, E * H, I))
    want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
    dev = dict(x=dev_bf16(x), logits=dev_f32(logits), gate=dev_qw(*gate), up=dev_qw(*up),
               down=dev_qw(*down))
    return dict(x=x, logits=logits, gate=gate, up=up, down=down, want=want, dev=dev)


def test_cfg3_moe_prefill_full_size(cuda_ctx, cfg3):
    d, want = cfg3["dev"], cfg3["want"]
    counts = np.bincount(want["ids"].ravel(), minlength=E)
    assert (counts > 0).sum() == E, "Zipf routing reaches every expert"
    ws = torch.zeros(lfm.moe_prefill_workspace_size(M, E, H, I), dtype=torch.uint8, device="cuda")
    out = empty_bf16(M, H)
    lfm.moe_prefill(cuda_ctx, d["x"], d["logits"], d["gate"], d["up"], d["down"], ws, out,
                    n_experts=E, check=True)
    v = lfm.prefill_workspace_view(ws, M, E, H, I)
    assert np.array_equal(host_u32(v["ids"]), want["ids"])
    assert np.array_equal(host_bits(v["gw"]), want["gw"])
    assert np.array_equal(host_u32(v["ids_sorted"]), want["ids_sorted"])
    assert np.array_equal(host_u32(v["slotpos"]), want["slotpos"])
    act = host_bits(v["act"])
    record_stats("cfg3 act", bf16_err_stats(act, want["act"]))
    assert_close_bf16(act, want["act"], "cfg3 act", ulps=ACT_ULPS)
    # the down GEMM on the GPU's own act isolates it from act's roundings
    c, o, _, _ = oracle.moe_sort(want["ids"], E)
    ed_ref = oracle.gemm_q4_grouped(act, cfg3["down"], c, o, E)
    ed = host_bits(v["ed"])
    record_stats("cfg3 ed (teacher-forced act)", bf16_err_stats(ed, ed_ref))
    assert_close_bf16(ed, ed_ref, "cfg3 ed (teacher-forced act)", min_equal=0.8)
    got = host_bits(out)
    record_stats("cfg3 out", bf16_err_stats(got, want["out"]))
    assert_rows_close(got, want, np.arange(M), "cfg3 out")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_cfg3_expert_parallel_emulated_full_size(cuda_ctx, cfg3, world):
    d, want = cfg3["dev"], cfg3["want"]
    per = M // world
    xs = [d["x"][r * per:(r + 1) * per].contiguous() for r in range(world)]
    lg = [d["logits"][r * per:(r + 1) * per].contiguous() for r in range(world)]
    outs, status, inner = ep.moe_prefill_ep_emulated(cuda_ctx, xs, lg, d["gate"], d["up"],
                                                     d["down"], E, return_state=True)
    assert status == 0
    for r in range(world):
        rows = np.arange(r * per, (r + 1) * per)
        ids = host_u32(inner[r]["ids"])
        assert np.array_equal(ids, want["ids"][rows]), f"rank {r} ids"
        assert np.array_equal(host_bits(inner[r]["gw"]), want["gw"][rows]), f"rank {r} gw"
        _, _, srt, slot = oracle.moe_sort(ids, E)
        assert np.array_equal(host_u32(inner[r]["ids_sorted"]), srt), f"rank {r} ids_sorted"
        assert np.array_equal(host_u32(inner[r]["slotpos"]), slot), f"rank {r} slotpos"
        got = host_bits(outs[r])
        if r == 0:
            record_stats(f"cfg3 ep{world} out (rank 0)", bf16_err_stats(got, want["out"][rows]))
        assert_rows_close(got, want, rows, f"ep{world} rank {r} out")


# ----------------------------------------------------------------- cfg4

L4, V = 4, 65536


@pytest.fixture(scope="module")
def cfg4():
    g = synth.rng(4004)
    layers = []
    for _ in range(L4):
        layers.append(dict(proj=synth.quant_weights_np(g, H, H, centre=7.5),
                           norm_w=synth.norm_weight_np(g), router=synth.router_np(g, E),
                           gate=synth.quant_weights_np(g, E * I, H, centre=7.5),
                           up=synth.quant_weights_np(g, E * I, H, centre=7.5),
                           down=synth.quant_weights_np(g, E * H, I, centre=7.5)))
    head = synth.quant_weights_np(g, V, H, 6, centre=31.5)
    embed = synth.activations_np(g, V, H)
    dl = [dict(proj=dev_qw(*l["proj"]), norm_w=dev_bf16(l["norm_w"]), router=dev_bf16(l["router"]),
               gate=dev_qw(*l["gate"]), up=dev_qw(*l["up"]), down=dev_qw(*l["down"]))
          for l in layers]
    return dict(layers=layers, head=head, embed=embed, dl=dl, dhead=dev_qw(*head, bits=6),
                dembed=dev_bf16(embed))


def _oracle_layer(L, x):
    p = oracle.gemv_quant(*L["proj"], 4, x)
    _, normed, logits, ids, wts = oracle.router_addnorm_route(x, p, L["norm_w"], L["router"], 0,
                                                              None, 0)
    act = oracle.gemv_gather_act(L["gate"], L["up"], normed, ids, n_experts=E)
    out = oracle.gemv_gather_down_combine4(L["down"], act, ids, wts, n_experts=E)
    return p, normed, logits, ids, wts, out


@pytest.mark.parametrize("batch", [8, 32])
def test_cfg4_stack_gemv_path_full_size(cuda_ctx, cfg4, batch):
    """Per-token GEMV expert path at full shapes: every step's tokens equal
    the oracle's bit for bit."""
    steps = 3
    st = DecodeStack(cuda_ctx, cfg4["dl"], cfg4["dhead"], cfg4["dembed"], batch, n_experts=E,
                     moe_path="gemv")
    toks = (np.arange(batch, dtype=np.uint32) * 7919 + 11) % V
    st.start(torch.from_numpy(toks.view(np.int32)).cuda())
    distinct = []
    for s in range(steps):
        x = cfg4["embed"][toks]
        for l, L in enumerate(cfg4["layers"]):
            *_, ids, _, x = _oracle_layer(L, x)
            distinct.append(len(np.unique(ids)))
        _, toks = oracle.head_argmax(*cfg4["head"], 6, x)
        st.step()
        got = st.read_tokens().numpy().view(np.uint32)
        assert np.array_equal(got, toks), f"batch {batch} step {s}: {got} != {toks}"
    assert max(distinct) > 4, "the batch routes to more than one expert set"


def test_cfg4_grouped_path_teacher_forced_full_size(cuda_ctx, cfg4):
    """The tensor-core expert path of batch 32, one layer at a time on the
    oracle's layer input. That path computes the experts with the reference's
    prefill arithmetic (weights dequantised to bf16, fp32 sums), so it is
    checked against the oracle's prefill FFN on the same normed rows and
    router logits: ids bit-exact, output within the prefill tolerance. Its
    distance from the decode GEMV arithmetic (exact fp32 dequant) is recorded."""
    B = 32
    ctx = cuda_ctx
    toks = (np.arange(B, dtype=np.uint32) * 104729 + 5) % V
    x = cfg4["embed"][toks]
    pws = torch.zeros(lfm.moe_prefill_workspace_size(B, E, H, I), dtype=torch.uint8,
                      device="cuda")
    for l, (L, dL) in enumerate(zip(cfg4["layers"], cfg4["dl"])):
        p, normed_o, logits_o, ids_o, wts_o, out_o = _oracle_layer(L, x)
        xd = dev_bf16(x)
        pd, hout, normed = empty_bf16(B, H), empty_bf16(B, H), empty_bf16(B, H)
        logits = torch.empty((B, E), dtype=torch.float32, device="cuda")
        ids, wts, counter = zeros_u32(B, 4), empty_bf16(B, 4), zeros_u32(B)
        lfm.gemv_quant(ctx, dL["proj"], xd, pd)
        lfm.router_addnorm_route(ctx, xd, pd, dL["norm_w"], hout, normed, dL["router"], logits,
                                 None, ids, wts, counter)
        out = empty_bf16(B, H)
        lfm.moe_prefill(ctx, normed, logits, dL["gate"], dL["up"], dL["down"], pws, out,
                        n_experts=E, check=True)
        assert np.array_equal(host_bits(pd), p), f"layer {l}: projection"
        assert np.array_equal(host_u32(ids), ids_o), f"layer {l}: router ids"
        assert np.array_equal(host_bits(normed), normed_o), f"layer {l}: normed rows"
        want = oracle.moe_prefill(normed_o, logits_o, L["gate"], L["up"], L["down"], n_experts=E)
        v = lfm.prefill_workspace_view(pws, B, E, H, I)
        assert np.array_equal(host_u32(v["ids"]), ids_o), f"layer {l}: prefill ids"
        assert np.array_equal(want["ids"], ids_o), f"layer {l}: oracle prefill ids"
        got = host_bits(out)
        record_stats(f"cfg4 grouped layer {l} out vs prefill oracle",
                     bf16_err_stats(got, want["out"]))
        record_stats(f"cfg4 grouped layer {l} out vs decode GEMV oracle",
                     bf16_err_stats(got, out_o))
        assert_rows_close(got, want, np.arange(B), f"layer {l}: out")
        x = out_o


def test_cfg3_ep_through_the_c_abi_one_rank_full_size(cfg3):
    """cfg3 through mc_ep_moe_prefill on a one-rank communicator (the
    library's whole expert-parallel step: NCCL counts all-gather, dispatch,
    device barriers, GEMMs, return, combine), with replicated slots."""
    from tests.test_ep_capi_gpu import _run_rank
    want = cfg3["want"]
    load = np.bincount(want["ids"].ravel(), minlength=E)[None, :]
    ctx = lfm.Context(0)
    try:
        outs, status, counts = _run_rank(ctx, 0, 1, cfg3["x"], cfg3["logits"],
                                         (cfg3["gate"], cfg3["up"], cfg3["down"]), E, I, E + 4,
                                         load, steps=1)
    finally:
        ctx.close()
    assert status == 0
    assert counts.sum() == 4 * M
    record_stats("cfg3 ep (C ABI, one rank) out", bf16_err_stats(outs[0], want["out"]))
    assert_rows_close(outs[0], want, np.arange(M), "cfg3 ep C ABI out")
