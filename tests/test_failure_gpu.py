"""Failure detection on the GPU without a fault: a bounded device wait is made
to run out on purpose (the router warps of the fused decode layer publish no
logits, so every CTA's logit wait gives up) with a 1 ms limit set on the
context. The kernel must return within the limit with status bit 1 set, and
the next normal call on the same context and workspace must succeed and
match the oracle bit for bit."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import _lib, lfm, synth
from tests.gpu_util import dev_bf16, dev_qw, empty_bf16, host_bits, host_u32, zeros_u32

pytestmark = pytest.mark.gpu

E, H, I = 8, 2048, 512


@pytest.fixture(scope="module")
def small_layer():
    g = synth.rng(4040)
    host = dict(gate=synth.quant_weights_np(g, E * I, H), up=synth.quant_weights_np(g, E * I, H),
                down=synth.quant_weights_np(g, E * H, I), router=synth.router_np(g, E),
                norm_w=synth.norm_weight_np(g))
    dev = dict(gate=dev_qw(*host["gate"]), up=dev_qw(*host["up"]), down=dev_qw(*host["down"]),
               router=dev_bf16(host["router"]), norm_w=dev_bf16(host["norm_w"]))
    return host, dev


def _bufs():
    return dict(hout=empty_bf16(1, H), normed=empty_bf16(1, H),
                logits=torch.empty((1, E), dtype=torch.float32, device="cuda"),
                ids=zeros_u32(1, 4), wts=empty_bf16(1, 4), out=empty_bf16(1, H))


def _layer(ctx, dev, h, b, o, ws=None, status=None):
    if ws is not None:
        lfm.moe_decode_layer(ctx, h, b, dev["norm_w"], o["hout"], o["normed"], dev["router"],
                             o["logits"], None, o["ids"], o["wts"], dev["gate"], dev["up"],
                             dev["down"], o["out"], ws, n_experts=E)
    else:
        lfm.moe_decode_layer_noalloc(ctx, h, b, dev["norm_w"], o["hout"], o["normed"],
                                     dev["router"], o["logits"], None, o["ids"], o["wts"],
                                     dev["gate"], dev["up"], dev["down"], o["out"], status,
                                     n_experts=E)


@pytest.mark.parametrize("entry", ["workspace", "noalloc"])
def test_decode_wait_runs_out_and_context_stays_usable(small_layer, entry):
    host, dev = small_layer
    ctx = lfm.Context(0)
    g = synth.rng(4041)
    h_np, b_np = synth.activations_np(g, 1, H), synth.activations_np(g, 1, H)
    h, b = dev_bf16(h_np), dev_bf16(b_np)
    ws = zeros_u32(lfm.moe_decode_workspace_words(I)) if entry == "workspace" else None
    status = zeros_u32(1)
    try:
        # the failing call: nothing publishes the logits, 1 ms limit per wait
        ctx.set_wait_limit(1_000_000)
        ctx.set_test_flags(_lib.TEST_SKIP_LOGIT_PUBLISH)
        o = _bufs()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        _layer(ctx, dev, h, b, o, ws, status)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        word = int(host_u32(ws[2:3])[0]) if ws is not None else int(host_u32(status)[0])
        assert word & 1, f"status {word}: the logit wait did not report giving up"
        # each CTA gives up after 1 ms on the logits and skips the rest
        assert ms < 50.0, f"the failing launch took {ms:.1f} ms with a 1 ms limit"
        # the next normal call on the same context and scratch succeeds
        ctx.set_test_flags(0)
        ctx.set_wait_limit(0)
        if ws is not None:
            ws[2:3].zero_()  # the workspace's status word is sticky: the caller clears it
        o = _bufs()
        _layer(ctx, dev, h, b, o, ws, status)
        torch.cuda.synchronize()
        word = int(host_u32(ws[2:3])[0]) if ws is not None else int(host_u32(status)[0])
        assert word == 0, f"status {word} after recovery"
        _, no, _, io, wo = oracle.router_addnorm_route(h_np, b_np, host["norm_w"],
                                                       host["router"], 0, None, 0)
        act_o = oracle.gemv_gather_act(host["gate"], host["up"], no, io, n_experts=E)
        out_o = oracle.gemv_gather_down_combine4(host["down"], act_o, io, wo, n_experts=E)
        assert np.array_equal(host_u32(o["ids"]), io)
        assert np.array_equal(host_bits(o["out"]), out_o)
    finally:
        ctx.set_test_flags(0)
        ctx.set_wait_limit(0)
        ctx.close()


def test_status_words_surface_as_errors(small_layer):
    """The Python mirrors raise McError(MC_ETIMEOUT) on a nonzero status word
    when asked to check, so a wait that ran out never passes silently."""
    host, dev = small_layer
    ctx = lfm.Context(0)
    g = synth.rng(4042)
    h, b = dev_bf16(synth.activations_np(g, 1, H)), dev_bf16(synth.activations_np(g, 1, H))
    ws = zeros_u32(lfm.moe_decode_workspace_words(I))
    try:
        ctx.set_wait_limit(1_000_000)
        ctx.set_test_flags(_lib.TEST_SKIP_LOGIT_PUBLISH)
        o = _bufs()
        with pytest.raises(_lib.McError, match="status") as ei:
            lfm.moe_decode_layer(ctx, h, b, dev["norm_w"], o["hout"], o["normed"], dev["router"],
                                 o["logits"], None, o["ids"], o["wts"], dev["gate"], dev["up"],
                                 dev["down"], o["out"], ws, n_experts=E, check=True)
        assert ei.value.code == _lib.MC_ETIMEOUT
    finally:
        ctx.set_test_flags(0)
        ctx.set_wait_limit(0)
        ctx.close()
