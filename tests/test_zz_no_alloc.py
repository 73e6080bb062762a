"""mc_moe_decode_layer_noalloc (built-in scratch, no allocation) against the
workspace entry point mc_moe_decode_layer on the same inputs, through the C
ABI, and against the CPU oracle. Both entry points run the same bit-exact
kernel, so the tolerance is zero: every output is compared bit for bit, on
two consecutive calls with different tokens (the second call reuses the
scratch state the first one left)."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import _lib, lfm, synth
from tests.gpu_util import dev_bf16, dev_f32, dev_qw, empty_bf16, host_bits, host_u32, zeros_u32

pytestmark = pytest.mark.gpu

E, H, I = 64, 2048, 1536


@pytest.fixture(scope="module")
def layer():
    g = synth.rng(77)
    host = dict(gate=synth.quant_weights_np(g, E * I, H), up=synth.quant_weights_np(g, E * I, H),
                down=synth.quant_weights_np(g, E * H, I), router=synth.router_np(g),
                norm_w=synth.norm_weight_np(g), ebias=g.normal(0, 0.1, E).astype(np.float32))
    L = dict(gate=dev_qw(*host["gate"]), up=dev_qw(*host["up"]), down=dev_qw(*host["down"]),
             router=dev_bf16(host["router"]), norm_w=dev_bf16(host["norm_w"]),
             ebias=dev_f32(host["ebias"]), host=host)
    return L


def outputs():
    return dict(hout=empty_bf16(1, H), normed=empty_bf16(1, H),
                logits=torch.empty((1, E), dtype=torch.float32, device="cuda"),
                ids=zeros_u32(1, 4), wts=empty_bf16(1, 4), out=empty_bf16(1, H))


@pytest.mark.parametrize("mode", [lfm.ROUTE_SOFTMAX_RENORM, lfm.ROUTE_SIGMOID_BIAS])
def test_noalloc_matches_workspace_entry_point(cuda_ctx, layer, mode):
    g = synth.rng(300 + mode)
    ws = zeros_u32(lfm.moe_decode_workspace_words())
    status = zeros_u32(1)
    hw = layer["host"]
    for it in range(2):
        h_np, b_np = synth.activations_np(g, 1, H), synth.activations_np(g, 1, H)
        h, badd = dev_bf16(h_np), dev_bf16(b_np)
        a, b = outputs(), outputs()
        lfm.moe_decode_layer(cuda_ctx, h, badd, layer["norm_w"], a["hout"], a["normed"],
                             layer["router"], a["logits"], layer["ebias"], a["ids"], a["wts"],
                             layer["gate"], layer["up"], layer["down"], a["out"], ws,
                             route_mode=mode)
        status.fill_(-1)
        lfm.moe_decode_layer_noalloc(cuda_ctx, h, badd, layer["norm_w"], b["hout"], b["normed"],
                                     layer["router"], b["logits"], layer["ebias"], b["ids"],
                                     b["wts"], layer["gate"], layer["up"], layer["down"],
                                     b["out"], status, route_mode=mode)
        torch.cuda.synchronize()
        assert int(host_u32(status)[0]) == 0, f"call {it}: status {host_u32(status)[0]}"
        assert int(host_u32(ws[2:3])[0]) == 0
        for k in ("hout", "normed", "ids", "wts", "out"):
            assert np.array_equal(host_bits(a[k]) if a[k].dtype == torch.bfloat16
                                  else host_u32(a[k]),
                                  host_bits(b[k]) if b[k].dtype == torch.bfloat16
                                  else host_u32(b[k])), f"call {it}: {k} differs"
        assert np.array_equal(a["logits"].cpu().numpy().view(np.uint32),
                              b["logits"].cpu().numpy().view(np.uint32)), f"call {it}: logits"
        # and the CPU oracle, bit for bit (ids, gate weights, output row)
        _, no, _, io, wo = oracle.router_addnorm_route(
            h_np, b_np, hw["norm_w"], hw["router"], 0, hw["ebias"] if mode else None, mode)
        act_o = oracle.gemv_gather_act(hw["gate"], hw["up"], no, io, n_experts=E)
        out_o = oracle.gemv_gather_down_combine4(hw["down"], act_o, io, wo, n_experts=E)
        assert np.array_equal(host_u32(b["ids"]), io), f"call {it}: ids vs oracle"
        assert np.array_equal(host_bits(b["wts"]), wo), f"call {it}: weights vs oracle"
        assert np.array_equal(host_bits(b["out"]), out_o), f"call {it}: out vs oracle"


def test_noalloc_rejects_wide_experts(cuda_ctx, layer):
    """An expert width above the built-in scratch's 2048 is refused before any
    launch (the weights are never read)."""
    g = synth.rng(5)
    n_exp, wide = 4, 2112
    gate = dev_qw(*synth.quant_weights_np(g, n_exp * wide, H))
    down = dev_qw(*synth.quant_weights_np(g, n_exp * H, wide))
    router = dev_bf16(synth.router_np(g)[:n_exp])
    o = outputs()
    with pytest.raises(_lib.McError, match="built-in scratch"):
        lfm.moe_decode_layer_noalloc(cuda_ctx, dev_bf16(synth.activations_np(g, 1, H)), None,
                                     layer["norm_w"], o["hout"], o["normed"], router,
                                     o["logits"][:, :n_exp], None, o["ids"], o["wts"], gate,
                                     gate, down, o["out"], n_experts=n_exp)
