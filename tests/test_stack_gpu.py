"""BASELINE cfg4's stacked decode loop (molten_b200.stack) on a small stack:
every step's argmax tokens equal the CPU oracle's bit for bit, eagerly and
when one step is captured in a CUDA graph and replayed (token fed back on the
device)."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import synth
from molten_b200.stack import DecodeStack
from tests.gpu_util import dev_bf16, dev_qw

pytestmark = pytest.mark.gpu

H = 2048


def make_stack(seed, L, E, I, V):
    g = synth.rng(seed)
    layers = []
    for _ in range(L):
        layers.append(dict(proj=synth.quant_weights_np(g, H, H), norm_w=synth.norm_weight_np(g),
                           router=synth.router_np(g, E), gate=synth.quant_weights_np(g, E * I, H),
                           up=synth.quant_weights_np(g, E * I, H),
                           down=synth.quant_weights_np(g, E * H, I)))
    head = synth.quant_weights_np(g, V, H, 6)
    embed = synth.activations_np(g, V, H)
    return layers, head, embed


def oracle_tokens(layers, head, embed, toks, steps, E):
    out = []
    for _ in range(steps):
        x = embed[toks]
        for L in layers:
            p = oracle.gemv_quant(*L["proj"], 4, x)
            _, normed, _, ids, wts = oracle.router_addnorm_route(x, p, L["norm_w"], L["router"], 0,
                                                                 None, 0)
            act = oracle.gemv_gather_act(L["gate"], L["up"], normed, ids, n_experts=E)
            x = oracle.gemv_gather_down_combine4(L["down"], act, ids, wts, n_experts=E)
        _, toks = oracle.head_argmax(*head, 6, x)
        out.append(toks.copy())
    return out


@pytest.mark.parametrize("batch", [1, 3])
def test_stacked_decode_matches_oracle(cuda_ctx, batch):
    L, E, I, V, steps = 3, 8, 512, 4096, 3
    layers, head, embed = make_stack(80 + batch, L, E, I, V)
    start = np.arange(7, 7 + batch, dtype=np.uint32) * 37 % V
    want = oracle_tokens(layers, head, embed, start, 2 * steps, E)
    dl = [dict(proj=dev_qw(*l["proj"]), norm_w=dev_bf16(l["norm_w"]), router=dev_bf16(l["router"]),
               gate=dev_qw(*l["gate"]), up=dev_qw(*l["up"]), down=dev_qw(*l["down"])) for l in layers]
    # batch 1: the fused layer; batch 3: the per-token GEMV path (both bit-exact)
    st = DecodeStack(cuda_ctx, dl, dev_qw(*head, bits=6), dev_bf16(embed), batch, n_experts=E,
                     moe_path="fused" if batch == 1 else "gemv")
    st.start(torch.from_numpy(start.view(np.int32)).cuda())
    for s in range(steps):  # eager
        st.step()
        torch.cuda.synchronize()
        got = st.read_tokens().numpy().view(np.uint32)
        assert np.array_equal(got, want[s]), f"step {s}: {got} != {want[s]}"
    assert int(st.keys.abs().sum().cpu()) == 0, "token tail leaves the keys cleared"
    g = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            st.step()
    torch.cuda.current_stream().wait_stream(stream)
    # capture records the step without running it; replays continue the sequence
    for s in range(steps, 2 * steps):
        g.replay()
        torch.cuda.synchronize()
        got = st.read_tokens().numpy().view(np.uint32)
        assert np.array_equal(got, want[s]), f"graph step {s}: {got} != {want[s]}"


def test_stacked_decode_grouped_path(cuda_ctx):
    """The batched decode's tensor-core expert path (moe_prefill per layer),
    teacher-forced from the bit-exact GEMV path's tokens every step: the
    hidden rows after the last layer agree within the prefill tolerance, and
    the greedy tokens agree except on near-ties of the head (checked on the
    oracle's head values of the GEMV path's rows)."""
    L, E, I, V, steps, batch = 3, 8, 512, 4096, 3, 5
    layers, head, embed = make_stack(91, L, E, I, V)
    dl = [dict(proj=dev_qw(*l["proj"]), norm_w=dev_bf16(l["norm_w"]), router=dev_bf16(l["router"]),
               gate=dev_qw(*l["gate"]), up=dev_qw(*l["up"]), down=dev_qw(*l["down"])) for l in layers]
    stacks = {p: DecodeStack(cuda_ctx, dl, dev_qw(*head, bits=6), dev_bf16(embed), batch,
                             n_experts=E, moe_path=p) for p in ("gemv", "grouped")}
    toks = torch.from_numpy((np.arange(batch, dtype=np.uint32) * 53 % V).view(np.int32)).cuda()
    for s in range(steps):
        for st in stacks.values():
            st.start(toks)
            st.step()
        torch.cuda.synchronize()
        a = stacks["gemv"].outs[(L - 1) % 2].float()
        b = stacks["grouped"].outs[(L - 1) % 2].float()
        rms = float(a.pow(2).mean().sqrt())
        err = float((a - b).abs().max())
        assert err <= 2e-2 * rms + 2e-2 * float(a.abs().max()), f"step {s}: max err {err}, rms {rms}"
        ta = stacks["gemv"].read_tokens().numpy().view(np.uint32)
        tb = stacks["grouped"].read_tokens().numpy().view(np.uint32)
        for r in np.nonzero(ta != tb)[0]:
            x = stacks["gemv"].outs[(L - 1) % 2][r:r + 1].contiguous().view(torch.int16).cpu().numpy()
            v = synth.bf16_bits_to_f32(oracle.gemv_quant(*head, 6, x.view(np.uint16))[0])
            gap = float(v[ta[r]] - v[tb[r]])
            assert 0.0 <= gap <= 2e-2 * float(np.abs(v).max()), f"step {s} row {r}: gap {gap}"
        toks = stacks["gemv"].tokens.clone()
    assert stacks["grouped"].launches_per_step() == L * 9 + 2


def test_stacked_decode_with_sampling_matches_oracle(cuda_ctx):
    """The sampled decode loop (batch 1, top-k + top-p + repetition penalty):
    every step's token equals the oracle's draw on the oracle's head logits,
    eagerly and when one step is captured in a CUDA graph and replayed (the
    position and the seen set advance on the device)."""
    from molten_b200.sample import Sampling
    L, E, I, V, steps = 2, 8, 512, 4096, 3
    layers, head, embed = make_stack(97, L, E, I, V)
    dl = [dict(proj=dev_qw(*l["proj"]), norm_w=dev_bf16(l["norm_w"]), router=dev_bf16(l["router"]),
               gate=dev_qw(*l["gate"]), up=dev_qw(*l["up"]), down=dev_qw(*l["down"])) for l in layers]
    s = Sampling(temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.3, seed=2024)
    st = DecodeStack(cuda_ctx, dl, dev_qw(*head, bits=6), dev_bf16(embed), 1, n_experts=E,
                     moe_path="fused", sampling=s)
    tok, pos, seen = 123, 17, [5, 99, 123]
    st.start(torch.tensor([tok], dtype=torch.int32).cuda(), pos=pos, seen=seen[:-1])
    seen_bits = np.zeros(V // 32, np.uint32)
    for t in seen:
        seen_bits[t >> 5] |= np.uint32(1 << (t & 31))

    def oracle_next(tok, pos):
        x = embed[[tok]]
        for Lw in layers:
            p = oracle.gemv_quant(*Lw["proj"], 4, x)
            _, normed, _, ids, wts = oracle.router_addnorm_route(x, p, Lw["norm_w"], Lw["router"],
                                                                 0, None, 0)
            act = oracle.gemv_gather_act(Lw["gate"], Lw["up"], normed, ids, n_experts=E)
            x = oracle.gemv_gather_down_combine4(Lw["down"], act, ids, wts, n_experts=E)
        logits = oracle.gemv_quant(*head, 6, x)[0]
        key, _ = oracle.sample_draw(logits, seen_bits, 0.8, 40, 0.9, 1.3, 2024, pos)
        return (~key) & 0xffffffff

    g = None
    for s_i in range(2 * steps):
        want = oracle_next(tok, pos)
        if s_i < steps:
            st.step()
        else:
            if g is None:
                g = torch.cuda.CUDAGraph()
                stream = torch.cuda.Stream()
                stream.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g, stream=stream):
                        st.step()
                torch.cuda.current_stream().wait_stream(stream)
            g.replay()
        torch.cuda.synchronize()
        got = int(st.read_tokens().numpy().view(np.uint32)[0])
        assert got == want, f"step {s_i}: {got} != {want}"
        tok, pos = got, pos + 1
        seen_bits[tok >> 5] |= np.uint32(1 << (tok & 31))
        assert int(st.pos.cpu()[0]) == pos
