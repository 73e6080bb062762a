"""The sampling draw on the GPU (mc_sample_draw) against the CPU oracle, bit
for bit: the drawn 64-bit key for the temperature-only draw, top-k, top-p,
both, and the repetition penalty, at the BASELINE vocabulary (65536) and the
reference model's (128000), on logits with many bf16 ties; the workspace is
left zeroed, the key folds through the greedy token tail, and the seen set is
extended on the device."""
import numpy as np
import pytest
import torch

import oracle
from molten_b200 import lfm, synth
from molten_b200.sample import Sampling, SampleScratch
from tests.gpu_util import dev_bf16

pytestmark = pytest.mark.gpu

CASES = [  # temperature, top_k, top_p, penalty
    (1.0, 0, 1.0, 1.0),
    (0.7, 50, 1.0, 1.0),
    (1.3, 0, 0.9, 1.0),
    (0.8, 40, 0.6, 1.0),
    (1.0, 1, 1.0, 1.0),
    (0.9, 0, 1e-6, 1.0),
    (1.1, 200, 0.95, 1.3),
    (2.0, 0, 1.0, 0.5),
]


@pytest.mark.parametrize("vocab", [65536, 128000])
@pytest.mark.parametrize("temp,top_k,top_p,pen", CASES)
def test_sample_draw_matches_oracle(cuda_ctx, vocab, temp, top_k, top_p, pen):
    g = synth.rng(vocab + int(temp * 100) + top_k)
    # bf16 logits of a peaked distribution (many exact ties in the tail)
    logits = synth.f32_to_bf16_bits((g.standard_t(4, vocab) * 2.0).astype(np.float32))
    seen_tok = g.integers(0, vocab, 300)
    sc = SampleScratch(cuda_ctx, vocab)
    sc.upload_seen(seen_tok)
    seen_np = sc.seen.cpu().numpy().view(np.uint32)
    s = Sampling(temp, top_k, top_p, pen, seed=(0x1234_5678_9abc_def0 + vocab) % 2 ** 64)
    dl = dev_bf16(logits)
    for pos in (0, 17, 70001):
        best = torch.zeros(1, dtype=torch.int64, device="cuda")
        sc.encode_draw(dl, best, s, pos)
        torch.cuda.synchronize()
        got = int(best.cpu().numpy().view(np.uint64)[0])
        want, _ = oracle.sample_draw(logits, seen_np if pen != 1.0 else None, temp, top_k,
                                     top_p, pen, s.seed, pos)
        assert got == want, f"pos {pos}: key {got:#x} != {want:#x}"
    # the control part (plan and histogram, ahead of the w scratch) is left zero
    assert int(sc.ws[:256 + 2048 * 12].abs().sum()) == 0, "the control words are left zeroed"


def test_sampled_token_feeds_the_token_tail_and_seen_set(cuda_ctx):
    vocab = 65536
    g = synth.rng(5150)
    logits = synth.f32_to_bf16_bits(g.normal(0, 3, vocab).astype(np.float32))
    sc = SampleScratch(cuda_ctx, vocab)
    s = Sampling(1.0, 64, 0.9, 1.5, seed=99)
    best = torch.zeros(1, dtype=torch.int64, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    toks = []
    for pos in range(5):
        sc.encode_draw(dev_bf16(logits), best, s, pos)
        lfm.token_tail(cuda_ctx, best, tok)
        sc.encode_mark(tok)
        torch.cuda.synchronize()
        toks.append(int(tok.cpu()[0]))
        assert int(best.cpu()[0]) == 0, "the token tail clears the key"
    # the oracle, fed the same growing seen set
    seen = np.zeros(vocab // 32, np.uint32)
    for pos, t in enumerate(toks):
        key, _ = oracle.sample_draw(logits, seen, 1.0, 64, 0.9, 1.5, 99, pos)
        assert (~key) & 0xffffffff == t, f"pos {pos}"
        seen[t >> 5] |= np.uint32(1 << (t & 31))
    assert np.array_equal(sc.seen.cpu().numpy().view(np.uint32), seen)
