"""Expert-parallel prefill driven through the C ABI alone
(mc_ep_init / mc_ep_reserve / mc_ep_place / mc_ep_moe_prefill): a
one-rank communicator on one GPU (plain and with replicated slots), a
barrier made to run out on purpose (status bit 8, the context usable after),
and a two-GPU run (skipped on one GPU). Every rank's output is checked
against the CPU oracle's prefill of that rank's tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H = 2048


def _layer(seed, E, I):
    from molten_b200 import synth
    g = synth.rng(seed)
    return (synth.quant_weights_np(g, E * I, H), synth.quant_weights_np(g, E * I, H),
            synth.quant_weights_np(g, E * H, I))


def _tokens(seed, m, E):
    from molten_b200 import synth
    g = synth.rng(seed)
    return synth.activations_np(g, m, H), synth.zipf_logits_np(g, m, E)


def _run_rank(ctx, rank, world, x, logits, weights, E, I, spr, load, steps=2):
    """Sets up expert parallelism on ctx and runs `steps` steps; returns the
    outputs (host bf16 bits), the status and the counts of the last step."""
    from molten_b200 import ep, synth
    from tests.gpu_util import dev_qw
    epp = ep.EpPrefill(ctx, rank, world)
    try:
        epp.reserve(x.shape[0], E, spr, H, I)
        tables, slot_expert = ep.place_slots(load, world, spr)
        mine = slot_expert[rank * spr:(rank + 1) * spr]
        full = [dev_qw(*w) for w in weights]
        gate, up, down = (ep.slot_weights(w, mine, E) for w in full)
        table = torch.from_numpy(tables[rank].view(np.int32).copy()).cuda()
        xd, ld = synth.bf16_tensor(x).cuda(), torch.from_numpy(logits).cuda()
        outs = []
        for _ in range(steps):
            out = torch.empty((x.shape[0], H), dtype=torch.bfloat16, device="cuda")
            epp.step(xd, ld, gate, up, down, table, out)
            outs.append(synth.tensor_bits(out))
        return outs, epp.status(), epp.counts()
    finally:
        epp.finalize()


@pytest.mark.parametrize("E,I,m,spr", [(8, 256, 96, 8), (8, 256, 200, 11)])
def test_one_rank_ep_through_the_c_abi(E, I, m, spr):
    import oracle
    from molten_b200 import lfm
    from tests.test_grouped_gemm_gpu import assert_out_close
    weights = _layer(3100 + spr, E, I)
    x, logits = _tokens(3200 + m, m, E)
    load = np.bincount(oracle.moe_route_batch(logits)[0].ravel(), minlength=E)[None, :]
    ctx = lfm.Context(0)
    try:
        outs, status, counts = _run_rank(ctx, 0, 1, x, logits, weights, E, I, spr, load)
    finally:
        ctx.close()
    assert status == 0, f"status {status}"
    assert counts.sum() == 4 * m
    want = oracle.moe_prefill(x, logits, *weights, n_experts=E)
    for o in outs:
        assert_out_close(o, want, "ep world 1")
    assert np.array_equal(outs[0], outs[1]), "identical steps give identical rows"


def test_ep_barrier_wait_runs_out_and_the_next_step_succeeds():
    """One rank that does not arrive at its barriers (test flag) with a 1 ms
    limit: the step ends with status bit 8 instead of hanging; after the
    flag is cleared the next step is correct."""
    import oracle
    from molten_b200 import _lib, ep, lfm, synth
    from tests.gpu_util import dev_qw
    from tests.test_grouped_gemm_gpu import assert_out_close
    E, I, m = 8, 256, 64
    weights = _layer(3300, E, I)
    x, logits = _tokens(3301, m, E)
    ctx = lfm.Context(0)
    epp = ep.EpPrefill(ctx, 0, 1)
    try:
        epp.reserve(m, E, E, H, I)
        tables, slot_expert = ep.place_slots(np.ones((1, E), np.uint64), 1, E)
        gate, up, down = (ep.slot_weights(dev_qw(*w), slot_expert, E) for w in weights)
        table = torch.from_numpy(tables[0].view(np.int32).copy()).cuda()
        xd, ld = synth.bf16_tensor(x).cuda(), torch.from_numpy(logits).cuda()
        out = torch.empty((m, H), dtype=torch.bfloat16, device="cuda")
        ctx.set_wait_limit(1_000_000)
        ctx.set_test_flags(_lib.TEST_SKIP_BARRIER_ARRIVE)
        epp.step(xd, ld, gate, up, down, table, out)
        assert epp.status() & 8, "the barrier reported giving up"
        ctx.set_test_flags(0)
        ctx.set_wait_limit(0)
        epp.step(xd, ld, gate, up, down, table, out)
        assert epp.status() == 0
        want = oracle.moe_prefill(x, logits, *weights, n_experts=E)
        assert_out_close(synth.tensor_bits(out), want, "after recovery")
    finally:
        ctx.set_test_flags(0)
        ctx.set_wait_limit(0)
        epp.finalize()
        ctx.close()


def _rank_main(rank, world, port, spr, q):
    try:
        import datetime
        import torch.distributed as dist
        import oracle
        from molten_b200 import build, lfm
        from tests.test_grouped_gemm_gpu import assert_out_close
        build.build()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        E, I, m = 8, 256, 96
        weights = _layer(3400, E, I)
        toks = [_tokens(3410 + r, m, E) for r in range(world)]
        load = np.stack([np.bincount(oracle.moe_route_batch(l)[0].ravel(), minlength=E)
                         for _, l in toks])
        x, logits = toks[rank]
        ctx = lfm.Context(rank)
        outs, status, counts = _run_rank(ctx, rank, world, x, logits, weights, E, I, spr, load)
        ctx.close()
        assert status == 0, f"status {status}"
        want = oracle.moe_prefill(x, logits, *weights, n_experts=E)
        for o in outs:
            assert_out_close(o, want, f"rank {rank}")
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, int(counts.sum())))
    except Exception as exc:
        q.put((rank, False, repr(exc)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.multigpu
@pytest.mark.parametrize("spr", [4, 5])
def test_two_gpu_ep_through_the_c_abi(spr):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, spr, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, info in sorted(results, key=lambda t: t[0]):
        assert ok, f"rank {rank}: {info}"
