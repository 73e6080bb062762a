"""Expert-parallel prefill: the peer-memory exchange kernels with W ranks
emulated on one GPU, and a real two-GPU run (NCCL point-to-point exchange and
the peer-memory exchange over NVLink). Every rank's output is checked against
the CPU oracle run on that rank's tokens with all experts."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _case(seed_w, seeds, ms, E, I, H=2048):
    from molten_b200 import synth
    g = synth.rng(seed_w)
    gate = synth.quant_weights_np(g, E * I, H)
    up = synth.quant_weights_np(g, E * I, H)
    down = synth.quant_weights_np(g, E * H, I)
    toks = []
    for sd, m in zip(seeds, ms):
        gr = synth.rng(sd)
        toks.append((synth.activations_np(gr, m, H), synth.zipf_logits_np(gr, m, E)))
    return gate, up, down, toks


@pytest.mark.parametrize("world,ms,placed", [(2, (48, 30), False), (4, (64, 17, 40, 5), False),
                                              (4, (64, 33, 20, 50), True)])
def test_ep_peer_kernels_emulated_on_one_gpu(cuda_ctx, world, ms, placed):
    """placed: a load-balanced expert placement (experts no longer in
    contiguous ranges, ids relabelled on the device before sorting)."""
    import oracle
    from molten_b200 import ep, synth
    from tests.gpu_util import dev_qw
    from tests.test_grouped_gemm_gpu import assert_out_close
    E, I = 8, 256
    gate, up, down, toks = _case(950, [960 + r for r in range(world)], ms, E, I)
    xs = [synth.bf16_tensor(x).cuda() for x, _ in toks]
    lg = [torch.from_numpy(l).cuda() for _, l in toks]
    placement = None
    if placed:
        load = np.zeros(E)
        for _, l in toks:
            ids, _ = oracle.moe_route_batch(l)
            load += np.bincount(ids.ravel(), minlength=E)
        placement = ep.place_experts(load, world)
        assert placement[0].tolist() != list(range(E))
    outs, status = ep.moe_prefill_ep_emulated(cuda_ctx, xs, lg, dev_qw(*gate), dev_qw(*up),
                                              dev_qw(*down), E, placement)
    assert status == 0
    for r, (x, l) in enumerate(toks):
        want = oracle.moe_prefill(x, l, gate, up, down, n_experts=E)
        assert_out_close(synth.tensor_bits(outs[r]), want, f"emulated rank {r}")


def _rank_main(rank, world, port, q):
    try:
        import torch.distributed as dist
        import oracle
        from molten_b200 import build, ep, lfm, synth
        from tests.gpu_util import dev_qw
        from tests.test_grouped_gemm_gpu import assert_out_close
        build.build()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        E, H, I, m = 8, 2048, 256, 96
        g = synth.rng(930)
        gate = synth.quant_weights_np(g, E * I, H)
        up = synth.quant_weights_np(g, E * I, H)
        down = synth.quant_weights_np(g, E * H, I)
        gr = synth.rng(940 + rank)
        x = synth.activations_np(gr, m, H)
        logits = synth.zipf_logits_np(gr, m, E)
        ctx = lfm.Context(rank)
        full = {k: dev_qw(*w) for k, w in (("gate", gate), ("up", up), ("down", down))}
        sl = {k: ep.expert_slice(w, rank, world, E) for k, w in full.items()}
        ops = ep.CudaOps(ctx, sl["gate"], sl["up"], sl["down"], E, rank, world)
        xd, ld = synth.bf16_tensor(x).cuda(), torch.from_numpy(logits).cuda()
        results = []
        for _ in range(2):  # NCCL point-to-point exchange, twice (plans rebuilt each step)
            out, plan = ep.moe_prefill_ep(ops, xd, ld, rank, world)
            torch.cuda.synchronize()
            results.append(synth.tensor_bits(out))
        px = ep.PeerExchange(ctx, rank, world, m, H, I, E)
        for _ in range(2):  # peer-memory exchange over NVLink, twice (buffers reused)
            out = ep.moe_prefill_ep_peer(ops, px, xd, ld)
            torch.cuda.synchronize()
            results.append(synth.tensor_bits(out))
        peer_status = int(px.status.cpu()[0])
        px.close()
        assert int(ops.status.cpu()[0]) == 0 and peer_status == 0, "status"
        want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
        for r in results:
            assert_out_close(r, want, f"rank {rank} out")
        for r in results[1:]:
            assert np.array_equal(results[0], r), "identical steps differ"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, plan.recv_rows))
    except Exception as exc:
        q.put((rank, False, repr(exc)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.multigpu
def test_two_gpu_expert_parallel_prefill():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, info in sorted(results, key=lambda t: t[0]):
        assert ok, f"rank {rank}: {info}"
