"""Expert-parallel prefill on two GPUs (NCCL): every rank's output against the
CPU oracle run on that rank's tokens with all experts. Needs 2 GPUs; with
fewer it is skipped (the host logic is covered on CPU by test_ep_cpu)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


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
        results = []
        for _ in range(2):  # twice: buffers and plans are rebuilt every step
            out, plan = ep.moe_prefill_ep(ops, synth.bf16_tensor(x).cuda(),
                                          torch.from_numpy(logits).cuda(), rank, world)
            torch.cuda.synchronize()
            results.append(synth.tensor_bits(out))
        assert int(ops.status.cpu()[0]) == 0, "grouped GEMM status"
        want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)
        for r in results:
            assert_out_close(r, want, f"rank {rank} out")
        assert np.array_equal(results[0], results[1]), "two identical steps differ"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, True, plan.recv_rows))
    except Exception as exc:
        q.put((rank, False, repr(exc)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


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
