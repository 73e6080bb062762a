"""Expert-parallel prefill (molten_b200.ep) on CPU: the exchange plan's
invariants, and a two-rank gloo run whose compute steps are the oracle's,
checked bit for bit against the one-device oracle on each rank's tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from molten_b200 import ep, synth


def random_counts(g, world, E, pairs):
    c = np.zeros((world, E), np.int64)
    for s in range(world):
        p = g.dirichlet(np.full(E, 0.3))
        c[s] = g.multinomial(pairs, p)
    return c


@pytest.mark.parametrize("world,E", [(1, 8), (2, 8), (4, 64), (8, 64)])
def test_plan_invariants(world, E):
    g = synth.rng(500 + world)
    counts = random_counts(g, world, E, 4 * 300)
    plans = [ep.plan_exchange(counts, r) for r in range(world)]
    per = E // world
    for r, p in enumerate(plans):
        # sends cover this rank's sorted rows exactly once, in order
        off = 0
        for peer, o, n in p.send:
            assert o == off and n > 0
            off += n
        assert off == counts[r].sum()
        # received rows: every local expert's rows contiguous, all covered
        assert p.recv_rows == counts[:, r * per:(r + 1) * per].sum()
        covered = np.zeros(p.recv_rows, np.int32)
        for peer, o, n in p.recv:
            covered[o:o + n] += 1
        assert (covered == 1).all()
        # tiles: <= 256 rows of one local expert, cover every received row once
        cov = np.zeros(p.recv_rows, np.int32)
        for m0, m1, j, _ in p.tiles:
            assert 0 < m1 - m0 <= ep.CHUNK and j < per
            assert p.local_offsets[j] <= m0 and m1 <= p.local_offsets[j] + p.local_counts[j]
            cov[m0:m1] += 1
        assert (cov == 1).all()
        heights = [int(t[1] - t[0]) for t in p.tiles]
        nfull = sum(h == ep.CHUNK for h in heights)
        assert heights[:nfull] == [ep.CHUNK] * nfull
        assert heights[nfull:] == sorted(heights[nfull:], reverse=True)
    # the i-th send from s to r pairs with the i-th receive at r from s
    for s in range(world):
        for r in range(world):
            sends = [n for peer, _, n in plans[s].send if peer == r]
            recvs = [n for peer, _, n in plans[r].recv if peer == s]
            assert sends == recvs


class OracleOps(ep.Ops):
    """The CPU oracle as the compute steps of one rank (test only)."""

    def __init__(self, gate, up, down, E, rank, world):
        per = E // world
        self.E, self.per = E, per
        sl = lambda w, rows: tuple(a[rank * per * rows:(rank + 1) * per * rows] for a in w)
        I, H = gate[0].shape[0] // E, down[0].shape[0] // E
        self.gate, self.up, self.down = sl(gate, I), sl(up, I), sl(down, H)

    def route(self, logits):
        ids, gw = oracle.moe_route_batch(logits.numpy())
        return ids, gw

    def sort(self, ids, m):
        counts, offsets, ids_sorted, slotpos = oracle.moe_sort(ids, self.E)
        return torch.from_numpy(counts.view(np.int32).copy()), slotpos, ids_sorted

    def gather(self, x, ids_sorted):
        return synth.bf16_tensor(oracle.gather_rows(synth.tensor_bits(x), ids_sorted))

    def ffn(self, rows, plan):
        a = synth.tensor_bits(rows[:plan.recv_rows])
        c, o = plan.local_counts, plan.local_offsets
        g = oracle.gemm_q4_grouped(a, self.gate, c, o, self.per)
        u = oracle.gemm_q4_grouped(a, self.up, c, o, self.per)
        act = oracle.silu_mul(g, u)
        ed = oracle.gemm_q4_grouped(act, self.down, c, o, self.per)
        return synth.bf16_tensor(ed) if ed.size else rows[:1].clone()

    def combine(self, ed, slotpos, gw, m):
        return oracle.moe_combine(synth.tensor_bits(ed), slotpos, gw, m, ed.shape[1])

    def empty_rows(self, n, like):
        return torch.zeros((n, like.shape[1]), dtype=torch.bfloat16)


def _rank_main(rank, world, port, E, m, I, q):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = synth.rng(900)
        H = 2048
        gate = synth.quant_weights_np(g, E * I, H)
        up = synth.quant_weights_np(g, E * I, H)
        down = synth.quant_weights_np(g, E * H, I)
        gr = synth.rng(910 + rank)
        x = synth.activations_np(gr, m, H)
        logits = synth.zipf_logits_np(gr, m, E)
        ops = OracleOps(gate, up, down, E, rank, world)
        out, plan = ep.moe_prefill_ep(ops, synth.bf16_tensor(x), torch.from_numpy(logits), rank,
                                      world)
        want = oracle.moe_prefill(x, logits, gate, up, down, n_experts=E)["out"]
        ok = bool(np.array_equal(np.asarray(out), want))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, plan.recv_rows))
    except Exception as exc:  # reported to the parent
        q.put((rank, False, repr(exc)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_multi_rank_gloo_matches_one_device_oracle(world):
    """The host-side expert-parallel step on `world` gloo ranks (CPU, oracle
    arithmetic per rank) equals the one-device oracle."""
    E, m, I = 8, 48, 256
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, E, m, I, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in sorted(results, key=lambda t: t[0]):
        assert ok, f"rank {rank}: {info}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_placement_balances_zipf_load(world):
    """Greedy placement: every rank gets E/world distinct experts, and on a
    Zipf load the heaviest rank carries less than with contiguous ranges."""
    E = 64
    g = synth.rng(700 + world)
    load = 1.0 / (1 + g.permutation(E))            # Zipf(1) over a random order
    table, experts = ep.place_experts(load, world)
    assert sorted(table.tolist()) == list(range(E))
    per = E // world
    for r, ex in enumerate(experts):
        assert len(ex) == per
        for j, e in enumerate(ex):
            assert table[e] == r * per + j
    placed = max(load[ex].sum() for ex in experts)
    contiguous = max(load[r * per:(r + 1) * per].sum() for r in range(world))
    assert placed <= contiguous + 1e-12
    # a bound of greedy packing: within the heaviest expert of the ideal share
    assert placed <= load.sum() / world + load.max() + 1e-12


def _failing_rank_main(rank, world, port, mode, q):
    """Step 1 on both ranks; before step 2 rank 1 either raises (its process
    ends) or stays away from the step; rank 0 must see its next collective
    fail within the process group's short timeout instead of hanging."""
    import datetime
    import time as _t
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        E, m, I, H = 8, 16, 128, 2048
        g = synth.rng(920)
        gate, up = synth.quant_weights_np(g, E * I, H), synth.quant_weights_np(g, E * I, H)
        down = synth.quant_weights_np(g, E * H, I)
        gr = synth.rng(930 + rank)
        x, logits = synth.activations_np(gr, m, H), synth.zipf_logits_np(gr, m, E)
        ops = OracleOps(gate, up, down, E, rank, world)
        ep.moe_prefill_ep(ops, synth.bf16_tensor(x), torch.from_numpy(logits), rank, world)
        if rank == 1:
            if mode == "raise":
                raise RuntimeError("injected failure between steps")
            _t.sleep(20)          # alive, but never joins step 2
            q.put((rank, True, "stayed away"))
            return
        t0 = _t.time()
        try:
            ep.moe_prefill_ep(ops, synth.bf16_tensor(x), torch.from_numpy(logits), rank, world)
            q.put((rank, False, "step 2 completed without its peer"))
        except Exception as exc:  # the collective with the missing rank fails
            q.put((rank, True, f"{type(exc).__name__} after {_t.time() - t0:.1f} s"))
    except Exception as exc:
        q.put((rank, mode == "raise" and rank == 1, repr(exc)))


@pytest.mark.parametrize("mode", ["raise", "absent"])
def test_a_failed_rank_makes_the_others_fail_cleanly(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, world, port, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in range(world):
            rank, ok, info = q.get(timeout=120)
            results[rank] = (ok, info)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    ok0, info0 = results[0]
    assert ok0, f"rank 0: {info0}"
    secs = float(info0.split(" after ")[1].split(" s")[0])
    assert secs < 60.0, f"rank 0 took {secs} s to notice"
