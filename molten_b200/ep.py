"""Expert-parallel prefill MoE FFN over several GPUs (one process per GPU).

The reference runs the prefill MoE FFN (lfm.rs:847-965, `moe_prefill`) on one
device. Here the 64 experts are split over the ranks -- rank r holds experts
[r*E/N, (r+1)*E/N) -- and each rank keeps its own tokens. One step:

1. route the rank's tokens (top-4) and sort its pairs by expert; because a
   rank's experts are contiguous, the expert-sorted gather buffer is already
   grouped by destination rank;
2. all-gather the per-expert pair counts (N x E integers) so every rank can
   plan the exchange without further messages;
3. send every (destination, expert) segment of rows to its owner, which
   receives them expert-major: all rows of one local expert contiguous, in
   source-rank order;
4. run the grouped gate/up (+SwiGLU) and down GEMMs on the received rows;
5. send the results back to the slots the rows came from;
6. combine at home with the rank's own slot positions and gate weights.

Rows travel as int32 pairs of bf16 values, so the same exchange runs over NCCL
(GPU) and gloo (the CPU tests). Arithmetic per pair is that of the one-device
path, so the result equals `moe_prefill` on each rank's tokens bit for bit
wherever the one-device path is deterministic.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

CHUNK = 256  # token rows per grouped-GEMM chunk


@dataclass
class Plan:
    rank: int
    world: int
    n_experts: int
    per_rank: int                 # experts per rank
    send: list[tuple[int, int, int]]   # (peer, row offset in the send buffer, rows)
    recv: list[tuple[int, int, int]]   # (peer, row offset in the receive buffer, rows)
    recv_rows: int
    local_counts: np.ndarray      # rows per local expert (u32 [per_rank])
    local_offsets: np.ndarray     # first receive row of each local expert
    tiles: np.ndarray             # u32 [T, 4] row chunks {m0, m_end, local expert, 0}


def plan_exchange(counts_all: np.ndarray, rank: int, chunk: int = CHUNK) -> Plan:
    """counts_all[s][e]: pairs of rank s routed to expert e. Segment lists are
    in (peer, expert) order on both sides, so the i-th send from s to r and
    the i-th receive at r from s have the same size."""
    counts_all = np.asarray(counts_all, dtype=np.int64)
    world, E = counts_all.shape
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    mine = counts_all[rank]
    my_off = np.concatenate([[0], np.cumsum(mine)[:-1]])
    send = []
    for peer in range(world):
        for e in range(peer * per, (peer + 1) * per):
            if mine[e]:
                send.append((peer, int(my_off[e]), int(mine[e])))
    e0 = rank * per
    totals = counts_all[:, e0:e0 + per].sum(axis=0)
    base = np.concatenate([[0], np.cumsum(totals)[:-1]])
    recv = []
    for peer in range(world):
        for j in range(per):
            n = counts_all[peer, e0 + j]
            if n:
                off = base[j] + counts_all[:peer, e0 + j].sum()
                recv.append((peer, int(off), int(n)))
    full, part = [], []
    for j in range(per):
        for m0 in range(0, int(totals[j]), chunk):
            t = (int(base[j] + m0), int(base[j] + min(m0 + chunk, totals[j])), j, 0)
            (full if t[1] - t[0] == chunk else part).append(t)
    part.sort(key=lambda t: (-(t[1] - t[0]), t[2]))
    tiles = np.array(full + part, dtype=np.uint32).reshape(-1, 4)
    return Plan(rank, world, E, per, send, recv, int(totals.sum()),
                totals.astype(np.uint32), base.astype(np.uint32), tiles)


def _as_words(rows: torch.Tensor) -> torch.Tensor:
    """bf16 rows [n, H] -> int32 [n, H/2] view (H even) for the wire."""
    return rows.view(torch.int32)


def exchange(src: torch.Tensor, dst: torch.Tensor, outgoing, incoming, rank: int,
             group=None) -> None:
    """Moves row segments: outgoing (peer, row offset in src, rows), incoming
    (peer, row offset in dst, rows). Segments to/from this rank are copied
    locally, in order; the rest go as one batch of point-to-point ops."""
    s, d = _as_words(src), _as_words(dst)
    local_out = [seg for seg in outgoing if seg[0] == rank]
    local_in = [seg for seg in incoming if seg[0] == rank]
    if len(local_out) != len(local_in):
        raise RuntimeError("local segments do not pair up")
    for (_, so, n), (_, do, n2) in zip(local_out, local_in):
        if n != n2:
            raise RuntimeError("local segment sizes differ")
        d[do:do + n].copy_(s[so:so + n])
    ops = []
    for peer, off, n in incoming:
        if peer != rank:
            ops.append(dist.P2POp(dist.irecv, d[off:off + n], peer, group))
    for peer, off, n in outgoing:
        if peer != rank:
            ops.append(dist.P2POp(dist.isend, s[off:off + n], peer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


def gather_counts(counts: torch.Tensor, world: int, group=None) -> np.ndarray:
    """All-gathers every rank's per-expert pair counts -> numpy [world, E]."""
    c = counts.to(torch.int32).reshape(-1).contiguous()
    parts = [torch.empty_like(c) for _ in range(world)]
    dist.all_gather(parts, c, group=group)
    return torch.stack(parts).cpu().numpy().view(np.uint32).astype(np.int64)


class Ops:
    """Compute steps of one rank (the GPU implementation is `CudaOps`)."""

    def route(self, logits):            # -> ids [m,4], gw [m,4]
        raise NotImplementedError

    def sort(self, ids, m):             # -> counts[E], slot positions, sorted token ids
        raise NotImplementedError

    def gather(self, x, ids_sorted):    # -> send rows [4m, H]
        raise NotImplementedError

    def ffn(self, rows, plan):          # -> expert outputs [recv_rows, H]
        raise NotImplementedError

    def combine(self, ed, slotpos, gw, m):  # -> out [m, H]
        raise NotImplementedError

    def empty_rows(self, n, like):      # -> uninitialised rows [n, H] like `like`
        return torch.empty((n, like.shape[1]), dtype=like.dtype, device=like.device)


def moe_prefill_ep(ops: Ops, x: torch.Tensor, logits: torch.Tensor, rank: int, world: int,
                   group=None):
    """One expert-parallel prefill MoE FFN step on this rank's tokens.
    Returns (out rows [m, H], the exchange plan)."""
    m = x.shape[0]
    ids, gw = ops.route(logits)
    counts, slotpos, ids_sorted = ops.sort(ids, m)
    send_rows = ops.gather(x, ids_sorted)
    plan = plan_exchange(gather_counts(counts, world, group), rank)
    recv_rows = ops.empty_rows(max(plan.recv_rows, 1), send_rows)
    exchange(send_rows, recv_rows, plan.send, plan.recv, rank, group)
    ed_recv = ops.ffn(recv_rows, plan)
    ed_home = ops.empty_rows(max(4 * m, 1), send_rows)
    exchange(ed_recv, ed_home, plan.recv, plan.send, rank, group)
    return ops.combine(ed_home, slotpos, gw, m), plan


class CudaOps(Ops):
    """The CUDA kernels of molten_b200 (C ABI) on this rank's expert slice."""

    def __init__(self, ctx, gate, up, down, n_experts: int, rank: int, world: int,
                 route_mode: int = 0, bias=None):
        from molten_b200 import lfm
        self.lfm, self.ctx = lfm, ctx
        self.E, self.per = n_experts, n_experts // world
        self.gate, self.up, self.down = gate, up, down   # this rank's experts only
        self.route_mode, self.bias = route_mode, bias
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def route(self, logits):
        m = logits.shape[0]
        ids = torch.zeros((m, 4), dtype=torch.int32, device="cuda")
        gw = torch.empty((m, 4), dtype=torch.bfloat16, device="cuda")
        self.lfm.moe_route_batch(self.ctx, logits, self.bias, ids, gw, m, route_mode=self.route_mode)
        return ids, gw

    def sort(self, ids, m):
        E, S = self.E, 4 * m
        z = lambda *s: torch.zeros(s, dtype=torch.int32, device="cuda")
        counts, offsets, ids_sorted, slotpos = z(E), z(E), z(S), z(S)
        max_tiles = (S + CHUNK - 1) // CHUNK + E
        tiles, n_tiles = z(max_tiles, 4), z(1)
        self.lfm.moe_sort_map(self.ctx, ids, counts, offsets, ids_sorted, slotpos, tiles, n_tiles,
                              m, CHUNK)
        return counts, slotpos, ids_sorted

    def gather(self, x, ids_sorted):
        out = torch.empty((ids_sorted.numel(), x.shape[1]), dtype=x.dtype, device="cuda")
        self.lfm.gather_rows_bf16(self.ctx, x, ids_sorted, out)
        return out

    def ffn(self, rows, plan):
        n = plan.recv_rows
        H = rows.shape[1]
        I = self.gate.out_features // self.per
        act = torch.empty((max(n, 1), I), dtype=torch.bfloat16, device="cuda")
        ed = torch.empty((max(n, 1), H), dtype=torch.bfloat16, device="cuda")
        if n and plan.tiles.shape[0]:
            tiles = torch.from_numpy(plan.tiles.view(np.int32)).to("cuda")
            n_tiles = torch.tensor([plan.tiles.shape[0]], dtype=torch.int32, device="cuda")
            self.lfm.gemm_q4_grouped_gu(self.ctx, rows[:n], self.gate, self.up, act[:n], tiles,
                                        n_tiles, self.per, self.status)
            self.lfm.gemm_q4_grouped(self.ctx, act[:n], self.down, ed[:n], tiles, n_tiles,
                                     self.per, self.status)
        return ed

    def combine(self, ed, slotpos, gw, m):
        out = torch.empty((m, ed.shape[1]), dtype=torch.bfloat16, device="cuda")
        self.lfm.moe_combine_rows(self.ctx, ed, slotpos, gw, out)
        return out


def expert_slice(w, rank: int, world: int, n_experts: int):
    """This rank's experts of a stacked [E*N][K] QuantWeights (a view)."""
    from molten_b200.quant import QuantWeights
    per = n_experts // world
    rows = w.codes.shape[0] // n_experts
    r0, r1 = rank * per * rows, (rank + 1) * per * rows
    return QuantWeights(w.codes[r0:r1], w.scales[r0:r1], w.biases[r0:r1], w.group_size, w.bits)
