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
                 route_mode: int = 0, bias=None, placement=None):
        """gate/up/down: this rank's experts only (in placement order when a
        placement table -- model expert -> position, see place_experts -- is
        given; contiguous expert ranges otherwise)."""
        from molten_b200 import _lib, lfm
        self.lfm, self.lib, self.ctx = lfm, _lib, ctx
        self.E, self.per = n_experts, n_experts // world
        self.gate, self.up, self.down = gate, up, down
        self.route_mode, self.bias = route_mode, bias
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.table = None
        if placement is not None:
            self.table = torch.from_numpy(np.asarray(placement, np.uint32).view(np.int32)).cuda()

    def route(self, logits):
        m = logits.shape[0]
        ids = torch.zeros((m, 4), dtype=torch.int32, device="cuda")
        gw = torch.empty((m, 4), dtype=torch.bfloat16, device="cuda")
        self.lfm.moe_route_batch(self.ctx, logits, self.bias, ids, gw, m, route_mode=self.route_mode)
        if self.table is not None:  # route on model ids, sort by placement position
            self.lib.call("mc_map_ids", self.ctx.handle, ids.data_ptr(), ids.numel(),
                          self.table.data_ptr(), self.E, self.status.data_ptr())
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


def place_experts(load, world: int):
    """Skew-aware expert placement: experts by decreasing measured load, each
    to the rank with the least load so far among those with a free slot
    (every rank gets E/world experts; ties go to the lower rank). Returns
    (table[e] = position of model expert e in the rank-contiguous order,
    experts[r] = the model experts of rank r in position order)."""
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    per = E // world
    rank_load = np.zeros(world)
    experts = [[] for _ in range(world)]
    for e in np.argsort(-load, kind="stable"):
        free = [r for r in range(world) if len(experts[r]) < per]
        r = min(free, key=lambda q: (rank_load[q], q))
        experts[r].append(int(e))
        rank_load[r] += load[e]
    table = np.zeros(E, np.uint32)
    for r in range(world):
        for j, e in enumerate(experts[r]):
            table[e] = r * per + j
    return table, experts


def placed_slice(w, experts, n_experts: int):
    """The stacked rows of `experts` (in that order) of a [E*N][K] QuantWeights
    (a copy: a placement's experts need not be adjacent)."""
    from molten_b200.quant import QuantWeights
    rows = w.codes.shape[0] // n_experts
    pick = lambda t: torch.cat([t[e * rows:(e + 1) * rows] for e in experts]).contiguous()
    return QuantWeights(pick(w.codes), pick(w.scales), pick(w.biases), w.group_size, w.bits)


def expert_slice(w, rank: int, world: int, n_experts: int):
    """This rank's experts of a stacked [E*N][K] QuantWeights (a view)."""
    from molten_b200.quant import QuantWeights
    per = n_experts // world
    rows = w.codes.shape[0] // n_experts
    r0, r1 = rank * per * rows, (rank + 1) * per * rows
    return QuantWeights(w.codes[r0:r1], w.scales[r0:r1], w.biases[r0:r1], w.group_size, w.bits)


# ----------------------------------------------------------- peer-memory exchange
# The rows move by the library's own copy kernels straight into the other
# ranks' buffers over NVLink (CUDA IPC mappings); the counts, the receive
# layout and the GEMM row chunks are derived on the device from the gathered
# counts, so a step needs no host synchronisation.

class _DevBuf:
    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3, "strides": None}


def _rows_view(ptr: int, rows: int, hidden: int) -> torch.Tensor:
    t = torch.as_tensor(_DevBuf(ptr, rows * hidden * 2), device="cuda")
    return t.view(torch.bfloat16).view(rows, hidden)


def _ptr_table(ptrs):
    import ctypes as C
    return (C.c_void_p * len(ptrs))(*ptrs)


class PeerExchange:
    """Receive and home row buffers of every rank, mapped into this process.
    All ranks use the same capacities: receive = world * 4 * m_max rows (the
    case of every pair routed to one rank), home = 4 * m_max rows."""

    def __init__(self, ctx, rank: int, world: int, m_max: int, hidden: int, moe_inter: int,
                 n_experts: int, group=None):
        import ctypes as C
        from molten_b200 import _lib
        self.lib, self.ctx, self.rank, self.world, self.group = _lib, ctx, rank, world, group
        self.H, self.E, self.per = hidden, n_experts, n_experts // world
        self.recv_cap, self.home_cap = world * 4 * m_max, 4 * m_max
        own = []
        for rows in (self.recv_cap, self.home_cap):
            p = C.c_void_p()
            _lib.call("mc_ep_alloc", ctx.handle, rows * hidden * 2, C.byref(p))
            own.append(p.value)
        self.own = own
        handles = []
        for p in own:
            h = (C.c_char * 64)()
            _lib.call("mc_ipc_handle", ctx.handle, p, h)
            handles.append(bytes(h))
        every = [None] * world
        dist.all_gather_object(every, handles, group=group)
        self.opened = []
        self.recv_ptrs, self.home_ptrs = [], []
        for r in range(world):
            for k, table in enumerate((self.recv_ptrs, self.home_ptrs)):
                if r == rank:
                    table.append(own[k])
                else:
                    p = C.c_void_p()
                    hb = (C.c_char * 64).from_buffer_copy(every[r][k])
                    _lib.call("mc_ipc_open", ctx.handle, hb, C.byref(p))
                    self.opened.append(p.value)
                    table.append(p.value)
        self.recv = _rows_view(own[0], self.recv_cap, hidden)
        self.home = _rows_view(own[1], self.home_cap, hidden)
        dev = "cuda"
        self.act = torch.empty((self.recv_cap, moe_inter), dtype=torch.bfloat16, device=dev)
        self.ed = torch.empty((self.recv_cap, hidden), dtype=torch.bfloat16, device=dev)
        self.max_tiles = self.recv_cap // CHUNK + self.per + 1
        self.tiles = torch.zeros((self.max_tiles, 4), dtype=torch.int32, device=dev)
        self.n_tiles = torch.zeros(1, dtype=torch.int32, device=dev)
        self.rows = torch.zeros(1, dtype=torch.int32, device=dev)
        self.counts_all = torch.zeros((world, n_experts), dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self._recv_tab, self._home_tab = _ptr_table(self.recv_ptrs), _ptr_table(self.home_ptrs)

    def barrier(self):
        """In-stream cross-rank barrier: every rank's earlier kernels finished."""
        dist.all_reduce(self.flag, group=self.group)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.call("mc_ipc_close", self.ctx.handle, p)
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.own:
            self.lib.call("mc_ep_free", self.ctx.handle, p)
        self.own = []


def moe_prefill_ep_peer(ops: "CudaOps", px: PeerExchange, x: torch.Tensor,
                        logits: torch.Tensor) -> torch.Tensor:
    """One expert-parallel step with the peer-memory exchange (no host sync)."""
    lib, h = px.lib, px.ctx.handle
    m, H = x.shape
    ids, gw = ops.route(logits)
    counts, slotpos, ids_sorted = ops.sort(ids, m)
    dist.all_gather_into_tensor(px.counts_all.view(-1), counts.view(-1), group=px.group)
    lib.call("mc_ep_tiles", h, px.counts_all.data_ptr(), px.rank, px.world, px.E, CHUNK,
             px.tiles.data_ptr(), px.n_tiles.data_ptr(), px.rows.data_ptr(), px.max_tiles)
    lib.call("mc_ep_dispatch", h, x.data_ptr(), m, H, ids_sorted.data_ptr(),
             px.counts_all.data_ptr(), px.rank, px.world, px.E, px._recv_tab, px.recv_cap,
             px.status.data_ptr())
    px.barrier()
    ops.lfm.gemm_q4_grouped_gu(ops.ctx, px.recv, ops.gate, ops.up, px.act, px.tiles, px.n_tiles,
                               px.per, px.status)
    ops.lfm.gemm_q4_grouped(ops.ctx, px.act, ops.down, px.ed, px.tiles, px.n_tiles, px.per,
                            px.status)
    lib.call("mc_ep_return", h, px.ed.data_ptr(), px.recv_cap, H, px.counts_all.data_ptr(),
             px.rank, px.world, px.E, px._home_tab, px.home_cap, px.status.data_ptr())
    px.barrier()
    return ops.combine(px.home[:4 * m], slotpos, gw, m)


def moe_prefill_ep_emulated(ctx, xs, logits, gate, up, down, n_experts: int, placement=None,
                            return_state: bool = False):
    """`world = len(xs)` ranks emulated on ONE GPU with the same device code as
    moe_prefill_ep_peer (dispatch, row chunks, grouped GEMMs on each rank's
    expert slice, return, combine), the ranks' kernels run one after another
    so stream order stands in for the barriers. Returns every rank's output
    and the status word (and, with return_state, each rank's ids, gate
    weights, sorted order and slot positions)."""
    from molten_b200 import _lib, lfm
    world = len(xs)
    E, per = n_experts, n_experts // world
    m_max = max(x.shape[0] for x in xs)
    H = xs[0].shape[1]
    I = gate.out_features // E
    recv_cap, home_cap = world * 4 * m_max, 4 * m_max
    recv = [torch.zeros((recv_cap, H), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    home = [torch.zeros((home_cap, H), dtype=torch.bfloat16, device="cuda") for _ in range(world)]
    recv_tab = _ptr_table([t.data_ptr() for t in recv])
    home_tab = _ptr_table([t.data_ptr() for t in home])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    if placement is None:
        ops = [CudaOps(ctx, expert_slice(gate, r, world, E), expert_slice(up, r, world, E),
                       expert_slice(down, r, world, E), E, r, world) for r in range(world)]
    else:
        table, experts = placement
        ops = [CudaOps(ctx, placed_slice(gate, experts[r], E), placed_slice(up, experts[r], E),
                       placed_slice(down, experts[r], E), E, r, world, placement=table)
               for r in range(world)]
    st = []
    for r in range(world):
        ids, gw = ops[r].route(logits[r])
        counts, slotpos, ids_sorted = ops[r].sort(ids, xs[r].shape[0])
        st.append((gw, counts, slotpos, ids_sorted, ids))
    counts_all = torch.stack([s[1] for s in st]).contiguous()
    max_tiles = recv_cap // CHUNK + per + 1
    eds = []
    for r in range(world):
        _lib.call("mc_ep_dispatch", ctx.handle, xs[r].data_ptr(), xs[r].shape[0], H,
                  st[r][3].data_ptr(), counts_all.data_ptr(), r, world, E, recv_tab, recv_cap,
                  status.data_ptr())
    for r in range(world):
        tiles = torch.zeros((max_tiles, 4), dtype=torch.int32, device="cuda")
        n_tiles = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.call("mc_ep_tiles", ctx.handle, counts_all.data_ptr(), r, world, E, CHUNK,
                  tiles.data_ptr(), n_tiles.data_ptr(), None, max_tiles)
        act = torch.empty((recv_cap, I), dtype=torch.bfloat16, device="cuda")
        ed = torch.empty((recv_cap, H), dtype=torch.bfloat16, device="cuda")
        lfm.gemm_q4_grouped_gu(ctx, recv[r], ops[r].gate, ops[r].up, act, tiles, n_tiles, per,
                               status)
        lfm.gemm_q4_grouped(ctx, act, ops[r].down, ed, tiles, n_tiles, per, status)
        eds.append(ed)
    for r in range(world):
        _lib.call("mc_ep_return", ctx.handle, eds[r].data_ptr(), recv_cap, H, counts_all.data_ptr(),
                  r, world, E, home_tab, home_cap, status.data_ptr())
    outs = [ops[r].combine(home[r][:4 * xs[r].shape[0]], st[r][2], st[r][0], xs[r].shape[0])
            for r in range(world)]
    torch.cuda.synchronize()
    for o in ops:
        status |= o.status
    if return_state:
        inner = [dict(ids=s[4], gw=s[0], ids_sorted=s[3], slotpos=s[2]) for s in st]
        return outs, int(status.cpu()[0]), inner
    return outs, int(status.cpu()[0])


# ------------------------------------------------- the C-ABI expert-parallel step
# The whole step runs inside the library (mc_ep_moe_prefill): routing, slot
# relabelling, sort, the counts exchange and the dispatch over NVLink,
# device-side barriers, the grouped GEMMs, the return and the combine. Python only bootstraps the NCCL unique id and loads each
# rank's slot weights.

def place_slots(load, world: int, slots_per_rank: int):
    """Slot placement with hot-expert replication (mc_ep_place): load[s][e]
    pairs -> (tables u32 [world][E], slot_expert i32 [world * spr])."""
    import ctypes as C
    from molten_b200 import _lib
    load = np.ascontiguousarray(np.asarray(load, dtype=np.uint64))
    W, E = load.shape
    tables = np.zeros((W, E), np.uint32)
    slot_expert = np.zeros(W * slots_per_rank, np.int32)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    _lib.call("mc_ep_place", ptr(load), W, E, slots_per_rank, ptr(tables), ptr(slot_expert))
    return tables, slot_expert


def slot_weights(w, slot_expert_of_rank, n_experts: int):
    """This rank's slot weights: the rows of each slot's expert of a stacked
    [E*N][K] QuantWeights, in slot order (an empty slot repeats expert 0; no
    row is ever routed to it)."""
    return placed_slice(w, [int(e) if e >= 0 else 0 for e in slot_expert_of_rank], n_experts)


class EpPrefill:
    """One rank's expert-parallel prefill through the C ABI."""

    def __init__(self, ctx, rank: int, world: int, timeout_ms: int = 120000, group=None):
        import ctypes as C
        from molten_b200 import _lib
        self.lib, self.ctx, self.rank, self.world = _lib, ctx, rank, world
        uid = (C.c_char * 128)()
        if rank == 0:
            _lib.call("mc_ep_unique_id", uid)
        if world > 1:
            obj = [bytes(uid) if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0, group=group)
            uid = (C.c_char * 128).from_buffer_copy(obj[0])
        _lib.call("mc_ep_init", ctx.handle, world, rank, uid, timeout_ms)
        self.reserved = False

    def reserve(self, m_max: int, n_experts: int, slots_per_rank: int, hidden: int,
                moe_inter: int) -> None:
        self.E, self.spr, self.H, self.I = n_experts, slots_per_rank, hidden, moe_inter
        self.lib.call("mc_ep_reserve", self.ctx.handle, m_max, n_experts, slots_per_rank, hidden,
                      moe_inter)
        self.reserved = True

    def step(self, x, logits, gate, up, down, table, out, route_mode: int = 0, bias=None):
        """x bf16 [m][H], logits f32 [m][E], this rank's slot weights,
        table: device int32 [E] (this rank's row of the placement), out bf16 [m][H]."""
        from molten_b200 import lfm
        m = x.shape[0]
        lfm.ensure(logits.shape == (m, self.E), "logits shape")
        self.lib.call("mc_ep_moe_prefill", self.ctx.handle, lfm._p(x), lfm._p(logits), m,
                      self.lib.C.byref(gate.qw()), self.lib.C.byref(up.qw()),
                      self.lib.C.byref(down.qw()), lfm._p(table), route_mode, lfm._p(bias),
                      lfm._p(out))

    def status(self) -> int:
        import ctypes as C
        v = C.c_uint32(0)
        self.lib.call("mc_ep_status", self.ctx.handle, C.byref(v))
        return int(v.value)

    def counts(self) -> np.ndarray:
        """The last step's pair counts of every rank [world][world * spr]."""
        import ctypes as C
        n = self.world * self.world * self.spr
        a = np.zeros(n, np.uint32)
        self.lib.call("mc_ep_counts", self.ctx.handle, a.ctypes.data_as(C.c_void_p), n)
        return a.reshape(self.world, self.world * self.spr)

    def set_profile(self, on: bool) -> None:
        self.lib.call("mc_ep_set_profile", self.ctx.handle, 1 if on else 0)

    PHASES = ("route_sort", "counts_exchange", "dispatch", "dispatch_barrier", "gemms_return",
              "return_barrier", "combine")

    def phase_ms(self) -> dict:
        """The last profiled step's phase times (ms)."""
        import ctypes as C
        a = (C.c_float * len(self.PHASES))()
        self.lib.call("mc_ep_phase_ms", self.ctx.handle, a)
        return {k: float(v) for k, v in zip(self.PHASES, a)}

    def finalize(self) -> None:
        if self.ctx is not None and self.ctx.h:
            self.lib.call("mc_ep_finalize", self.ctx.handle)
