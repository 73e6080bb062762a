// Expert-parallel prefill exchange over NVLink peer memory (no reference
// counterpart: the reference's moe_prefill, lfm.rs:847-965, runs on one
// device).
//
// Rank r of W holds experts [r*P, (r+1)*P), P = E/W. Every rank has sorted its
// own pairs by expert (mc_moe_sort_map) and all ranks share the pair counts
// counts_all[W][E] (an all-gather). From those counts alone every rank
// derives the same layout, with no further messages:
//   * receive buffer of owner r: expert-major -- the rows of its local expert
//     j contiguous from base_r[j] = sum_{j'<j} total_r[j'], and within them
//     the rows of source s from base_r[j] + sum_{s'<s} counts_all[s'][r*P+j];
//   * the rows of source s, expert e sit in s's own sorted order at
//     off_s[e] = sum_{e'<e} counts_all[s][e'].
// dispatch copies each of this rank's sorted rows (gathered from the token
// rows through ids_sorted) straight into the owner's receive buffer; return
// copies each received row's expert output back to the source's slot. Both
// move whole rows with 16-byte stores, local or through peer pointers (CUDA
// IPC mappings of the other ranks' buffers). The caller orders them with the
// GEMMs and puts a cross-rank barrier after each (the receiver may read only
// once every sender's kernel has finished).
#include <string.h>

#include <algorithm>

#include "mc_internal.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxExperts = 256;

struct PeerPtrs {
  uint16_t* p[kMaxRanks];
};

// Segment starts for one expert e: where its rows from `src` land in the
// owner's receive buffer, and where they sit in src's sorted order.
// counts_all may be global or shared memory.
__device__ __forceinline__ void segment_bases(const uint32_t* counts_all, int W, int E, int e,
                                              int src, uint32_t* recv_row, uint32_t* src_row) {
  const int P = E / W, owner = e / P, j0 = owner * P;
  uint32_t base = 0;
  for (int jj = j0; jj < e; ++jj)
    for (int s = 0; s < W; ++s) base += counts_all[s * E + jj];
  for (int s = 0; s < src; ++s) base += counts_all[s * E + e];
  uint32_t off = 0;
  for (int ee = 0; ee < e; ++ee) off += counts_all[src * E + ee];
  *recv_row = base;
  *src_row = off;
}

// Row chunks of this rank's receive buffer for the grouped GEMMs, from the
// count table ca (shared memory, W x E): full bm-row chunks first (local
// expert order), then the partial ones by decreasing height (ties: lower
// expert). Run by a whole CTA (it synchronises); total_s: P words of shared
// scratch.
__device__ void tiles_body(const uint32_t* ca, int rank, int W, int E, int bm, uint4* tiles,
                           uint32_t* n_tiles, uint32_t* rows, int max_tiles, uint32_t* total_s) {
  const int P = E / W;
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    uint32_t t = 0;
    for (int s = 0; s < W; ++s) t += ca[s * E + rank * P + j];
    total_s[j] = t;
  }
  __syncthreads();
  uint32_t full_all = 0, parts = 0, all_rows = 0;
  for (int jj = 0; jj < P; ++jj) {
    full_all += total_s[jj] / bm;
    parts += (total_s[jj] % bm) != 0;
    all_rows += total_s[jj];
  }
  if (threadIdx.x == 0) {
    *n_tiles = full_all + parts;
    if (rows) *rows = all_rows;
  }
  for (int j = threadIdx.x; j < P; j += blockDim.x) {
    const uint32_t tj = total_s[j], pj = tj % bm;
    uint32_t base = 0, full_before = 0, rank_p = 0;
    for (int jj = 0; jj < P; ++jj) {
      const uint32_t t = total_s[jj], p = t % bm;
      if (jj < j) {
        base += t;
        full_before += t / bm;
      }
      if (p && (p > pj || (p == pj && jj < j))) ++rank_p;
    }
    const uint32_t nfull = tj / bm;
    for (uint32_t c = 0; c < nfull; ++c) {
      const uint32_t slot = full_before + c;
      if (slot < (uint32_t)max_tiles)
        tiles[slot] = make_uint4(base + c * bm, base + (c + 1) * bm, (uint32_t)j, 0u);
    }
    if (pj) {
      const uint32_t slot = full_all + rank_p;
      if (slot < (uint32_t)max_tiles)
        tiles[slot] = make_uint4(base + nfull * bm, base + tj, (uint32_t)j, 0u);
    }
  }
}

// The return map of this rank's local slots from the count table ca: the
// rows of local slot j from source s are seg_row[j][s] .. seg_row[j][s+1] of
// the receive buffer and go to rows from seg_home[j][s] of s's home buffer
// (s's own sorted order).
__device__ void segments_body(const uint32_t* ca, int rank, int W, int E, uint32_t* seg_row,
                              uint32_t* seg_home) {
  const int spr = E / W;
  for (int t = threadIdx.x; t < spr * (W + 1); t += blockDim.x) {
    const int j = t / (W + 1), s = t % (W + 1), slot = rank * spr + j;
    uint32_t row = 0;
    for (int jj = rank * spr; jj < slot; ++jj)
      for (int q = 0; q < W; ++q) row += ca[q * E + jj];
    for (int q = 0; q < s; ++q) row += ca[q * E + slot];
    seg_row[j * (W + 1) + s] = row;
    if (s < W) {
      uint32_t h = 0;
      for (int e = 0; e < slot; ++e) h += ca[s * E + e];
      seg_home[j * W + s] = h;
    }
  }
}

// What the expert-parallel step also wants from the dispatch launch (all null
// for mc_ep_dispatch): the receive side's row chunks and the return map,
// built by the last CTA from the count table it has staged anyway, so they
// cost no launch of their own.
struct Plan {
  uint4* tiles;
  uint32_t* n_tiles;
  uint32_t* rows;
  uint32_t* seg_row;
  uint32_t* seg_home;
  int bm, max_tiles;
  // arrival (set when done is not null): once every CTA's rows are written,
  // the last CTA advances the rank's epoch word and stores it into this
  // rank's slot of every rank's flag words -- the arrival half of the
  // barrier after the dispatch (the consumer's GEMM does the waiting)
  uint32_t* flag_p[kMaxRanks];
  uint32_t* epoch;
  uint32_t* done;
  int skip;  // test aid: do not arrive
};

// This rank's expert-sorted rows -> the owners' receive buffers. Every warp
// takes rows across all experts (grid-stride over the sorted order), so a hot
// expert's rows are spread over the whole grid; each CTA first lays out the
// experts' starts (in the sorted order and in the owners' buffers) in shared
// memory, then finds a row's expert by binary search. 16 bytes per lane per
// step.
__global__ void __launch_bounds__(256)
ep_dispatch_kernel(const uint4* __restrict__ x, int m, int h16,
                   const uint32_t* __restrict__ ids_sorted, const uint32_t* __restrict__ counts_all,
                   int rank, int W, int E, PeerPtrs recv, uint32_t cap, uint32_t* status,
                   const Plan plan) {
  __shared__ uint32_t src0[kMaxExperts + 1], dst0[kMaxExperts];
  __shared__ uint32_t ca[kMaxRanks * kMaxExperts];  // the count table, staged once
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) ca[i] = counts_all[i];
  __syncthreads();
  if (plan.tiles && blockIdx.x == gridDim.x - 1) {  // uniform over the CTA
    tiles_body(ca, rank, W, E, plan.bm, plan.tiles, plan.n_tiles, plan.rows, plan.max_tiles,
               dst0);
    segments_body(ca, rank, W, E, plan.seg_row, plan.seg_home);
    __syncthreads();  // dst0 is reused below
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    uint32_t d, s;
    segment_bases(ca, W, E, e, rank, &d, &s);
    src0[e] = s;
    dst0[e] = d;
  }
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int e = 0; e < E; ++e) t += ca[rank * E + e];
    src0[E] = t;
  }
  __syncthreads();
  const uint32_t total = src0[E];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = E / W;
  // The sorted rows are grouped by owner rank; walked in that order by every
  // source, all ranks would write into rank 0 first, then all into rank 1,
  // ..., one destination's inbound link at a time. Source s starts at the
  // rows for rank s + 1 instead (a rotation of the same rows).
  const uint32_t rot = W > 1 ? src0[((rank + 1) % W) * P] : 0u;
  for (uint32_t i = blockIdx.x * 8 + warp; i < total; i += gridDim.x * 8) {
    uint32_t r = i + rot;
    if (r >= total) r -= total;
    int lo = 0, hi = E;  // src0[lo] <= r < src0[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (src0[mid] <= r) lo = mid;
      else hi = mid;
    }
    const uint32_t k = r - src0[lo];
    const uint32_t tok = __ldg(ids_sorted + r);
    if (dst0[lo] + k >= cap || tok >= (uint32_t)m) {  // inconsistent counts: never write past a buffer
      if (lane == 0 && status) atomicOr(status, 4u);
      continue;
    }
    const uint4* row = x + (size_t)tok * h16;
    uint4* out = reinterpret_cast<uint4*>(recv.p[lo / P]) + (size_t)(dst0[lo] + k) * h16;
    mc_copy_row16(out, row, h16, lane);
  }
  __threadfence_system();
  if (plan.done) {  // uniform over the grid
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(plan.done, 1u) == gridDim.x - 1) {
      *plan.done = 0u;
      const uint32_t ep = *plan.epoch + 1u;
      *plan.epoch = ep;
      __threadfence_system();
      if (!plan.skip)
        for (int p = 0; p < W; ++p)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(plan.flag_p[p] + rank), "r"(ep)
                       : "memory");
    }
  }
}

// Expert outputs of this rank's received rows -> each source's slot.
// grid (W * P, Y): block x = (source, local expert).
__global__ void __launch_bounds__(256)
ep_return_kernel(const uint4* __restrict__ ed, uint32_t ed_rows, int h16,
                 const uint32_t* __restrict__ counts_all, int rank, int W, int E, PeerPtrs home,
                 uint32_t cap, uint32_t* status) {
  const int P = E / W;
  const int src = blockIdx.x / P, e = rank * P + blockIdx.x % P;
  __shared__ uint32_t row0, slot0, n;
  if (threadIdx.x == 0) {
    segment_bases(counts_all, W, E, e, src, &row0, &slot0);
    n = counts_all[src * E + e];
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(home.p[src]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t k = blockIdx.y * 8 + warp; k < n; k += gridDim.y * 8) {
    if (slot0 + k >= cap || row0 + k >= ed_rows) {  // never write or read past a buffer
      if (lane == 0 && status) atomicOr(status, 4u);
      continue;
    }
    const uint4* row = ed + (size_t)(row0 + k) * h16;
    uint4* out = dst + (size_t)(slot0 + k) * h16;
    mc_copy_row16(out, row, h16, lane);
  }
  __threadfence_system();
}

// Row chunks of this rank's receive buffer for the grouped GEMMs (see
// tiles_body). One CTA.
__global__ void __launch_bounds__(256)
ep_tiles_kernel(const uint32_t* __restrict__ counts_all, int rank, int W, int E, int bm,
                uint4* __restrict__ tiles, uint32_t* __restrict__ n_tiles, uint32_t* __restrict__ rows,
                int max_tiles) {
  __shared__ uint32_t total_s[kMaxExperts];
  __shared__ uint32_t ca[kMaxRanks * kMaxExperts];  // the count table, staged once
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) ca[i] = counts_all[i];
  __syncthreads();
  tiles_body(ca, rank, W, E, bm, tiles, n_tiles, rows, max_tiles, total_s);
}

int check_ranks(int rank, int W, int E, const char* what) {
  MC_REQUIRE(W >= 1 && W <= kMaxRanks && rank >= 0 && rank < W, "%s: rank %d of %d", what, rank,
             W);
  MC_REQUIRE(E >= 1 && E <= kMaxExperts && E % W == 0, "%s: %d experts over %d ranks", what, E, W);
  return MC_OK;
}

int fill_peers(PeerPtrs* pp, void* const* ptrs, int W, const char* what) {
  MC_REQUIRE(ptrs, "%s: null peer pointer table", what);
  for (int r = 0; r < kMaxRanks; ++r) pp->p[r] = nullptr;
  for (int r = 0; r < W; ++r) {
    MC_REQUIRE(ptrs[r] && mc_aligned(ptrs[r], 16), "%s: peer buffer %d null or not 16-byte aligned",
               what, r);
    pp->p[r] = static_cast<uint16_t*>(ptrs[r]);
  }
  return MC_OK;
}

}  // namespace

extern "C" int mc_ep_alloc(mc_ctx* ctx, size_t bytes, void** out) {
  MC_REQUIRE(ctx && out && bytes > 0, "ep_alloc: bad arguments");
  MC_CUDA(cudaMalloc(out, bytes));
  return MC_OK;
}

extern "C" int mc_ep_free(mc_ctx* ctx, void* ptr) {
  MC_REQUIRE(ctx, "ep_free: null context");
  if (ptr) MC_CUDA(cudaFree(ptr));
  return MC_OK;
}

extern "C" int mc_ipc_handle(mc_ctx* ctx, void* base, void* handle_out) {
  MC_REQUIRE(ctx && base && handle_out, "ipc_handle: bad arguments");
  cudaIpcMemHandle_t h;
  MC_CUDA(cudaIpcGetMemHandle(&h, base));
  memcpy(handle_out, &h, sizeof(h));
  return MC_OK;
}

extern "C" int mc_ipc_open(mc_ctx* ctx, const void* handle, void** out) {
  MC_REQUIRE(ctx && handle && out, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  MC_CUDA(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
  return MC_OK;
}

extern "C" int mc_ipc_close(mc_ctx* ctx, void* ptr) {
  MC_REQUIRE(ctx, "ipc_close: null context");
  if (ptr) MC_CUDA(cudaIpcCloseMemHandle(ptr));
  return MC_OK;
}

extern "C" int mc_ep_dispatch(mc_ctx* ctx, const uint16_t* x, int m, int hidden,
                              const uint32_t* ids_sorted, const uint32_t* counts_all, int rank,
                              int world, int n_experts, void* const* recv_bufs,
                              size_t recv_cap_rows, uint32_t* status) {
  MC_REQUIRE(ctx && x && ids_sorted && counts_all, "ep_dispatch: null pointer");
  int rc;
  if ((rc = check_ranks(rank, world, n_experts, "ep_dispatch"))) return rc;
  MC_REQUIRE(hidden > 0 && hidden % 8 == 0 && mc_aligned(x, 16), "ep_dispatch: rows");
  PeerPtrs pp;
  if ((rc = fill_peers(&pp, recv_bufs, world, "ep_dispatch"))) return rc;
  MC_REQUIRE(m >= 1 && recv_cap_rows >= 1 && recv_cap_rows <= 0xffffffffu,
             "ep_dispatch: m %d / capacity %zu", m, recv_cap_rows);
  const int grid = std::max(1, std::min((4 * m + 7) / 8, ctx->num_sms * 2));
  ep_dispatch_kernel<<<grid, 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(x), m, hidden / 8, ids_sorted, counts_all, rank, world,
      n_experts, pp, (uint32_t)recv_cap_rows, status, Plan{});
  return mc_after_launch("ep_dispatch_kernel");
}

int mc_ep_dispatch_plan(mc_ctx* ctx, const uint16_t* x, int m, int hidden,
                        const uint32_t* ids_sorted, const uint32_t* counts_all, int rank,
                        int world, int n_experts, void* const* recv_bufs, size_t recv_cap_rows,
                        uint32_t* status, int bm, uint32_t* tiles, uint32_t* n_tiles,
                        uint32_t* rows, int max_tiles, uint32_t* seg_row, uint32_t* seg_home,
                        uint32_t* const* flag_ptrs, uint32_t* epoch, uint32_t* done, int skip) {
  MC_REQUIRE(ctx && x && ids_sorted && counts_all && tiles && n_tiles && seg_row && seg_home,
             "ep_dispatch_plan: null pointer");
  MC_REQUIRE(!done || (flag_ptrs && epoch), "ep_dispatch_plan: arrival needs flags and epoch");
  int rc;
  if ((rc = check_ranks(rank, world, n_experts, "ep_dispatch_plan"))) return rc;
  MC_REQUIRE(hidden > 0 && hidden % 8 == 0 && mc_aligned(x, 16), "ep_dispatch_plan: rows");
  MC_REQUIRE(bm >= 1 && bm <= 4096 && max_tiles >= 1 && mc_aligned(tiles, 16),
             "ep_dispatch_plan: bm %d / max_tiles %d", bm, max_tiles);
  PeerPtrs pp;
  if ((rc = fill_peers(&pp, recv_bufs, world, "ep_dispatch_plan"))) return rc;
  MC_REQUIRE(m >= 1 && recv_cap_rows >= 1 && recv_cap_rows <= 0xffffffffu,
             "ep_dispatch_plan: m %d / capacity %zu", m, recv_cap_rows);
  Plan plan{reinterpret_cast<uint4*>(tiles), n_tiles, rows, seg_row, seg_home, bm, max_tiles,
            {}, epoch, done, skip};
  if (done)
    for (int r = 0; r < world; ++r) {
      MC_REQUIRE(flag_ptrs[r], "ep_dispatch_plan: flag words of rank %d", r);
      plan.flag_p[r] = flag_ptrs[r];
    }
  const int grid = std::max(1, std::min((4 * m + 7) / 8, ctx->num_sms * 2));
  ep_dispatch_kernel<<<grid, 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(x), m, hidden / 8, ids_sorted, counts_all, rank, world,
      n_experts, pp, (uint32_t)recv_cap_rows, status, plan);
  return mc_after_launch("ep_dispatch_kernel");
}

extern "C" int mc_ep_return(mc_ctx* ctx, const uint16_t* ed, size_t ed_rows, int hidden,
                            const uint32_t* counts_all, int rank, int world, int n_experts,
                            void* const* home_bufs, size_t home_cap_rows, uint32_t* status) {
  MC_REQUIRE(ctx && ed && counts_all, "ep_return: null pointer");
  int rc;
  if ((rc = check_ranks(rank, world, n_experts, "ep_return"))) return rc;
  MC_REQUIRE(hidden > 0 && hidden % 8 == 0 && mc_aligned(ed, 16), "ep_return: rows");
  PeerPtrs pp;
  if ((rc = fill_peers(&pp, home_bufs, world, "ep_return"))) return rc;
  MC_REQUIRE(ed_rows >= 1 && ed_rows <= 0xffffffffu && home_cap_rows >= 1 &&
                 home_cap_rows <= 0xffffffffu,
             "ep_return: rows %zu / capacity %zu", ed_rows, home_cap_rows);
  ep_return_kernel<<<dim3(n_experts, 8), 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(ed), (uint32_t)ed_rows, hidden / 8, counts_all, rank, world,
      n_experts, pp, (uint32_t)home_cap_rows, status);
  return mc_after_launch("ep_return_kernel");
}

extern "C" int mc_ep_tiles(mc_ctx* ctx, const uint32_t* counts_all, int rank, int world,
                           int n_experts, int bm, uint32_t* tiles, uint32_t* n_tiles,
                           uint32_t* rows, int max_tiles) {
  MC_REQUIRE(ctx && counts_all && tiles && n_tiles, "ep_tiles: null pointer");
  int rc;
  if ((rc = check_ranks(rank, world, n_experts, "ep_tiles"))) return rc;
  MC_REQUIRE(bm >= 1 && bm <= 4096 && max_tiles >= 1 && mc_aligned(tiles, 16),
             "ep_tiles: bm %d / max_tiles %d", bm, max_tiles);
  ep_tiles_kernel<<<1, 256, 0, ctx->stream>>>(counts_all, rank, world, n_experts, bm,
                                              reinterpret_cast<uint4*>(tiles), n_tiles, rows,
                                              max_tiles);
  return mc_after_launch("ep_tiles_kernel");
}
