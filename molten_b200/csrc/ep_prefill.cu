// Expert-parallel prefill MoE FFN behind the C ABI alone: no PyTorch, no
// host synchronisation inside a step. The reference's moe_prefill
// (lfm.rs:847-965) runs on one device; here the expert slots are spread over
// W ranks (one process per GPU) and one call runs a whole step:
//
//   route (top-4) -> relabel model experts to slots (this rank's table) ->
//   sort by slot -> publish the per-slot pair counts into every rank's
//   count table (peer stores) + barrier -> dispatch: rows stored straight
//   into the owners' receive buffers over NVLink (CUDA IPC mappings), the
//   launch's last CTA also building the receive-side row chunks and the
//   return map -> barrier -> grouped gate/up
//   (+SwiGLU) and down GEMMs, the down GEMM's epilogue storing each expert
//   row straight into its source's home buffer -> barrier -> weighted
//   combine at home.
//
// (The return from the epilogue overlaps the NVLink traffic with the GEMM.
// While the epilogue stored one 2-byte value per thread and row it lost to a
// separate grid-stride copy after the GEMM (0.668 against 0.640 ms per step
// on two B200s); with the outputs staged in shared memory and stored as
// 16-byte rows it wins: 0.566 against 0.605 ms.)
//
// Slots. E_slots = W * slots_per_rank; rank r owns slots [r*spr, (r+1)*spr)
// and holds their weights stacked in slot order. With spr = E / W and an
// identity table this is plain expert parallelism; with spare slots the hot
// experts are replicated (mc_ep_place) and every source rank routes each
// expert to one of its replicas through its own table, which spreads the
// hottest experts' rows over several ranks.
//
// Barriers are device-side: each rank's barrier kernel stores an epoch into
// every peer's flag word for it (a release store at system scope after a
// system fence, so the rows the previous kernels stored are visible first)
// and polls its own flag words (acquire loads) with a deadline; a wait that
// runs out sets status bit 8 and the kernel returns. The NCCL communicator
// (non-blocking: every call on it is followed by polling
// ncclCommGetAsyncError with a host deadline, and mc_sync / mc_ep_finalize
// abort it, ncclCommAbort, when the deadline passes) sets the ranks up and
// tears them down; a step itself makes no NCCL call.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy already in the
// process if there is one), so the library loads and its single-GPU entry
// points work on hosts without NCCL.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <vector>

#include "mc_internal.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kChunk = 256;  // token rows per grouped-GEMM chunk
constexpr unsigned long long kBarrierNs = 1000000000ull;  // default barrier limit: 1 s
// Phases of a step timed by mc_ep_set_profile: route + relabel + sort, the
// counts exchange (peer stores + barrier), row chunks + return map +
// dispatch + barrier, the two grouped GEMMs and the return, the barrier
// after the return, combine.
constexpr int kPhases = 7;
constexpr size_t kCountsOff = 256;  // count table after the flag words in the control area

// ------------------------------------------------------------ NCCL at run time
struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi* nccl() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api.h ? &api : nullptr;
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return nullptr;
  auto sym = [&](const char* n) { return dlsym(h, n); };
  api.get_unique_id = (decltype(api.get_unique_id))sym("ncclGetUniqueId");
  api.init_rank_config = (decltype(api.init_rank_config))sym("ncclCommInitRankConfig");
  api.get_async_error = (decltype(api.get_async_error))sym("ncclCommGetAsyncError");
  api.abort = (decltype(api.abort))sym("ncclCommAbort");
  api.finalize = (decltype(api.finalize))sym("ncclCommFinalize");
  api.destroy = (decltype(api.destroy))sym("ncclCommDestroy");
  api.all_gather = (decltype(api.all_gather))sym("ncclAllGather");
  api.all_reduce = (decltype(api.all_reduce))sym("ncclAllReduce");
  api.error_string = (decltype(api.error_string))sym("ncclGetErrorString");
  if (!api.get_unique_id || !api.init_rank_config || !api.get_async_error || !api.abort ||
      !api.destroy || !api.all_gather || !api.all_reduce)
    return nullptr;
  api.h = h;
  return &api;
}

double now_s() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return t.tv_sec + 1e-9 * t.tv_nsec;
}

}  // namespace

// Everything one rank keeps between expert-parallel steps.
struct mc_ep_state {
  int world = 1, rank = 0, timeout_ms = 0;
  ncclComm_t comm = nullptr;
  bool comm_bad = false;
  // capacities and shapes (mc_ep_reserve)
  int reserved = 0, m_max = 0, E = 0, spr = 0, E_slots = 0, H = 0, I = 0;
  size_t recv_cap = 0, home_cap = 0;
  // one IPC buffer per rank: receive rows | home rows | flag words
  uint8_t* own = nullptr;
  size_t recv_off = 0, home_off = 0, flag_off = 0;
  void* peer_base[kMaxRanks] = {};
  void* recv_ptr[kMaxRanks] = {};
  void* home_ptr[kMaxRanks] = {};
  uint32_t* flag_ptr[kMaxRanks] = {};
  uint32_t* counts_ptr[kMaxRanks] = {};  // every rank's count table [W][E_slots]
  // local device scratch
  uint8_t* scratch = nullptr;
  uint32_t *ids, *counts, *offsets, *ids_sorted, *slotpos, *sort_tiles, *sort_ntiles;
  uint32_t *counts_all, *tiles, *n_tiles, *rows, *status, *epoch, *done;
  uint16_t *gw, *act;
  uint32_t *seg_row, *seg_home;  // return map (built by the dispatch launch)
  int sort_max_tiles = 0, max_tiles = 0;
  // phase timing (mc_ep_set_profile): events at the step's phase boundaries
  int profile = 0;
  cudaEvent_t ev[kPhases + 1] = {};
};

namespace {

// Waits until the communicator's last operation has left ncclInProgress (or
// reports its error), bounded by the context's timeout; aborts on expiry.
int nccl_settle(mc_ctx* ctx, ncclResult_t r, const char* what) {
  const NcclApi* api = nccl();
  mc_ep_state* ep = ctx->ep;
  const double deadline = now_s() + (ep->timeout_ms > 0 ? ep->timeout_ms : 60000) * 1e-3;
  while (r == ncclInProgress) {
    if (now_s() > deadline) {
      api->abort(ep->comm);
      ep->comm = nullptr;
      ep->comm_bad = true;
      return mc_fail(MC_ETIMEOUT, "%s: NCCL did not complete within %d ms; communicator aborted",
                     what, ep->timeout_ms);
    }
    ncclResult_t a = ncclSuccess;
    api->get_async_error(ep->comm, &a);
    r = a;
  }
  if (r != ncclSuccess) {
    api->abort(ep->comm);
    ep->comm = nullptr;
    ep->comm_bad = true;
    return mc_fail(MC_ENCCL, "%s: %s", what, api->error_string ? api->error_string(r) : "NCCL error");
  }
  return MC_OK;
}

struct FlagPtrs {
  uint32_t* p[kMaxRanks];
};


__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-rank barrier: one thread stores this barrier's epoch into slot
// `rank` of every rank's flag words, then waits (bounded) until every slot of
// its own flag words has reached the epoch. test_skip: this rank does not
// arrive (a failure-detection test with one rank makes its own wait run out).
__device__ void ep_barrier_thread(const FlagPtrs& flags, uint32_t* epoch_word, int rank, int W,
                                  unsigned long long timeout_ns, uint32_t* status,
                                  int test_skip) {
  const uint32_t epoch = *epoch_word + 1u;
  *epoch_word = epoch;
  __threadfence_system();
  if (!test_skip)
    for (int p = 0; p < W; ++p) st_release_sys(flags.p[p] + rank, epoch);
  const uint32_t* mine = flags.p[rank];
  const unsigned long long deadline = mc_globaltimer() + timeout_ns;
  for (int q = 0; q < W; ++q) {
    while ((int)(ld_acquire_sys(mine + q) - epoch) < 0) {
      if (mc_globaltimer() > deadline) {
        atomicOr(status, 8u);
        return;
      }
      __nanosleep(200);
    }
  }
}

__global__ void ep_barrier_kernel(FlagPtrs flags, uint32_t* epoch_word, int rank, int W,
                                  unsigned long long timeout_ns, uint32_t* status, int test_skip) {
  if (threadIdx.x == 0) ep_barrier_thread(flags, epoch_word, rank, W, timeout_ns, status, test_skip);
}

// This rank's pair counts into row `rank` of every rank's count table, then
// the barrier: afterwards every rank holds all ranks' counts.
__global__ void __launch_bounds__(256)
ep_publish_counts_kernel(const uint32_t* __restrict__ counts, FlagPtrs tables, int E_slots,
                         FlagPtrs flags, uint32_t* epoch_word, int rank, int W,
                         unsigned long long timeout_ns, uint32_t* status, int test_skip) {
  for (int e = threadIdx.x; e < E_slots; e += blockDim.x) {
    const uint32_t v = counts[e];
    for (int p = 0; p < W; ++p) tables.p[p][(size_t)rank * E_slots + e] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) ep_barrier_thread(flags, epoch_word, rank, W, timeout_ns, status, test_skip);
}


int ep_barrier(mc_ctx* ctx) {
  mc_ep_state* ep = ctx->ep;
  FlagPtrs f;
  for (int r = 0; r < kMaxRanks; ++r) f.p[r] = r < ep->world ? ep->flag_ptr[r] : nullptr;
  const unsigned long long lim = mc_wait_limit(ctx, kBarrierNs);
  ep_barrier_kernel<<<1, 32, 0, ctx->stream>>>(f, ep->epoch, ep->rank, ep->world, lim, ep->status,
                                                (ctx->test_flags & MC_TEST_SKIP_BARRIER_ARRIVE) ? 1 : 0);
  return mc_after_launch("ep_barrier_kernel");
}

void free_state(mc_ep_state* ep, bool close_peers) {
  for (int k = 0; k <= kPhases; ++k)
    if (ep->ev[k]) {
      cudaEventDestroy(ep->ev[k]);
      ep->ev[k] = nullptr;
    }
  if (close_peers)
    for (int r = 0; r < ep->world; ++r)
      if (r != ep->rank && ep->peer_base[r]) cudaIpcCloseMemHandle(ep->peer_base[r]);
  if (ep->own) cudaFree(ep->own);
  if (ep->scratch) cudaFree(ep->scratch);
  ep->own = nullptr;
  ep->scratch = nullptr;
  ep->reserved = 0;
}

}  // namespace

extern "C" int mc_ep_unique_id(void* out) {
  MC_REQUIRE(out, "ep_unique_id: null output");
  const NcclApi* api = nccl();
  if (!api) return mc_fail(MC_ENCCL, "ep_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return mc_fail(MC_ENCCL, "ncclGetUniqueId failed (%d)", (int)r);
  memcpy(out, &id, sizeof(id));
  return MC_OK;
}

extern "C" int mc_ep_init(mc_ctx* ctx, int nranks, int rank, const void* nccl_unique_id,
                          int timeout_ms) {
  MC_REQUIRE(ctx, "ep_init: null context");
  MC_REQUIRE(!ctx->ep, "ep_init: expert parallelism already initialised on this context");
  MC_REQUIRE(nranks >= 1 && nranks <= kMaxRanks && rank >= 0 && rank < nranks,
             "ep_init: rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
  MC_REQUIRE(nccl_unique_id, "ep_init: null NCCL unique id");
  MC_REQUIRE(timeout_ms > 0, "ep_init: timeout_ms %d", timeout_ms);
  const NcclApi* api = nccl();
  if (!api) return mc_fail(MC_ENCCL, "ep_init: libnccl.so.2 could not be loaded");
  MC_CUDA(cudaSetDevice(ctx->device));
  mc_ep_state* ep = new mc_ep_state();
  ep->world = nranks;
  ep->rank = rank;
  ep->timeout_ms = timeout_ms;
  ctx->ep = ep;
  ncclUniqueId id;
  memcpy(&id, nccl_unique_id, sizeof(id));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // calls return at once; progress is polled with a deadline
  ncclResult_t r = api->init_rank_config(&ep->comm, nranks, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    ctx->ep = nullptr;
    delete ep;
    return mc_fail(MC_ENCCL, "ncclCommInitRankConfig: %s",
                   api->error_string ? api->error_string(r) : "error");
  }
  const int rc = nccl_settle(ctx, r == ncclSuccess ? ncclInProgress : r, "ep_init");
  if (rc) {
    ctx->ep = nullptr;
    delete ep;
    return rc;
  }
  return MC_OK;
}

extern "C" int mc_ep_reserve(mc_ctx* ctx, int m_max, int n_experts, int slots_per_rank,
                             int hidden, int moe_inter) {
  MC_REQUIRE(ctx && ctx->ep, "ep_reserve: call mc_ep_init first");
  mc_ep_state* ep = ctx->ep;
  MC_REQUIRE(!ep->comm_bad && ep->comm, "ep_reserve: the communicator was aborted");
  MC_REQUIRE(!ep->reserved, "ep_reserve: buffers already reserved");
  MC_REQUIRE(m_max >= 1 && m_max <= (1 << 20), "ep_reserve: m_max %d", m_max);
  MC_REQUIRE(n_experts >= 4 && n_experts <= 256, "ep_reserve: n_experts %d", n_experts);
  MC_REQUIRE(slots_per_rank >= 1 && (long)slots_per_rank * ep->world >= n_experts &&
                 slots_per_rank * ep->world <= 256,
             "ep_reserve: %d slots per rank x %d ranks cannot hold %d experts", slots_per_rank,
             ep->world, n_experts);
  MC_REQUIRE(hidden % 128 == 0 && moe_inter % 128 == 0, "ep_reserve: hidden %d / width %d",
             hidden, moe_inter);
  const NcclApi* api = nccl();
  const int W = ep->world;
  ep->m_max = m_max;
  ep->E = n_experts;
  ep->spr = slots_per_rank;
  ep->E_slots = W * slots_per_rank;
  ep->H = hidden;
  ep->I = moe_inter;
  ep->recv_cap = (size_t)W * 4 * m_max;
  ep->home_cap = 4 * (size_t)m_max;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  ep->recv_off = 0;
  ep->home_off = al(ep->recv_cap * hidden * 2);
  ep->flag_off = al(ep->home_off + ep->home_cap * hidden * 2);
  const size_t ctl_bytes = kCountsOff + (size_t)W * (W * slots_per_rank) * 4;
  const size_t own_bytes = ep->flag_off + al(ctl_bytes);
  MC_CUDA(cudaSetDevice(ctx->device));
  void* p = nullptr;
  MC_CUDA(cudaMalloc(&p, own_bytes));
  ep->own = static_cast<uint8_t*>(p);
  MC_CUDA(cudaMemsetAsync(ep->own + ep->flag_off, 0, al(ctl_bytes), ctx->stream));
  // local scratch
  const size_t S = 4 * (size_t)m_max;
  ep->sort_max_tiles = (int)((S + kChunk - 1) / kChunk + ep->E_slots);
  ep->max_tiles = (int)(ep->recv_cap / kChunk + slots_per_rank + 1);
  size_t o = 0;
  std::vector<std::pair<void**, size_t>> parts;
  auto carve = [&](void** dst, size_t bytes) { parts.push_back({dst, o}); o = al(o + bytes); };
  carve((void**)&ep->ids, S * 4);
  carve((void**)&ep->gw, S * 2);
  carve((void**)&ep->counts, (size_t)ep->E_slots * 4);
  carve((void**)&ep->offsets, (size_t)ep->E_slots * 4);
  carve((void**)&ep->ids_sorted, S * 4);
  carve((void**)&ep->slotpos, S * 4);
  carve((void**)&ep->sort_tiles, (size_t)ep->sort_max_tiles * 16);
  carve((void**)&ep->sort_ntiles, 16);
  carve((void**)&ep->seg_row, (size_t)slots_per_rank * (W + 1) * 4);
  carve((void**)&ep->seg_home, (size_t)slots_per_rank * W * 4);
  carve((void**)&ep->tiles, (size_t)ep->max_tiles * 16);
  carve((void**)&ep->n_tiles, 16);
  carve((void**)&ep->rows, 16);
  carve((void**)&ep->status, 16);
  carve((void**)&ep->epoch, 16);
  carve((void**)&ep->done, 16);
  carve((void**)&ep->act, ep->recv_cap * moe_inter * 2);
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, o);
  if (e != cudaSuccess) {
    free_state(ep, false);
    (void)cudaGetLastError();
    return mc_fail(MC_ECUDA, "ep_reserve: %zu bytes of scratch: %s", o, cudaGetErrorString(e));
  }
  ep->scratch = static_cast<uint8_t*>(q);
  for (auto& pr : parts) *pr.first = ep->scratch + pr.second;
  MC_CUDA(cudaMemsetAsync(ep->scratch, 0, o, ctx->stream));
  // exchange the IPC handles of every rank's buffer (NCCL all-gather of 64 B each)
  cudaIpcMemHandle_t h;
  MC_CUDA(cudaIpcGetMemHandle(&h, ep->own));
  std::vector<uint8_t> all((size_t)W * sizeof(h));
  uint8_t* dev_h = reinterpret_cast<uint8_t*>(ep->act);  // scratch, unused until the first step
  MC_CUDA(cudaMemcpyAsync(dev_h + (size_t)ep->rank * sizeof(h), &h, sizeof(h),
                          cudaMemcpyHostToDevice, ctx->stream));
  int rc = nccl_settle(ctx,
                       api->all_gather(dev_h + (size_t)ep->rank * sizeof(h), dev_h, sizeof(h),
                                       ncclUint8, ep->comm, ctx->stream),
                       "ep_reserve all-gather");
  if (rc) return rc;
  MC_CUDA(cudaMemcpyAsync(all.data(), dev_h, all.size(), cudaMemcpyDeviceToHost, ctx->stream));
  rc = mc_sync(ctx);
  if (rc) return rc;
  for (int r = 0; r < W; ++r) {
    if (r == ep->rank) {
      ep->peer_base[r] = ep->own;
    } else {
      cudaIpcMemHandle_t hr;
      memcpy(&hr, all.data() + (size_t)r * sizeof(h), sizeof(h));
      void* b = nullptr;
      MC_CUDA(cudaIpcOpenMemHandle(&b, hr, cudaIpcMemLazyEnablePeerAccess));
      ep->peer_base[r] = b;
    }
    uint8_t* b = static_cast<uint8_t*>(ep->peer_base[r]);
    ep->recv_ptr[r] = b + ep->recv_off;
    ep->home_ptr[r] = b + ep->home_off;
    ep->flag_ptr[r] = reinterpret_cast<uint32_t*>(b + ep->flag_off);
    ep->counts_ptr[r] = reinterpret_cast<uint32_t*>(b + ep->flag_off + kCountsOff);
  }
  ep->counts_all = ep->counts_ptr[ep->rank];
  MC_CUDA(cudaMemsetAsync(ep->act, 0, (size_t)W * sizeof(h), ctx->stream));
  ep->reserved = 1;
  // every rank's flags are zero and mapped before the first barrier
  rc = ep_barrier(ctx);
  if (rc) return rc;
  return mc_sync(ctx);
}

extern "C" int mc_ep_moe_prefill(mc_ctx* ctx, const uint16_t* x, const float* logits, int m,
                                 const mc_qweights* gate, const mc_qweights* up,
                                 const mc_qweights* down, const uint32_t* slot_table,
                                 int route_mode, const float* expert_bias, uint16_t* out) {
  MC_REQUIRE(ctx && ctx->ep && ctx->ep->reserved, "ep_moe_prefill: call mc_ep_reserve first");
  mc_ep_state* ep = ctx->ep;
  MC_REQUIRE(!ep->comm_bad && ep->comm, "ep_moe_prefill: the communicator was aborted");
  MC_REQUIRE(x && logits && gate && up && down && slot_table && out, "ep_moe_prefill: null pointer");
  MC_REQUIRE(m >= 1 && m <= ep->m_max, "ep_moe_prefill: m %d outside [1, %d]", m, ep->m_max);
  MC_REQUIRE(gate->in_features == ep->H && gate->out_features == ep->spr * ep->I &&
                 up->out_features == gate->out_features && up->in_features == ep->H &&
                 down->in_features == ep->I && down->out_features == ep->spr * ep->H,
             "ep_moe_prefill: local weights must be this rank's %d slots stacked ([%d][%d], "
             "[%d][%d])",
             ep->spr, ep->spr * ep->I, ep->H, ep->spr * ep->H, ep->I);
  const int S = 4 * m, W = ep->world;
  int rc;
  auto mark = [&](int k) -> int {
    if (ep->profile) MC_CUDA(cudaEventRecord(ep->ev[k], ctx->stream));
    return MC_OK;
  };
  if ((rc = mark(0))) return rc;
  if ((rc = mc_moe_route_batch(ctx, logits, m, ep->E, route_mode, expert_bias, 1e-6f, ep->ids,
                               ep->gw)))
    return rc;
  if ((rc = mc_map_ids(ctx, ep->ids, (size_t)S, slot_table, ep->E, ep->status))) return rc;
  if ((rc = mc_moe_sort_map(ctx, ep->ids, m, ep->E_slots, kChunk, ep->counts, ep->offsets,
                            ep->ids_sorted, ep->slotpos, ep->sort_tiles, ep->sort_ntiles,
                            ep->sort_max_tiles)))
    return rc;
  if ((rc = mark(1))) return rc;
  {
    FlagPtrs tables, flags;
    for (int r = 0; r < kMaxRanks; ++r) {
      tables.p[r] = r < W ? ep->counts_ptr[r] : nullptr;
      flags.p[r] = r < W ? ep->flag_ptr[r] : nullptr;
    }
    ep_publish_counts_kernel<<<1, 256, 0, ctx->stream>>>(
        ep->counts, tables, ep->E_slots, flags, ep->epoch, ep->rank, W,
        mc_wait_limit(ctx, kBarrierNs), ep->status,
        (ctx->test_flags & MC_TEST_SKIP_BARRIER_ARRIVE) ? 1 : 0);
    if ((rc = mc_after_launch("ep_publish_counts_kernel"))) return rc;
  }
  if ((rc = mark(2))) return rc;
  // the dispatch; its last CTA also builds the receive side's row chunks and
  // the return map (two single-CTA launches of their own cost ~20 us a step
  // on the critical path)
  if ((rc = mc_ep_dispatch_plan(ctx, x, m, ep->H, ep->ids_sorted, ep->counts_all, ep->rank, W,
                                ep->E_slots, ep->recv_ptr, ep->recv_cap, ep->status, kChunk,
                                ep->tiles, ep->n_tiles, ep->rows,
                                ep->max_tiles, ep->seg_row, ep->seg_home, ep->flag_ptr,
                                ep->epoch, ep->done,
                                (ctx->test_flags & MC_TEST_SKIP_BARRIER_ARRIVE) ? 1 : 0)))
    return rc;
  if ((rc = mark(3))) return rc;
  // the barrier after the dispatch: the dispatch launch arrives (its last
  // CTA stores the epoch into every rank's flag slot) and the gate/up GEMM
  // waits before its first token load, its set-up and first weight stages
  // overlapping the wait (a barrier launch of its own sat between them)
  if ((rc = mark(4))) return rc;
  uint16_t* recv = static_cast<uint16_t*>(ep->recv_ptr[ep->rank]);
  const int rows = (int)ep->recv_cap;
  if ((rc = mc_gemm_q4_grouped_gu_after(ctx, recv, rows, gate, up, ep->spr, ep->act, ep->tiles,
                                        ep->n_tiles, ep->max_tiles, ep->status,
                                        ep->flag_ptr[ep->rank], ep->epoch, W)))
    return rc;
  // the down GEMM stores each expert row straight into its source's home row
  if ((rc = mc_gemm_q4_grouped_return(ctx, ep->act, rows, down, ep->spr, ep->seg_row, ep->seg_home,
                                       ep->home_ptr, W, ep->home_cap, ep->tiles, ep->n_tiles,
                                       ep->max_tiles, ep->status)))
    return rc;
  if ((rc = mark(5))) return rc;
  if ((rc = ep_barrier(ctx))) return rc;
  if ((rc = mark(6))) return rc;
  if ((rc = mc_moe_combine_rows(ctx, static_cast<uint16_t*>(ep->home_ptr[ep->rank]), ep->slotpos,
                                ep->gw, out, m, 4, ep->H)))
    return rc;
  return mark(7);
}

extern "C" int mc_ep_set_profile(mc_ctx* ctx, int on) {
  MC_REQUIRE(ctx && ctx->ep, "ep_set_profile: call mc_ep_init first");
  mc_ep_state* ep = ctx->ep;
  if (on && !ep->ev[0])
    for (int k = 0; k <= kPhases; ++k) MC_CUDA(cudaEventCreate(&ep->ev[k]));
  ep->profile = on ? 1 : 0;
  return MC_OK;
}

extern "C" int mc_ep_phase_ms(mc_ctx* ctx, float* out) {
  MC_REQUIRE(ctx && ctx->ep && out, "ep_phase_ms: bad arguments");
  mc_ep_state* ep = ctx->ep;
  MC_REQUIRE(ep->ev[0], "ep_phase_ms: profiling was never switched on");
  int rc = mc_sync(ctx);
  if (rc) return rc;
  for (int k = 0; k < kPhases; ++k) MC_CUDA(cudaEventElapsedTime(out + k, ep->ev[k], ep->ev[k + 1]));
  return MC_OK;
}

extern "C" int mc_ep_status(mc_ctx* ctx, uint32_t* out) {
  MC_REQUIRE(ctx && ctx->ep && ctx->ep->reserved && out, "ep_status: bad arguments");
  int rc = mc_sync(ctx);
  if (rc) return rc;
  MC_CUDA(cudaMemcpy(out, ctx->ep->status, 4, cudaMemcpyDeviceToHost));
  MC_CUDA(cudaMemset(ctx->ep->status, 0, 4));
  return MC_OK;
}

extern "C" int mc_ep_counts(mc_ctx* ctx, uint32_t* out, size_t n) {
  MC_REQUIRE(ctx && ctx->ep && ctx->ep->reserved && out, "ep_counts: bad arguments");
  mc_ep_state* ep = ctx->ep;
  MC_REQUIRE(n >= (size_t)ep->world * ep->E_slots, "ep_counts: %zu < %d words", n,
             ep->world * ep->E_slots);
  int rc = mc_sync(ctx);
  if (rc) return rc;
  MC_CUDA(cudaMemcpy(out, ep->counts_all, (size_t)ep->world * ep->E_slots * 4,
                     cudaMemcpyDeviceToHost));
  return MC_OK;
}

// Waits for the context's stream; with a communicator, polls its
// asynchronous error meanwhile and aborts it when the timeout passes.
int mc_ep_wait(mc_ctx* ctx) {
  mc_ep_state* ep = ctx->ep;
  const NcclApi* api = nccl();
  const double deadline = now_s() + ep->timeout_ms * 1e-3;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      (void)cudaGetLastError();
      return mc_fail(MC_ECUDA, "mc_sync: %s", cudaGetErrorString(q));
    }
    if (ep->comm && api) {
      ncclResult_t a = ncclSuccess;
      api->get_async_error(ep->comm, &a);
      if (a != ncclSuccess && a != ncclInProgress) {
        api->abort(ep->comm);
        ep->comm = nullptr;
        ep->comm_bad = true;
        return mc_fail(MC_ENCCL, "mc_sync: NCCL reported %s; communicator aborted",
                       api->error_string ? api->error_string(a) : "an error");
      }
    }
    if (now_s() > deadline) {
      if (ep->comm && api) api->abort(ep->comm);
      ep->comm = nullptr;
      ep->comm_bad = true;
      return mc_fail(MC_ETIMEOUT, "mc_sync: the stream did not drain within %d ms; "
                     "communicator aborted", ep->timeout_ms);
    }
    struct timespec ts = {0, 50000};
    nanosleep(&ts, nullptr);
  }
  MC_CUDA(cudaGetLastError());
  return MC_OK;
}

extern "C" int mc_ep_finalize(mc_ctx* ctx) {
  MC_REQUIRE(ctx, "ep_finalize: null context");
  mc_ep_state* ep = ctx->ep;
  if (!ep) return MC_OK;
  const NcclApi* api = nccl();
  int rc = MC_OK;
  if (ep->reserved && ep->comm && !ep->comm_bad) {
    // every rank stops using the others' buffers before any is freed
    rc = mc_sync(ctx);
    for (int r = 0; r < ep->world; ++r)
      if (r != ep->rank && ep->peer_base[r]) {
        cudaIpcCloseMemHandle(ep->peer_base[r]);
        ep->peer_base[r] = nullptr;
      }
    if (!rc) {
      rc = nccl_settle(ctx,
                       api->all_reduce(ep->status + 1, ep->status + 1, 1, ncclUint32, ncclSum,
                                       ep->comm, ctx->stream),
                       "ep_finalize barrier");
      if (!rc) rc = mc_sync(ctx);
    }
  }
  free_state(ep, false);
  if (ep->comm && api) {
    if (!ep->comm_bad && api->finalize) {
      ncclResult_t r = api->finalize(ep->comm);
      if (r == ncclInProgress || r == ncclSuccess) {
        const int rc2 = nccl_settle(ctx, ncclInProgress, "ep_finalize");
        if (!rc) rc = rc2;
      }
    }
    if (ep->comm) api->destroy(ep->comm);
  }
  ctx->ep = nullptr;
  delete ep;
  return rc;
}

// ------------------------------------------------------------ placement

namespace {

// One candidate placement: slot_expert[T], tables[W][E], and the rank loads.
struct Placement {
  std::vector<int32_t> slot_expert;
  std::vector<uint32_t> tables;
  std::vector<double> rank_load;
  double max_load() const { return *std::max_element(rank_load.begin(), rank_load.end()); }
};

// Builds a placement with `spare` of the W * spr - E spare slots used for
// replicas (the rest stay empty): replica counts by largest load per
// replica, replicas placed largest first on the least-loaded rank holding
// none of that expert, (source, expert) pairs of replicated experts sent,
// heaviest first, to the replica on the least-loaded rank (ties: the
// source's own rank, then the lower rank). Then a local search lowers the
// heaviest rank's load while it can: moving one (source, expert) pair to
// another replica of the expert, or moving an expert with one replica to
// another rank's free slot or swapping it with one there.
Placement build_placement(const unsigned long long* load, int W, int E, int spr, int spare) {
  const int T = W * spr;
  std::vector<double> L(E, 0.0);
  for (int s = 0; s < W; ++s)
    for (int e = 0; e < E; ++e) L[e] += (double)load[(size_t)s * E + e];
  std::vector<int> rep(E, 1);
  for (int x = 0; x < spare; ++x) {
    int best = -1;
    for (int e = 0; e < E; ++e)
      if (rep[e] < W && (best < 0 || L[e] / rep[e] > L[best] / rep[best])) best = e;
    if (best < 0) break;
    ++rep[best];
  }
  struct Unit { int e, j; double w; };
  std::vector<Unit> units;
  for (int e = 0; e < E; ++e)
    for (int j = 0; j < rep[e]; ++j) units.push_back({e, j, L[e] / rep[e]});
  std::stable_sort(units.begin(), units.end(), [](const Unit& a, const Unit& b) {
    if (a.w != b.w) return a.w > b.w;
    return a.e != b.e ? a.e < b.e : a.j < b.j;
  });
  Placement pl;
  pl.slot_expert.assign(T, -1);
  pl.tables.assign((size_t)W * E, 0u);
  std::vector<double> est(W, 0.0);
  std::vector<int> used(W, 0);
  std::vector<std::vector<int>> slot_of(E);
  auto holds = [&](int e, int r) {
    for (int sl : slot_of[e])
      if (sl / spr == r) return true;
    return false;
  };
  for (const Unit& u : units) {
    int pick = -1;
    for (int pass = 0; pass < 2 && pick < 0; ++pass)
      for (int r = 0; r < W; ++r) {
        if (used[r] >= spr || (pass == 0 && holds(u.e, r))) continue;
        if (pick < 0 || est[r] < est[pick]) pick = r;
      }
    if (pick < 0) break;
    const int slot = pick * spr + used[pick]++;
    est[pick] += u.w;
    slot_of[u.e].push_back(slot);
    pl.slot_expert[slot] = u.e;
  }
  pl.rank_load.assign(W, 0.0);
  struct Pair { int s, e; double w; };
  std::vector<Pair> pairs;
  for (int e = 0; e < E; ++e)
    for (int s = 0; s < W; ++s) {
      const double w = (double)load[(size_t)s * E + e];
      if (slot_of[e].size() == 1) {
        pl.tables[(size_t)s * E + e] = (uint32_t)slot_of[e][0];
        pl.rank_load[slot_of[e][0] / spr] += w;
      } else {
        pairs.push_back({s, e, w});
      }
    }
  std::stable_sort(pairs.begin(), pairs.end(), [](const Pair& a, const Pair& b) {
    if (a.w != b.w) return a.w > b.w;
    return a.e != b.e ? a.e < b.e : a.s < b.s;
  });
  for (const Pair& p : pairs) {
    int j = 0;
    for (int c = 1; c < (int)slot_of[p.e].size(); ++c) {
      const int rc = slot_of[p.e][c] / spr, rj = slot_of[p.e][j] / spr;
      const double lc = pl.rank_load[rc], lj = pl.rank_load[rj];
      if (lc < lj || (lc == lj && (rc == p.s || (rj != p.s && rc < rj)))) j = c;
    }
    pl.tables[(size_t)p.s * E + p.e] = (uint32_t)slot_of[p.e][j];
    pl.rank_load[slot_of[p.e][j] / spr] += p.w;
  }
  // ---- local search on the heaviest rank
  auto wl = [&](int s, int e) { return (double)load[(size_t)s * E + e]; };
  for (int iter = 0; iter < 4096; ++iter) {
    const int rm = (int)(std::max_element(pl.rank_load.begin(), pl.rank_load.end()) -
                         pl.rank_load.begin());
    const double cur = pl.rank_load[rm];
    double best = cur;
    int kind = -1, a0 = 0, a1 = 0, a2 = 0;
    // (a) one pair of a replicated expert to its replica on another rank
    for (int s = 0; s < W; ++s)
      for (int e = 0; e < E; ++e) {
        if (slot_of[e].size() < 2 || (int)pl.tables[(size_t)s * E + e] / spr != rm) continue;
        const double w = wl(s, e);
        for (int sl : slot_of[e]) {
          const int r2 = sl / spr;
          if (r2 == rm) continue;
          const double m = std::max(cur - w, pl.rank_load[r2] + w);
          if (m < best) { best = m; kind = 0; a0 = s; a1 = e; a2 = sl; }
        }
      }
    // (b) an expert with one replica on rm to a free slot or swapped with
    // a one-replica expert on another rank
    for (int sa = rm * spr; sa < (rm + 1) * spr; ++sa) {
      const int ea = pl.slot_expert[sa];
      if (ea < 0 || slot_of[ea].size() != 1) continue;
      const double la = L[ea];
      for (int sb = 0; sb < T; ++sb) {
        const int r2 = sb / spr;
        if (r2 == rm) continue;
        const int eb = pl.slot_expert[sb];
        if (eb >= 0 && slot_of[eb].size() != 1) continue;
        const double lb = eb >= 0 ? L[eb] : 0.0;
        const double m = std::max(cur - la + lb, pl.rank_load[r2] + la - lb);
        if (m < best) { best = m; kind = 1; a0 = sa; a1 = sb; }
      }
    }
    if (kind < 0 || best >= cur - 1e-9) break;
    if (kind == 0) {
      const double w = wl(a0, a1);
      pl.rank_load[rm] -= w;
      pl.rank_load[a2 / spr] += w;
      pl.tables[(size_t)a0 * E + a1] = (uint32_t)a2;
    } else {
      const int ea = pl.slot_expert[a0], eb = pl.slot_expert[a1];
      const double lb = eb >= 0 ? L[eb] : 0.0;
      pl.rank_load[rm] += lb - L[ea];
      pl.rank_load[a1 / spr] += L[ea] - lb;
      pl.slot_expert[a0] = eb;
      pl.slot_expert[a1] = ea;
      slot_of[ea][0] = a1;
      for (int s = 0; s < W; ++s) pl.tables[(size_t)s * E + ea] = (uint32_t)a1;
      if (eb >= 0) {
        slot_of[eb][0] = a0;
        for (int s = 0; s < W; ++s) pl.tables[(size_t)s * E + eb] = (uint32_t)a0;
      }
    }
  }
  return pl;
}

}  // namespace

// Skew-aware placement of E experts on W ranks of spr slots each (host
// only). load[s][e]: pairs of source rank s routed to expert e (one routing
// pass). Candidates use 0, 1, ... of the spare slots for replicas of the
// hottest experts (build_placement); the one whose heaviest rank carries the
// least wins (ties: fewer replicas), so spare slots never make it worse.
// tables[s][e] = the slot source s sends expert e's rows to;
// slot_expert[slot] = the expert a slot holds (-1: empty). Deterministic:
// every rank computes the same placement.
extern "C" int mc_ep_place(const unsigned long long* load, int world, int n_experts,
                           int slots_per_rank, uint32_t* tables, int32_t* slot_expert) {
  MC_REQUIRE(load && tables && slot_expert, "ep_place: null pointer");
  MC_REQUIRE(world >= 1 && world <= kMaxRanks, "ep_place: world %d", world);
  MC_REQUIRE(n_experts >= 1 && slots_per_rank >= 1 && (long)world * slots_per_rank >= n_experts &&
                 world * slots_per_rank <= 256,
             "ep_place: %d slots per rank x %d ranks for %d experts", slots_per_rank, world,
             n_experts);
  const int spare = world * slots_per_rank - n_experts;
  Placement best;
  for (int x = 0; x <= spare; ++x) {
    Placement p = build_placement(load, world, n_experts, slots_per_rank, x);
    if (best.rank_load.empty() || p.max_load() < best.max_load() - 1e-9) best = std::move(p);
  }
  for (int e = 0; e < n_experts; ++e) {
    bool placed = false;
    for (int32_t v : best.slot_expert) placed |= v == e;
    MC_REQUIRE(placed, "ep_place: expert %d got no slot", e);
  }
  std::copy(best.slot_expert.begin(), best.slot_expert.end(), slot_expert);
  std::copy(best.tables.begin(), best.tables.end(), tables);
  return MC_OK;
}

// Context teardown without the other ranks (mc_destroy): unmaps the peers'
// buffers, frees this rank's and aborts the communicator.
void mc_ep_release(mc_ctx* ctx) {
  mc_ep_state* ep = ctx->ep;
  if (!ep) return;
  free_state(ep, true);
  const NcclApi* api = nccl();
  if (ep->comm && api) api->abort(ep->comm);
  ctx->ep = nullptr;
  delete ep;
}
