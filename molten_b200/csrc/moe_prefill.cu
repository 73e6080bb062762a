// Prefill MoE dispatch around the grouped GEMM: the deterministic counting
// sort + row-tile list (lfm.metal:1604-1770), the row gather
// (elementwise.metal:41-52), SwiGLU (elementwise.metal:7-15) and the weighted
// combine (lfm.metal:915-940).
//
// Sort: two launches, one CTA per expert each. Launch 1 counts the expert's
// pairs (no atomics: every CTA scans the whole id list, 64 x 64 KB from L2 at
// the 4096-token chunk, so counts are deterministic). Launch 2 derives the
// expert's offset and tile slots from the 64 counts, scans its pairs in
// token-major, rank-major order (each thread a contiguous token range, block
// exclusive scan), and writes ids_sorted / slotpos and its row tiles (full
// tiles first in expert order, then partial tiles by decreasing height).
#include "mc_internal.cuh"

namespace {

__global__ void __launch_bounds__(256)
sort_count_kernel(const uint32_t* __restrict__ ids, int S, uint32_t* __restrict__ counts) {
  __shared__ uint32_t red[8];
  const uint32_t e = blockIdx.x;
  uint32_t c = 0;
  for (int i = threadIdx.x; i < S; i += 256) c += (__ldg(ids + i) == e);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) c += __shfl_xor_sync(0xffffffffu, c, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < 8; ++w) t += red[w];
    counts[e] = t;
  }
}

__global__ void __launch_bounds__(256)
sort_scatter_kernel(const uint32_t* __restrict__ ids, int m, int E, int bm,
                    const uint32_t* __restrict__ counts, uint32_t* __restrict__ offsets,
                    uint32_t* __restrict__ ids_sorted, uint32_t* __restrict__ slotpos,
                    uint4* __restrict__ tiles, uint32_t* __restrict__ n_tiles, int max_tiles) {
  __shared__ uint32_t warp_tot[8];
  __shared__ uint32_t base_s[3];
  __shared__ uint32_t cnt_s[1024];  // the E counts, staged once
  const uint32_t e = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int j = t; j < E; j += 256) cnt_s[j] = counts[j];
  __syncthreads();
  if (t == 0) {
    // Tile list order: every full bm-row tile first (expert order), then the
    // partial tiles by decreasing height (ties: lower expert first), so a
    // consumer that deals tiles out in list order balances its workers.
    const uint32_t ce = cnt_s[e], pe = ce % (uint32_t)bm;
    uint32_t off = 0, full_before = 0, full_all = 0, part_rank = 0, parts = 0;
    for (int j = 0; j < E; ++j) {
      const uint32_t c = cnt_s[j], pj = c % (uint32_t)bm;
      if ((uint32_t)j < e) {
        off += c;
        full_before += c / bm;
      }
      full_all += c / bm;
      if (pj) {
        ++parts;
        if (pj > pe || (pj == pe && (uint32_t)j < e)) ++part_rank;
      }
    }
    base_s[0] = off;
    base_s[1] = full_before;
    base_s[2] = full_all + part_rank;  // slot of this expert's partial tile
    offsets[e] = off;
    if (e == 0) *n_tiles = full_all + parts;
  }
  // contiguous token range per thread; a token's 4 ids are one 16-byte row,
  // read 8 rows at a time so their loads are in flight together (one scalar
  // load after another left the kernel latency-bound)
  const int per = (m + 255) / 256;
  const int t0 = min(m, t * per), t1 = min(m, t0 + per);
  const bool vec = (reinterpret_cast<uintptr_t>(ids) & 15) == 0;
  const uint4* ids4 = reinterpret_cast<const uint4*>(ids);
  auto row_ids = [&](int tok) -> uint4 {
    if (vec) return __ldg(ids4 + tok);
    return make_uint4(__ldg(ids + 4 * (size_t)tok), __ldg(ids + 4 * (size_t)tok + 1),
                      __ldg(ids + 4 * (size_t)tok + 2), __ldg(ids + 4 * (size_t)tok + 3));
  };
  uint32_t c = 0;
  for (int b0 = t0; b0 < t1; b0 += 8) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (b0 + j < t1) v[j] = row_ids(b0 + j);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (b0 + j < t1) c += (v[j].x == e) + (v[j].y == e) + (v[j].z == e) + (v[j].w == e);
  }
  // block exclusive scan of c
  uint32_t incl = c;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  uint32_t wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += warp_tot[w];
  uint32_t pos = base_s[0] + wbase + incl - c;
  for (int b0 = t0; b0 < t1; b0 += 8) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (b0 + j < t1) v[j] = row_ids(b0 + j);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (b0 + j >= t1) break;
      const int tok = b0 + j;
      const uint32_t r4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
        if (r4[r] == e) {
          ids_sorted[pos] = (uint32_t)tok;
          slotpos[4 * (size_t)tok + r] = pos;
          ++pos;
        }
    }
  }
  // row tiles of this expert
  const uint32_t n = cnt_s[e];
  const uint32_t nt = (n + bm - 1) / bm, nfull = n / bm;
  for (uint32_t j = t; j < nt; j += 256) {
    const uint32_t slot = j < nfull ? base_s[1] + j : base_s[2];
    if (slot < (uint32_t)max_tiles) {
      const uint32_t m0 = base_s[0] + j * bm;
      tiles[slot] = make_uint4(m0, min(m0 + (uint32_t)bm, base_s[0] + n), e, 0u);
    }
  }
}

__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint4* __restrict__ table, const uint32_t* __restrict__ ids, int rows,
                   int h16, uint4* __restrict__ out) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  const size_t total = (size_t)rows * h16;
  if (i >= total) return;
  const size_t r = i / h16, c = i % h16;
  out[i] = __ldg(table + (size_t)__ldg(ids + r) * h16 + c);
}

__global__ void __launch_bounds__(256)
silu_mul_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u, uint4* __restrict__ out,
                size_t n8) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n8) return;
  const uint4 gv = __ldg(g + i), uv = __ldg(u + i);
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t ow[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t o = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float gf = mc_bf16_to_f32((uint16_t)(gw[j] >> (16 * h)));
      const float uf = mc_bf16_to_f32((uint16_t)(uw[j] >> (16 * h)));
      const float s = mc_round_bf16(mc_silu(gf));
      o |= (uint32_t)mc_f32_to_bf16(__fmul_rn(s, uf)) << (16 * h);
    }
    ow[j] = o;
  }
  out[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// out[t][h] = bf16(sum_r bf16(gw[t][r] * ed[slotpos[t][r]][h])), rank order
// from +0; thread = 8 consecutive h.
__global__ void __launch_bounds__(256)
combine_kernel(const uint16_t* __restrict__ ed, const uint32_t* __restrict__ slotpos,
               const uint16_t* __restrict__ gw, uint16_t* __restrict__ out, int m, int topk,
               int h8) {
  const size_t i = (size_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= (size_t)m * h8) return;
  const size_t t = i / h8, c = i % h8;
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.0f;
  if (topk == 4 && (reinterpret_cast<uintptr_t>(slotpos) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(gw) & 7) == 0) {
    // the token's four slots and weights in one load each, the four expert
    // rows' loads in flight together, summed in rank order as below
    const uint4 pp = __ldg(reinterpret_cast<const uint4*>(slotpos) + t);
    const uint2 ww = __ldg(reinterpret_cast<const uint2*>(gw) + t);
    const uint32_t pr[4] = {pp.x, pp.y, pp.z, pp.w};
    const uint32_t wr[4] = {ww.x & 0xffffu, ww.x >> 16, ww.y & 0xffffu, ww.y >> 16};
    uint4 v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = __ldg(reinterpret_cast<const uint4*>(ed + (size_t)pr[r] * h8 * 8) + c);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float w = mc_bf16_to_f32((uint16_t)wr[r]);
      const uint32_t vw[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
      for (int j = 0; j < 8; ++j)
        s[j] = __fadd_rn(s[j], mc_round_bf16(__fmul_rn(
                                   w, mc_bf16_to_f32((uint16_t)(vw[j >> 1] >> (16 * (j & 1)))))));
    }
  } else
  for (int r = 0; r < topk; ++r) {
    const uint32_t p = __ldg(slotpos + t * topk + r);
    const float w = mc_bf16_to_f32(__ldg(gw + t * topk + r));
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(ed + (size_t)p * h8 * 8) + c);
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
      s[j] = __fadd_rn(s[j], mc_round_bf16(__fmul_rn(
                                 w, mc_bf16_to_f32((uint16_t)(vw[j >> 1] >> (16 * (j & 1)))))));
  }
  uint4 o;
  o.x = (uint32_t)mc_f32_to_bf16(s[0]) | ((uint32_t)mc_f32_to_bf16(s[1]) << 16);
  o.y = (uint32_t)mc_f32_to_bf16(s[2]) | ((uint32_t)mc_f32_to_bf16(s[3]) << 16);
  o.z = (uint32_t)mc_f32_to_bf16(s[4]) | ((uint32_t)mc_f32_to_bf16(s[5]) << 16);
  o.w = (uint32_t)mc_f32_to_bf16(s[6]) | ((uint32_t)mc_f32_to_bf16(s[7]) << 16);
  reinterpret_cast<uint4*>(out)[i] = o;
}

}  // namespace

extern "C" int mc_moe_sort_map(mc_ctx* ctx, const uint32_t* ids, int m, int n_experts, int bm,
                               uint32_t* counts, uint32_t* offsets, uint32_t* ids_sorted,
                               uint32_t* slotpos, uint32_t* tiles, uint32_t* n_tiles,
                               int max_tiles) {
  MC_REQUIRE(ctx, "moe_sort_map: null context");
  MC_REQUIRE(m >= 1 && m <= (1 << 22), "moe_sort_map: m %d out of range", m);
  MC_REQUIRE(n_experts >= 1 && n_experts <= 1024, "moe_sort_map: n_experts %d", n_experts);
  MC_REQUIRE(bm >= 1 && bm <= 4096, "moe_sort_map: bm %d", bm);
  MC_REQUIRE(ids && counts && offsets && ids_sorted && slotpos && tiles && n_tiles,
             "moe_sort_map: null pointer");
  MC_REQUIRE(mc_aligned(tiles, 16), "moe_sort_map: tiles must be 16-byte aligned");
  const long need = ((long)m * 4 + bm - 1) / bm + n_experts;
  MC_REQUIRE(max_tiles >= need, "moe_sort_map: max_tiles %d < %ld", max_tiles, need);
  sort_count_kernel<<<n_experts, 256, 0, ctx->stream>>>(ids, m * 4, counts);
  int rc = mc_after_launch("sort_count_kernel");
  if (rc) return rc;
  sort_scatter_kernel<<<n_experts, 256, 0, ctx->stream>>>(ids, m, n_experts, bm, counts, offsets,
                                                          ids_sorted, slotpos,
                                                          reinterpret_cast<uint4*>(tiles), n_tiles,
                                                          max_tiles);
  return mc_after_launch("sort_scatter_kernel");
}

extern "C" int mc_gather_rows_bf16(mc_ctx* ctx, const uint16_t* table, const uint32_t* ids,
                                   int rows, int hidden, uint16_t* out) {
  MC_REQUIRE(ctx, "gather_rows_bf16: null context");
  MC_REQUIRE(table && ids && out, "gather_rows_bf16: null pointer");
  MC_REQUIRE(hidden % 8 == 0 && hidden > 0, "gather_rows_bf16: hidden %d must be a multiple of 8",
             hidden);
  MC_REQUIRE(mc_aligned(table, 16) && mc_aligned(out, 16), "gather_rows_bf16: 16-byte alignment");
  MC_REQUIRE(rows >= 0, "gather_rows_bf16: rows %d", rows);
  if (rows == 0) return MC_OK;
  const size_t total = (size_t)rows * (hidden / 8);
  gather_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(table), ids, rows, hidden / 8, reinterpret_cast<uint4*>(out));
  return mc_after_launch("gather_rows_kernel");
}

extern "C" int mc_silu_mul_bf16(mc_ctx* ctx, const uint16_t* gate, const uint16_t* up,
                                uint16_t* out, size_t n) {
  MC_REQUIRE(ctx, "silu_mul_bf16: null context");
  MC_REQUIRE(gate && up && out, "silu_mul_bf16: null pointer");
  MC_REQUIRE(n % 8 == 0, "silu_mul_bf16: n %zu must be a multiple of 8", n);
  MC_REQUIRE(mc_aligned(gate, 16) && mc_aligned(up, 16) && mc_aligned(out, 16),
             "silu_mul_bf16: 16-byte alignment");
  if (n == 0) return MC_OK;
  const size_t n8 = n / 8;
  silu_mul_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint4*>(gate), reinterpret_cast<const uint4*>(up),
      reinterpret_cast<uint4*>(out), n8);
  return mc_after_launch("silu_mul_kernel");
}

extern "C" int mc_moe_combine_rows(mc_ctx* ctx, const uint16_t* ed, const uint32_t* slotpos,
                                   const uint16_t* gw, uint16_t* out, int m, int topk,
                                   int hidden) {
  MC_REQUIRE(ctx, "moe_combine_rows: null context");
  MC_REQUIRE(ed && slotpos && gw && out, "moe_combine_rows: null pointer");
  MC_REQUIRE(hidden % 8 == 0 && hidden > 0, "moe_combine_rows: hidden %d", hidden);
  MC_REQUIRE(topk >= 1 && topk <= 8, "moe_combine_rows: topk %d", topk);
  MC_REQUIRE(mc_aligned(ed, 16) && mc_aligned(out, 16), "moe_combine_rows: 16-byte alignment");
  MC_REQUIRE(m >= 0, "moe_combine_rows: m %d", m);
  if (m == 0) return MC_OK;
  const size_t total = (size_t)m * (hidden / 8);
  combine_kernel<<<(unsigned)((total + 255) / 256), 256, 0, ctx->stream>>>(ed, slotpos, gw, out, m,
                                                                           topk, hidden / 8);
  return mc_after_launch("combine_kernel");
}

// ---------------------------------------------------------------- orchestration
// moe_prefill (lfm.rs:847-965) from router logits on. Workspace carve-up
// (every piece 256-byte aligned): ids u32[4m], gw bf16[4m], counts/offsets
// u32[E], ids_sorted/slotpos u32[4m], tiles uint4[max_tiles], n_tiles +
// status u32, gx bf16[4m][H], act bf16[4m][I], ed bf16[4m][H].
namespace {
// token rows per grouped-GEMM chunk (the kernel's MMA N is at most 256)
constexpr int kPrefillChunk = 256;

struct PrefillWs {
  size_t ids, gw, counts, offsets, ids_sorted, slotpos, tiles, ctl, gx, act, ed, total;
  int max_tiles;
};
PrefillWs prefill_layout(int m, int E, int H, int I) {
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t S = (size_t)m * 4;
  PrefillWs w;
  w.max_tiles = (int)((S + kPrefillChunk - 1) / kPrefillChunk + E);
  size_t o = 0;
  w.ids = o; o = al(o + S * 4);
  w.gw = o; o = al(o + S * 2);
  w.counts = o; o = al(o + (size_t)E * 4);
  w.offsets = o; o = al(o + (size_t)E * 4);
  w.ids_sorted = o; o = al(o + S * 4);
  w.slotpos = o; o = al(o + S * 4);
  w.tiles = o; o = al(o + (size_t)w.max_tiles * 16);
  w.ctl = o; o = al(o + 8);
  w.gx = o; o = al(o + S * H * 2);
  w.act = o; o = al(o + S * I * 2);
  w.ed = o; o = al(o + S * H * 2);
  w.total = o;
  return w;
}
}  // namespace

extern "C" size_t mc_moe_prefill_workspace_size(int m, int n_experts, int hidden, int moe_inter) {
  if (m < 1 || n_experts < 1 || hidden < 1 || moe_inter < 1) return 0;
  return prefill_layout(m, n_experts, hidden, moe_inter).total;
}

extern "C" int mc_moe_prefill(mc_ctx* ctx, const uint16_t* x, const float* logits, int m,
                              const mc_qweights* gate, const mc_qweights* up,
                              const mc_qweights* down, int n_experts, int route_mode,
                              const float* expert_bias, void* workspace, size_t ws_bytes,
                              uint16_t* out) {
  MC_REQUIRE(ctx, "moe_prefill: null context");
  MC_REQUIRE(gate && up && down && x && logits && workspace && out, "moe_prefill: null pointer");
  MC_REQUIRE(n_experts >= 4 && n_experts <= 64, "moe_prefill: n_experts %d", n_experts);
  MC_REQUIRE(m >= 1, "moe_prefill: m %d", m);
  const int H = gate->in_features;
  MC_REQUIRE(gate->out_features % n_experts == 0, "moe_prefill: stacked gate rows");
  const int I = gate->out_features / n_experts;
  MC_REQUIRE(down->in_features == I && down->out_features == n_experts * H,
             "moe_prefill: down shape [%d][%d] does not match E*H x I", down->out_features,
             down->in_features);
  const PrefillWs w = prefill_layout(m, n_experts, H, I);
  MC_REQUIRE(ws_bytes >= w.total, "moe_prefill: workspace %zu < %zu bytes", ws_bytes, w.total);
  MC_REQUIRE(mc_aligned(workspace, 256), "moe_prefill: workspace must be 256-byte aligned");
  uint8_t* base = static_cast<uint8_t*>(workspace);
  auto U32 = [&](size_t off) { return reinterpret_cast<uint32_t*>(base + off); };
  auto B16 = [&](size_t off) { return reinterpret_cast<uint16_t*>(base + off); };
  const int S = 4 * m;
  int rc;
  if ((rc = mc_moe_route_batch(ctx, logits, m, n_experts, route_mode, expert_bias, 1e-6f,
                               U32(w.ids), B16(w.gw))))
    return rc;
  if ((rc = mc_moe_sort_map(ctx, U32(w.ids), m, n_experts, kPrefillChunk, U32(w.counts), U32(w.offsets),
                            U32(w.ids_sorted), U32(w.slotpos), U32(w.tiles), U32(w.ctl),
                            w.max_tiles)))
    return rc;
  MC_CUDA(cudaMemsetAsync(U32(w.ctl) + 1, 0, 4, ctx->stream));
  if ((rc = mc_gather_rows_bf16(ctx, x, U32(w.ids_sorted), S, H, B16(w.gx)))) return rc;
  if ((rc = mc_gemm_q4_grouped_gu(ctx, B16(w.gx), S, gate, up, n_experts, B16(w.act), U32(w.tiles),
                                  U32(w.ctl), w.max_tiles, U32(w.ctl) + 1)))
    return rc;
  if ((rc = mc_gemm_q4_grouped(ctx, B16(w.act), S, down, n_experts, B16(w.ed), U32(w.tiles),
                               U32(w.ctl), w.max_tiles, U32(w.ctl) + 1)))
    return rc;
  return mc_moe_combine_rows(ctx, B16(w.ed), U32(w.slotpos), B16(w.gw), out, m, 4, H);
}

namespace {
__global__ void __launch_bounds__(256)
map_ids_kernel(uint32_t* __restrict__ ids, size_t n, const uint32_t* __restrict__ table, int E,
               uint32_t* __restrict__ status) {
  for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256) {
    const uint32_t v = ids[i];
    if (v < (uint32_t)E) {
      ids[i] = __ldg(table + v);
    } else if (status) {
      atomicOr(status, 2u);
    }
  }
}
}  // namespace

// Relabels expert ids in place through table[E] (an expert placement): the
// expert-parallel path routes on the model's expert numbering and sorts by
// the placement's, so any assignment of experts to ranks keeps each rank's
// experts contiguous. Ids out of range are left as they are and flagged.
extern "C" int mc_map_ids(mc_ctx* ctx, uint32_t* ids, size_t n, const uint32_t* table,
                          int n_experts, uint32_t* status) {
  MC_REQUIRE(ctx && ids && table && n_experts >= 1, "map_ids: bad arguments");
  if (n == 0) return MC_OK;
  const size_t blocks = (n + 255) / 256, cap = (size_t)ctx->num_sms * 4;
  const int grid = (int)(blocks < cap ? blocks : cap);
  map_ids_kernel<<<grid, 256, 0, ctx->stream>>>(ids, n, table, n_experts, status);
  return mc_after_launch("map_ids_kernel");
}
