// moe_decode (lfm.rs:967-1011) behind the fused router (lfm.rs:1154-1169) as
// ONE persistent launch (one CTA per SM) for one token (batch 1): add + RMSNorm +
// router + top-4 (router_addnorm_route), the four experts' gate/up GEMVs with
// SwiGLU (gemv_gather_act) and their down GEMVs with the weighted combine
// (gemv_gather_down_combine4), bit-identical to those three kernels.
//
// One CTA per SM, 16 warps. Timeline of a launch:
//  * warp 0 of CTAs 0..E-1 loads one router row; every CTA adds h + b and
//    normalises the row (each needs the normed row); the router warps then
//    publish their expert's logit, epoch-tagged, to the workspace;
//  * warp 0 of every CTA waits for the E logits and picks the same top-4;
//  * warps 0..7 issue this CTA's slice of the 4 experts' gate/up rows (codes,
//    scales, biases; a few contiguous row ranges) and down codes as 1-D bulk
//    copies into shared memory: the scales and biases first, then the codes
//    in chunks of 16 row pairs with one mbarrier each, then the down codes,
//    so the whole slice (~160 KB at I = 1536) is in flight at once --
//    per-thread loads reach far less of HBM's rate for a burst of this size;
//  * the warps compute the row pairs of each chunk as it lands, then publish
//    the bf16 act values as tagged words; each CTA polls and stages all act
//    rows and computes its down rows from shared memory and the weighted
//    combine.
//
// Published values are self-validating words carrying the launch's epoch tag
// (logits: tag32 << 32 | f32 bits). The caller's workspace (u32 words, zeroed
// once, then owned by one chain of calls) holds:
//   ws[0]            epoch (advanced by the last CTA to finish)
//   ws[1]            CTAs finished (reset by the last one)
//   ws[2]            sticky error status bits: 1 logits wait gave up,
//                    2 expert id out of range, 8 act wait, 16 a copy wait,
//                    32 projection wait
//   ws[3]            reserved (zero)
//   ws[4]            CTAs whose projection rows are stored (fused
//                    projection only; reset by the last CTA to finish)
//   ws[5..8)         reserved (zero)
//   ws[8..136)       64 tagged logits (u64: tag32 << 32 | f32 bits)
//   ws[136..)        act values [slot][row], one tagged word each
//                    (tag16 << 16 | bf16 bits, tag16 = tag32 % 65535 + 1)
//   ws[136 + 4I..)   with the fused projection: its 2048 bf16 outputs
//                    (4 KB; 2048 words reserved)
// Every wait is bounded by a %globaltimer deadline; a CTA whose copies did
// not all land waits for them (bounded again) before it exits.
//
// Arithmetic per output is the canonical order of the separate kernels, so
// results are bit-identical to router_addnorm_route + gemv_gather_act +
// gemv_gather_down_combine4 and to the CPU oracle.
#include <atomic>

#include "gemv_common.cuh"
#include "mc_async.cuh"
#include "route_common.cuh"
#include "rownorm.cuh"

namespace {

constexpr int kThreads = 512;  // 16 warps, 4 per scheduler (<= 128 registers a thread)
constexpr int kWarps = kThreads / 32;
constexpr int kMaxChunks = 8;   // gate/up chunks: 16 row pairs, then 32 each (up to 240)
constexpr int kDnRows = 4;      // down rows per warp (16 warps, 4 per expert)
constexpr int H = 2048;
constexpr unsigned long long kTimeoutNs = 200000000ull;  // default limit per wait: 200 ms
constexpr int kLogitWord = 8;   // first tagged-logit word in the workspace
constexpr int kActWord = 136;   // first act word in the workspace
constexpr uint32_t kPrologueBytes = 8192 + 4096;  // normed row as f32 and as bf16

// Byte offsets in dynamic shared memory (identical on host and device).
// Gate/up chunk c (one mbarrier each) holds local row pairs
// [chunk_begin(c), chunk_begin(c + 1)): 16 first (one per warp, so compute
// starts early), then 32 (two per warp, two independent pairs in flight).
__host__ __device__ inline int chunk_begin(int c) {
  return c == 0 ? 0 : kWarps + 2 * kWarps * (c - 1);
}
__host__ __device__ inline int chunk_count(int np) {
  return np <= kWarps ? 1 : 1 + (np - kWarps + 2 * kWarps - 1) / (2 * kWarps);
}

struct Layout {
  int np_max, nr_max, nchunk_max;
  uint32_t uc, sb, dn, pro, pj, total;
};

// With `proj` the layout ends with this CTA's projection rows: nr_max rows of
// Q4 codes (1024 B each), then their scales, then their biases (64 B each).
__host__ __device__ inline Layout make_layout(int I, int G, bool proj = false) {
  Layout L;
  L.np_max = (4 * I + G - 1) / G;
  L.nr_max = (H + G - 1) / G;
  L.nchunk_max = chunk_count(L.np_max);
  L.uc = (uint32_t)L.np_max * (H / 2);      // gate codes at 0, up codes here
  L.sb = 2 * L.uc;                          // gate scales, gate biases, up scales, up biases
  L.dn = L.sb + 4u * (uint32_t)L.np_max * 64u;
  L.pro = L.dn + 4u * (uint32_t)L.nr_max * (uint32_t)(I / 2);
  const uint32_t act_bytes = 8u * (uint32_t)I;  // 4 x I bf16, reuses the prologue area
  L.total = L.pro + (act_bytes > kPrologueBytes ? act_bytes : kPrologueBytes);
  L.pj = L.total;
  if (proj) L.total += (uint32_t)L.nr_max * (H / 2 + 128u);
  return L;
}

struct Params {
  const uint16_t* h;
  const uint16_t* badd;
  const uint16_t* norm_w;
  uint16_t* h_out;
  uint16_t* normed;
  const void* router_w;
  const float* ebias;
  float* logits;
  uint32_t* ids;
  uint16_t* wts;
  mc_qweights gate, up, down;
  uint16_t* out;
  uint32_t* sync;
  float eps, route_eps;
  int mode, E, I;
  unsigned long long* trace;
  const uint8_t* pf[2];  // L2 prefetch ranges for the next layer (128-byte lines)
  uint32_t pf_lines[2];
  unsigned long long timeout_ns;  // limit of every bounded wait (mc_set_wait_limit)
  // report_status: the last CTA moves ws[2] to *status_out (when non-null)
  // and clears it, so the word reports one launch (the allocation-free entry
  // point); otherwise ws[2] stays sticky in the caller's workspace
  uint32_t* status_out;
  int report_status;
  int skip_publish;  // test aid (mc_set_test_flags): router warps publish nothing
  // fused projection (mc_moe_decode_layer_proj): b = bf16(proj . h) computed
  // here, row slice [i0, i1) per CTA, exchanged as tagged words; p_out
  // (nullable) receives b
  mc_qweights proj;
  uint16_t* p_out;
};

constexpr int kTraceSlots = 32;  // per-CTA phase timestamps (mc_set_trace)
#define TRACE(k) \
  do { if (P.trace && t == 0) P.trace[kTraceSlots * blockIdx.x + (k)] = mc_globaltimer(); } while (0)

__device__ __forceinline__ void record_error(uint32_t* sync, uint32_t bit) {
  atomicOr(sync + 2, bit);
}

// Waits for phase 0 of `bar` until `deadline`; the waiting warp sleeps
// between polls.
__device__ __forceinline__ bool wait_copies(uint64_t* bar, unsigned long long deadline) {
  while (!mc_mbar_test_sleep(bar, 0, 20000u))
    if (mc_globaltimer() > deadline) return false;
  return true;
}

// One Q4 group (32 code bytes) of a row in shared memory.
__device__ __forceinline__ float smem_group_qx(const uint8_t* p, const float2* xs) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  return q4_group_qx(q[0], q[1], xs);
}

template <int DT, bool PROJ>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(const Params P,
                                                                      const Layout L) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float red[8];
  __shared__ float zs[64];
  __shared__ uint32_t ids_s[4];
  __shared__ uint16_t wts_s[4];
  __shared__ float p_s[4][32];
  __shared__ float gu_s[2][256];  // bf16-rounded gate and up sums per local pair
  __shared__ uint32_t flag_s;
  __shared__ __align__(8) uint64_t bar_sb, bar_dn, bar_gu[kMaxChunks], bar_pj;

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int I = P.I;
  const int npairs = 4 * I;
  const int p0 = (int)(((long)cta * npairs) / G), p1 = (int)(((long)(cta + 1) * npairs) / G);
  const int i0 = (int)(((long)cta * H) / G), i1 = (int)(((long)(cta + 1) * H) / G);
  const int np = p1 - p0, nr = i1 - i0;
  const int nchunk = chunk_count(np);
  const int dn_code = I / 2, Gd = I / 64;
  uint32_t* sync = P.sync;
  unsigned long long* logits64 = reinterpret_cast<unsigned long long*>(sync + kLogitWord);
  uint32_t* actw = sync + kActWord;
  float* nrow = reinterpret_cast<float*>(sm + L.pro);
  uint16_t* nbf = reinterpret_cast<uint16_t*>(sm + L.pro + 8192);
  uint16_t* act_s = reinterpret_cast<uint16_t*>(sm + L.pro);  // after the prologue
  const bool router_cta = cta < P.E;
  const unsigned long long t_start = mc_globaltimer();
  bool ok = true;
  TRACE(0);

  // ---- barriers, the router row (warp 0 of a router CTA, into registers),
  // and this thread's h / b / norm_w words
  if (t == 0) {
    flag_s = 0;
    mc_mbar_init(&bar_sb, 1);
    mc_mbar_init(&bar_dn, 1);
    for (int c = 0; c < kMaxChunks; ++c) mc_mbar_init(bar_gu + c, 1);
    mc_mbar_init(&bar_pj, 1);
    mc_fence_barrier_init();
    // the byte counts of this CTA's expert-row copies depend only on its
    // slice, not on the experts chosen: posted now, so the copies can be
    // issued by several warps as soon as the top-4 is known
    mc_mbar_expect_tx(&bar_sb, (uint32_t)np * 256u);
    for (int c = 0; c < nchunk; ++c) {
      const int q0 = chunk_begin(c), q1 = min(np, chunk_begin(c + 1));
      mc_mbar_expect_tx(bar_gu + c, (uint32_t)(q1 - q0) * (uint32_t)H);
    }
    mc_mbar_expect_tx(&bar_dn, 4u * (uint32_t)nr * (uint32_t)dn_code);
    // this CTA's projection rows (weights: never written by earlier kernels,
    // so they stream in before the programmatic-dependent-launch wait)
    if (PROJ && nr > 0) {
      const uint64_t pol = mc_policy_evict_first();
      mc_mbar_expect_tx(&bar_pj, (uint32_t)nr * (H / 2 + 128u));
      mc_bulk_g2s(sm + L.pj, reinterpret_cast<const uint8_t*>(P.proj.codes) + (size_t)i0 * (H / 2),
                  (uint32_t)nr * (H / 2), &bar_pj, pol);
      mc_bulk_g2s(sm + L.pj + (uint32_t)L.nr_max * (H / 2), P.proj.scales + (size_t)i0 * 32,
                  (uint32_t)nr * 64u, &bar_pj, pol);
      mc_bulk_g2s(sm + L.pj + (uint32_t)L.nr_max * (H / 2 + 64u), P.proj.biases + (size_t)i0 * 32,
                  (uint32_t)nr * 64u, &bar_pj, pol);
    }
  }
  RouterRow<DT> rr;
  if (router_cta && warp == 0) {
    // the element assignment of RouterRow::load, as streaming loads issued now
    const uint4* row = reinterpret_cast<const uint4*>(
        reinterpret_cast<const uint8_t*>(P.router_w) + (size_t)cta * (DT == MC_DTYPE_BF16 ? 2 * H : 4 * H));
    uint4* w = reinterpret_cast<uint4*>(rr.w);
    if (DT == MC_DTYPE_BF16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) w[j] = mc_ldg_stream(row + 32 * j + lane);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        w[2 * j] = mc_ldg_stream(row + 64 * j + 2 * lane);
        w[2 * j + 1] = mc_ldg_stream(row + 64 * j + 2 * lane + 1);
      }
    }
  }
  uint4 hv = make_uint4(0, 0, 0, 0), bv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
  if (t < 256) wv = mc_ldg_stream(reinterpret_cast<const uint4*>(P.norm_w) + t);
  // weights above may be read before the previous kernel of the stream has
  // finished; its outputs (h, b, the workspace) only after this wait
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  TRACE(22);
  if (t < 256) {
    hv = mc_ldg_stream(reinterpret_cast<const uint4*>(P.h) + t);
    if (P.badd) bv = mc_ldg_stream(reinterpret_cast<const uint4*>(P.badd) + t);
  }
  if (P.trace && t == 0) {  // profiling aid: when the h / b and norm words arrive
    asm volatile("" ::"r"(hv.x), "r"(bv.w));
    TRACE(23);
    asm volatile("" ::"r"(wv.x), "r"(wv.w));
    TRACE(29);
  }
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(sync);
  const uint32_t tag32 = epoch == 0xffffffffu ? 1u : epoch + 1u;
  const uint32_t tag16 = tag32 % 65535u + 1u;  // never 0, differs from the last launch's

  // ---- fused projection: warp 1 + j computes row i0 + j of b = proj . h in
  // the canonical GEMV order (gemv_kernel, K = 2048: lane l owns group l,
  // term = fma(s, qx, b * xg), 32-lane butterfly), bit-identical to
  // gemv_quant, and stores it (bf16) into the workspace; once a CTA's rows
  // are stored (a barrier over the projection warps), one release increment
  // of ws[4] counts the CTA, and the CTAs read b once ws[4] reaches the grid
  // size. (Epoch-tagged
  // words polled by every thread, as the act rows are, measured far slower
  // here: 148 x 256 pollers over the same 8 KB of lines delayed the stores
  // they waited for by up to 12 us.)
  uint16_t* pw16 = reinterpret_cast<uint16_t*>(sync + kActWord + 4 * I);
  if (PROJ && warp >= 1 && warp <= nr) {
    const int j = warp - 1;
    float2 xsh[32];
    const float xgh = load_group_x<4>(P.h, lane, xsh);
    if (wait_copies(&bar_pj, mc_globaltimer() + P.timeout_ns)) {
      const uint16_t* psb = reinterpret_cast<const uint16_t*>(sm + L.pj + (uint32_t)L.nr_max * (H / 2));
      const float s = mc_bf16_to_f32(psb[j * 32 + lane]);
      const float bb = mc_bf16_to_f32(psb[L.nr_max * 32 + j * 32 + lane]);
      const float acc = __fadd_rn(
          0.0f, __fmaf_rn(s, smem_group_qx(sm + L.pj + (uint32_t)j * (H / 2) + 32 * lane, xsh),
                          __fmul_rn(bb, xgh)));
      const float sum = mc_warp_butterfly(acc);
      if (lane == 0) {
        const uint16_t v = (uint16_t)mc_f32_to_bf16(sum);
        __stcg(pw16 + i0 + j, v);
        if (P.p_out) P.p_out[i0 + j] = v;
        // profiling aid: when this CTA's first projection row is stored
        if (P.trace && j == 0) P.trace[kTraceSlots * blockIdx.x + 5] = mc_globaltimer();
      }
    } else if (lane == 0) {
      record_error(sync, 32u);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nr * 32) : "memory");
    if (warp == 1 && lane == 0) mc_red_release_add(sync + 4, 1u);
  }
  if (PROJ && t < 256) {
    if (t == 0) {
      const unsigned long long deadline = mc_globaltimer() + P.timeout_ns;
      while (mc_ld_acquire(sync + 4) < (uint32_t)G) {
        if (mc_globaltimer() > deadline) {
          record_error(sync, 32u);
          break;
        }
        __nanosleep(64);
      }
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    bv = __ldcg(reinterpret_cast<const uint4*>(pw16) + t);
    TRACE(8);
  }
  const bool has_b = P.badd != nullptr || PROJ;

  // ---- add + RMSNorm (canonical order of addnorm_row_2048)
  float hp[8];
  if (t < 256) {
    float acc = 0.0f;
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float hf = mc_bf16_to_f32((uint16_t)(hw[i >> 1] >> (16 * (i & 1))));
      float v = hf;
      if (has_b) v = __fadd_rn(hf, mc_bf16_to_f32((uint16_t)(bw[i >> 1] >> (16 * (i & 1)))));
      hp[i] = mc_round_bf16(v);
      acc = __fmaf_rn(hp[i], hp[i], acc);
    }
    acc = mc_warp_butterfly(acc);
    if (lane == 0) red[warp] = acc;
  }
  __syncthreads();
  if (t < 256) {
    float total = red[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) total = __fadd_rn(total, red[j]);
    const float inv =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(total, 1.0f / 2048.0f), P.eps)));
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float wf = mc_bf16_to_f32((uint16_t)(ww[i >> 1] >> (16 * (i & 1))));
      n[i] = mc_round_bf16(__fmul_rn(__fmul_rn(hp[i], inv), wf));
    }
    reinterpret_cast<float4*>(nrow)[2 * t] = make_float4(n[0], n[1], n[2], n[3]);
    reinterpret_cast<float4*>(nrow)[2 * t + 1] = make_float4(n[4], n[5], n[6], n[7]);
    const uint4 nb = pack8_bf16(n);
    // chunk t of the row = chunk t & 7 of group t >> 3, stored swizzled for
    // load_group_x<., 2>
    reinterpret_cast<uint4*>(nbf)[(t & ~7) | ((t & 7) ^ ((t >> 3) & 7))] = nb;
    if (cta == 0) {
      reinterpret_cast<uint4*>(P.h_out)[t] = pack8_bf16(hp);
      reinterpret_cast<uint4*>(P.normed)[t] = nb;
    }
  }
  __syncthreads();
  TRACE(1);

  // ---- router logit of expert `cta` (warp 0), published epoch-tagged: the
  // tag and the value share one 64-bit word, so a reader that sees this
  // launch's tag has the value (no fence, no counter)
  if (router_cta && warp == 0) {
    if (P.trace && t == 0) {  // profiling aid: when the router row arrives
      const uint4* w = reinterpret_cast<const uint4*>(rr.w);
      uint32_t all = 0;
#pragma unroll
      for (int j = 0; j < (DT == MC_DTYPE_BF16 ? 8 : 16); ++j) all ^= w[j].x ^ w[j].w;
      asm volatile("" ::"r"(all));
      TRACE(20);
      TRACE(21);
    }
    const float z = rr.dot(nrow, lane);
    TRACE(13);
    if (lane == 0 && !P.skip_publish) {
      P.logits[cta] = z;
      mc_st_publish_u64(logits64 + cta,
                        ((unsigned long long)tag32 << 32) | (unsigned long long)__float_as_uint(z));
    }
  }
  TRACE(2);

  // ---- gate/up activations prescaled once (all warps), meanwhile warp 0
  // gathers the tagged logits: lane l polls logits 2l, 2l+1 (one 16-byte
  // load) until both carry this launch's tag
  float2 xs[32];
  const float xg = load_group_x<4, 2>(nbf, lane, xs);
  if (warp == 0) {
    const unsigned long long deadline = mc_globaltimer() + P.timeout_ns;
    bool got = true;
    TRACE(14);
    if (2 * lane < P.E) {
      const int i = 2 * lane;
      unsigned long long v0, v1;
      for (;;) {
        mc_ld_poll_v2u64(logits64 + i, v0, v1);
        const bool ready0 = (v0 >> 32) == tag32, ready1 = i + 1 >= P.E || (v1 >> 32) == tag32;
        if (ready0 && ready1) break;
        if (mc_globaltimer() > deadline) {
          got = false;
          break;
        }
        __nanosleep(32);
      }
      zs[i] = __uint_as_float((uint32_t)v0);
      if (i + 1 < P.E) zs[i + 1] = __uint_as_float((uint32_t)v1);
    }
    got = __all_sync(0xffffffffu, got);
    TRACE(15);
    if (!got) {
      if (lane == 0) {
        record_error(sync, 1u);
        flag_s = 1;
      }
    } else {
      __syncwarp();
      uint32_t ids_l[4];
      uint16_t w_l[4];
      warp_top4(zs, P.E, P.mode, P.ebias, P.route_eps, ids_l, w_l);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          ids_s[r] = ids_l[r];
          wts_s[r] = w_l[r];
          if (ids_l[r] >= (uint32_t)P.E) flag_s = 2;
          if (cta == 0) {
            P.ids[r] = ids_l[r];
            P.wts[r] = w_l[r];
          }
        }
        if (flag_s == 2) record_error(sync, 2u);
      }
      TRACE(12);
    }
  }
  __syncthreads();
  TRACE(3);
  if (flag_s) ok = false;

  // ---- lane 0 of warps 0..7 issue this CTA's expert rows as bulk copies
  // (copy k from warp k % 8; their byte counts were posted at the start):
  // the gate/up scales and biases, the gate/up codes chunk by chunk, then
  // the down codes. (From one warp's lanes in turn the ~24 issues took
  // 0.2 us longer.)
  const bool issued = ok;
  if (ok && warp < 8) {
    const uint64_t pol = mc_policy_evict_first();
    int k = 0;
    auto emit = [&](uint32_t dst, const void* src, uint32_t n, uint64_t* bar) {
      if ((k++ & 7) == warp && lane == 0) mc_bulk_g2s(sm + dst, src, n, bar, pol);
    };
    // local pairs [0, qs) and [qs, np) each lie in one expert slot
    const int qs = min(np, (p0 / I + 1) * I - p0);
    const uint32_t sbs = (uint32_t)L.np_max * 64u;
#pragma unroll
    for (int sg = 0; sg < 2; ++sg) {
      const int qa = sg == 0 ? 0 : qs, qb = sg == 0 ? qs : np;
      if (qa >= qb) continue;
      const int slot = (p0 + qa) / I;
      const size_t row = (size_t)ids_s[slot] * I + (p0 + qa - slot * I);
      const uint32_t n = (uint32_t)(qb - qa) * 64u, d = L.sb + (uint32_t)qa * 64u;
      emit(d, P.gate.scales + row * 32, n, &bar_sb);
      emit(d + sbs, P.gate.biases + row * 32, n, &bar_sb);
      emit(d + 2 * sbs, P.up.scales + row * 32, n, &bar_sb);
      emit(d + 3 * sbs, P.up.biases + row * 32, n, &bar_sb);
    }
    for (int c = 0; c < nchunk; ++c) {
      const int q0 = chunk_begin(c), q1 = min(np, chunk_begin(c + 1));
#pragma unroll
      for (int sg = 0; sg < 2; ++sg) {
        const int qa = max(q0, sg == 0 ? 0 : qs), qb = min(q1, sg == 0 ? qs : np);
        if (qa >= qb) continue;
        const int slot = (p0 + qa) / I;
        const size_t row = (size_t)ids_s[slot] * I + (p0 + qa - slot * I);
        const uint32_t n = (uint32_t)(qb - qa);
        emit((uint32_t)qa * (H / 2), reinterpret_cast<const uint8_t*>(P.gate.codes) + row * (H / 2),
             n * (H / 2), bar_gu + c);
        emit(L.uc + (uint32_t)qa * (H / 2),
             reinterpret_cast<const uint8_t*>(P.up.codes) + row * (H / 2), n * (H / 2), bar_gu + c);
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const size_t row = (size_t)ids_s[r] * H + i0;
      emit(L.dn + (uint32_t)(r * L.nr_max) * (uint32_t)dn_code,
           reinterpret_cast<const uint8_t*>(P.down.codes) + row * dn_code,
           (uint32_t)(nr * dn_code), &bar_dn);
    }
  }
  TRACE(11);

  // ---- gate/up from shared memory as the chunks land: warp w takes pair w
  // of chunk 0 and pairs w, w + 16 of every later chunk; lane 0 keeps the
  // bf16-rounded sums, SwiGLU runs once all pairs are done
  bool copies_ok = true;
  if (ok) {
    const unsigned long long deadline = mc_globaltimer() + P.timeout_ns;
    const uint32_t sbs = (uint32_t)L.np_max * 64u;
    const uint16_t* sb16 = reinterpret_cast<const uint16_t*>(sm + L.sb);
    // gate and up sums of pair q (all lanes get the butterflied values)
    auto pair_terms = [&](int q, float& ag, float& au) {
      const float gs = mc_bf16_to_f32(sb16[(q * 64u) / 2 + lane]);
      const float gb = mc_bf16_to_f32(sb16[(sbs + q * 64u) / 2 + lane]);
      const float us = mc_bf16_to_f32(sb16[(2 * sbs + q * 64u) / 2 + lane]);
      const float ub = mc_bf16_to_f32(sb16[(3 * sbs + q * 64u) / 2 + lane]);
      ag = __fadd_rn(0.0f, __fmaf_rn(gs, smem_group_qx(sm + q * (H / 2) + 32 * lane, xs),
                                     __fmul_rn(gb, xg)));
      au = __fadd_rn(0.0f, __fmaf_rn(us, smem_group_qx(sm + L.uc + q * (H / 2) + 32 * lane, xs),
                                     __fmul_rn(ub, xg)));
    };
    if (warp < np && !wait_copies(&bar_sb, deadline)) copies_ok = false;
    for (int c = 0; copies_ok && c < nchunk; ++c) {
      const int qb = chunk_begin(c), qe = min(np, chunk_begin(c + 1));
      const int q = qb + warp;
      if (q >= qe) break;
      if (!wait_copies(bar_gu + c, deadline)) {
        copies_ok = false;
        break;
      }
      if (c < 8) TRACE(16 + c);
      if (c == 0) {
        float ag, au;
        pair_terms(q, ag, au);
        ag = mc_warp_butterfly(ag);
        au = mc_warp_butterfly(au);
        if (lane == 0) {
          gu_s[0][q] = mc_round_bf16(ag);
          gu_s[1][q] = mc_round_bf16(au);
        }
      } else {
        const int q2 = q + kWarps, q2c = min(q2, qe - 1);  // a repeat of q when absent
        float ag, au, ag2, au2;
        pair_terms(q, ag, au);
        pair_terms(q2c, ag2, au2);
        ag = mc_warp_butterfly(ag);
        au = mc_warp_butterfly(au);
        ag2 = mc_warp_butterfly(ag2);
        au2 = mc_warp_butterfly(au2);
        if (lane == 0) {
          gu_s[0][q] = mc_round_bf16(ag);
          gu_s[1][q] = mc_round_bf16(au);
          if (q2 < qe) {
            gu_s[0][q2] = mc_round_bf16(ag2);
            gu_s[1][q2] = mc_round_bf16(au2);
          }
        }
      }
      if (c < 8) TRACE(24 + c);
    }
    if (!copies_ok && lane == 0) {
      record_error(sync, 16u);
      flag_s = 1;
    }
  }
  __syncthreads();
  TRACE(4);
  // the next layer's router and norm weights into L2 (mc_set_l2_prefetch):
  // this CTA's share of the lines, while the act rows are exchanged
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint32_t n = P.pf_lines[r];
    for (uint32_t l = (uint32_t)cta * kThreads + t; l < n; l += (uint32_t)G * kThreads)
      asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(P.pf[r] + 128ull * l));
  }
  // SwiGLU per pair, one thread each: act = bf16(bf16(silu(g)) * u),
  // published as a tagged word (tag16 << 16 | bf16 bits)
  if (ok && t < np) {
    const float sl = mc_round_bf16(mc_silu(gu_s[0][t]));
    const uint32_t a = mc_f32_to_bf16(__fmul_rn(sl, gu_s[1][t]));
    mc_st_publish_u32(actw + p0 + t, (tag16 << 16) | a);
  }

  // ---- down scales and biases of this warp's rows (their rows are not
  // 16-byte multiples for every I), loaded while the act rows are exchanged
  const int dr = warp & 3, j0 = warp >> 2;  // slot, first row (rows j0, j0+4, ...)
  uint16_t dsc[kDnRows] = {}, dbi[kDnRows] = {};
  if (ok && lane < Gd) {
#pragma unroll
    for (int k = 0; k < kDnRows; ++k) {
      const int j = min(j0 + 4 * k, nr - 1);
      const size_t row = (size_t)ids_s[dr] * H + i0 + j;
      dsc[k] = __ldg(P.down.scales + row * Gd + lane);
      dbi[k] = __ldg(P.down.biases + row * Gd + lane);
    }
  }

  // ---- stage the act rows once per CTA: poll the tagged words (8 per
  // 32 bytes) until every tag is this launch's, then store the bf16 values
  // to shared memory, 16-byte chunks swizzled so the per-lane group reads
  // below are bank-conflict free
  if (ok) {
    const unsigned long long deadline = mc_globaltimer() + P.timeout_ns;
    const int nchunk16 = (4 * I) / 8;  // chunks of 8 act values
    bool got = true;
    for (int c = t; got && c < nchunk16; c += kThreads) {
      uint4 a, b;
      for (;;) {
        a = mc_ld_poll_v4(actw + 8 * c);
        b = mc_ld_poll_v4(actw + 8 * c + 4);
        const uint32_t hi = (a.x >> 16) & (a.y >> 16) & (a.z >> 16) & (a.w >> 16) &
                            (b.x >> 16) & (b.y >> 16) & (b.z >> 16) & (b.w >> 16);
        const uint32_t lo = (a.x >> 16) | (a.y >> 16) | (a.z >> 16) | (a.w >> 16) |
                            (b.x >> 16) | (b.y >> 16) | (b.z >> 16) | (b.w >> 16);
        if (hi == tag16 && lo == tag16) break;  // all eight tags equal tag16
        if (mc_globaltimer() > deadline) {
          got = false;
          break;
        }
        __nanosleep(64);
      }
      const uint4 v = make_uint4(__byte_perm(a.x, a.y, 0x5410), __byte_perm(a.z, a.w, 0x5410),
                                 __byte_perm(b.x, b.y, 0x5410), __byte_perm(b.z, b.w, 0x5410));
      const int g = c >> 3;  // 64-value group (across slots)
      reinterpret_cast<uint4*>(act_s)[(g << 3) | ((c & 7) ^ (g & 7))] = v;
    }
    if (!got) {
      record_error(sync, 8u);
      flag_s = 1;
    }
  }
  __syncthreads();
  TRACE(10);
  if (flag_s) ok = false;

  // ---- down rows from shared memory + weighted combine
  if (ok) {
    float2 dxs[32];
    float dxg = 0.0f;
    if (lane < Gd) {
      const int g = dr * Gd + lane;
      const uint4* src = reinterpret_cast<const uint4*>(act_s) + (g << 3);
      float xv[64];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = src[c ^ (g & 7)];
        const uint32_t wds[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          xv[8 * c + 2 * h] = __uint_as_float(wds[h] << 16);
          xv[8 * c + 2 * h + 1] = __uint_as_float(wds[h] & 0xffff0000u);
        }
      }
      dxg = prescale_group_x<4>(xv, dxs);
    }
    TRACE(28);
    const bool landed = wait_copies(&bar_dn, mc_globaltimer() + P.timeout_ns);
    if (!landed && lane == 0) record_error(sync, 16u);
    TRACE(9);
    if (landed && nr > 0) {
      float acc[kDnRows] = {};
      if (lane < Gd) {  // one branch around all rows so their chains interleave
#pragma unroll
        for (int k = 0; k < kDnRows; ++k) {
          const int j = min(j0 + 4 * k, nr - 1);
          const uint8_t* rowp = sm + L.dn + (uint32_t)(dr * L.nr_max + j) * (uint32_t)dn_code;
          const float s = mc_bf16_to_f32(dsc[k]);
          const float b = mc_bf16_to_f32(dbi[k]);
          acc[k] = __fadd_rn(0.0f, __fmaf_rn(s, smem_group_qx(rowp + 32 * lane, dxs),
                                             __fmul_rn(b, dxg)));
        }
      }
#pragma unroll
      for (int k = 0; k < kDnRows; ++k) {
        const float sum = mc_warp_butterfly(acc[k]);
        if (lane == 0 && j0 + 4 * k < nr) p_s[dr][j0 + 4 * k] = mc_round_bf16(sum);
      }
    }
  }
  __syncthreads();
  TRACE(6);
  if (ok && t < nr) {
    float tot = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r)
      tot = __fadd_rn(tot, mc_round_bf16(__fmul_rn(mc_bf16_to_f32(wts_s[r]), p_s[r][t])));
    P.out[i0 + t] = mc_f32_to_bf16(tot);
  }

  // ---- every issued copy has landed before the CTA exits (immediate unless
  // a wait above gave up)
  if (t == 0 && issued) {
    const unsigned long long deadline = mc_globaltimer() + P.timeout_ns;
    bool all = wait_copies(&bar_sb, deadline) && wait_copies(&bar_dn, deadline);
    for (int c = 0; issued && c < nchunk; ++c) all = wait_copies(bar_gu + c, deadline) && all;
    if (!all) record_error(sync, 16u);
  }
  if (t == 0 && PROJ && nr > 0 &&
      !wait_copies(&bar_pj, mc_globaltimer() + P.timeout_ns))
    record_error(sync, 16u);

  // ---- the last CTA to finish resets the counters and advances the epoch
  TRACE(7);
  if (t == 0) {
    if (P.report_status) __threadfence();  // this CTA's status bits before its count
    const uint32_t done = atomicAdd(sync + 1, 1u);
    if (done == (uint32_t)G - 1) {
      if (P.report_status) {
        __threadfence();
        const uint32_t st = atomicExch(sync + 2, 0u);
        if (P.status_out) *P.status_out = st;
      }
      sync[1] = 0u;
      sync[4] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(sync) = tag32;
    }
  }
}

}  // namespace

extern "C" size_t mc_moe_decode_workspace_words(int moe_inter) {
  return (size_t)kActWord + 4 * (size_t)(moe_inter > 0 ? moe_inter : 0);
}

extern "C" size_t mc_moe_decode_proj_workspace_words(int moe_inter) {
  return mc_moe_decode_workspace_words(moe_inter) + H;
}

// The fused decode layer behind both entry points. With `noalloc` the
// workspace arguments are ignored: every argument is checked first, then the
// library's built-in scratch is fetched (its first use on a device sets it
// up), and the launch reports its status word to `status_out` and clears it.
int mc_decode_layer_impl(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                         const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                         const void* router_w, int router_dtype, const float* expert_bias,
                         int route_mode, float* logits, uint32_t* ids, uint16_t* weights,
                         const mc_qweights* gate, const mc_qweights* up, const mc_qweights* down,
                         int n_experts, uint16_t* out, uint32_t* sync, size_t ws_words, float eps,
                         float route_eps, bool noalloc, uint32_t* status_out,
                         const mc_qweights* proj, uint16_t* p_out) {
  MC_REQUIRE(ctx, "moe_decode_layer: null context");
  int rc;
  if (proj) {
    if ((rc = mc_check_gemv_weights(proj, "moe_decode_layer_proj proj"))) return rc;
    MC_REQUIRE(proj->bits == 4 && proj->in_features == H && proj->out_features == H &&
                   proj->group_size == 64,
               "moe_decode_layer_proj: proj must be Q4 2048 x 2048, group 64");
    MC_REQUIRE(mc_aligned(proj->codes, 16) && mc_aligned(proj->scales, 16) &&
                   mc_aligned(proj->biases, 16),
               "moe_decode_layer_proj: proj buffers must be 16-byte aligned");
    MC_REQUIRE(!b && !noalloc, "moe_decode_layer_proj: b is computed, not passed");
  }
  if ((rc = mc_check_gemv_weights(gate, "moe_decode_layer gate"))) return rc;
  if ((rc = mc_check_gemv_weights(up, "moe_decode_layer up"))) return rc;
  if ((rc = mc_check_gemv_weights(down, "moe_decode_layer down"))) return rc;
  MC_REQUIRE(gate->bits == 4 && up->bits == 4 && down->bits == 4,
             "moe_decode_layer: experts must be 4-bit");
  MC_REQUIRE(n_experts >= 4 && n_experts <= 64, "moe_decode_layer: n_experts %d", n_experts);
  MC_REQUIRE(gate->in_features == H && up->in_features == H,
             "moe_decode_layer: hidden must be 2048");
  MC_REQUIRE(gate->out_features % n_experts == 0 && up->out_features == gate->out_features,
             "moe_decode_layer: stacked gate/up rows");
  const int I = gate->out_features / n_experts;
  MC_REQUIRE(I % 64 == 0 && I <= 2048 && 4 * I <= 4 * 2048 && down->in_features == I &&
                 down->out_features == n_experts * H,
             "moe_decode_layer: expert shapes (I=%d)", I);
  const size_t need = proj ? mc_moe_decode_proj_workspace_words(I)
                           : mc_moe_decode_workspace_words(I);
  MC_REQUIRE(noalloc || ws_words >= need, "moe_decode_layer: workspace of %zu words < %zu",
             ws_words, need);
  MC_REQUIRE(h && norm_w && h_out && normed && router_w && logits && ids && weights && out &&
                 (noalloc || sync),
             "moe_decode_layer: null pointer");
  MC_REQUIRE(!status_out || mc_aligned(status_out, 4), "moe_decode_layer: status misaligned");
  MC_REQUIRE(router_dtype == MC_DTYPE_BF16 || router_dtype == MC_DTYPE_F32,
             "moe_decode_layer: router dtype %d", router_dtype);
  MC_REQUIRE(route_mode == MC_ROUTE_SOFTMAX_RENORM || route_mode == MC_ROUTE_SIGMOID_BIAS,
             "moe_decode_layer: route mode %d", route_mode);
  const void* a16[] = {h,           norm_w,       h_out,        normed,     router_w,
                       gate->codes, gate->scales, gate->biases, up->codes,  up->scales,
                       up->biases,  down->codes,  down->scales, down->biases,
                       noalloc ? (const void*)h : (const void*)sync};
  for (const void* p : a16)
    MC_REQUIRE(mc_aligned(p, 16), "moe_decode_layer: buffers must be 16-byte aligned");
  MC_REQUIRE(!b || mc_aligned(b, 16), "moe_decode_layer: b must be 16-byte aligned");
  MC_REQUIRE((const void*)h_out != (const void*)h && (const void*)h_out != (const void*)b &&
                 (const void*)normed != (const void*)h && (const void*)normed != (const void*)b,
             "moe_decode_layer: h_out/normed must not alias h or b");
  MC_REQUIRE(!p_out || ((const void*)p_out != (const void*)h && (const void*)p_out != (const void*)out),
             "moe_decode_layer_proj: p_out must not alias h or out");
  const int G = ctx->num_sms;
  // each CTA: <= 16 down rows (4 warps x kDnRows per expert), <= kMaxChunks
  // chunks of gate/up pairs, one router row per expert among the CTAs, and
  // its whole slice of expert rows in shared memory
  const Layout L = make_layout(I, G, proj != nullptr);
  MC_REQUIRE(L.nr_max <= 4 * kDnRows && L.nchunk_max <= kMaxChunks && G >= n_experts,
             "moe_decode_layer: too few SMs (%d)", G);
  MC_REQUIRE((int)L.total + 4096 <= ctx->max_smem_optin,
             "moe_decode_layer: %u B of shared memory per CTA exceeds the device's %d", L.total,
             ctx->max_smem_optin);
  // every check has passed: only now may the built-in scratch be set up
  if (noalloc) {
    size_t words = 0;
    const int rc2 = mc_noalloc_decode_scratch(ctx, &sync, &words);
    if (rc2) return rc2;
    MC_REQUIRE(words >= mc_moe_decode_workspace_words(I), "moe_decode_layer: scratch too small");
  }
  Params P{h, b, norm_w, h_out, normed, router_w, expert_bias, logits, ids, weights, *gate, *up,
           *down, out, sync, eps, route_eps, route_mode, n_experts, I,
           ctx->trace && ctx->trace_len >= kTraceSlots * G ? ctx->trace : nullptr,
           {nullptr, nullptr},
           {0u, 0u},
           ctx->wait_limit_ns ? ctx->wait_limit_ns : kTimeoutNs,
           status_out,
           noalloc ? 1 : 0,
           (ctx->test_flags & MC_TEST_SKIP_LOGIT_PUBLISH) ? 1 : 0,
           proj ? *proj : mc_qweights{},
           p_out};
  for (int r = 0; r < 2; ++r) {
    if (!ctx->pf_ptr[r]) continue;
    // whole 128-byte lines covering the range
    const uintptr_t a = (uintptr_t)ctx->pf_ptr[r] & ~(uintptr_t)127;
    const uintptr_t e = (uintptr_t)ctx->pf_ptr[r] + ctx->pf_bytes[r];
    P.pf[r] = reinterpret_cast<const uint8_t*>(a);
    P.pf_lines[r] = (uint32_t)((e - a + 127) / 128);
    ctx->pf_ptr[r] = nullptr;
    ctx->pf_bytes[r] = 0;
  }
  void* fn = router_dtype == MC_DTYPE_BF16
                 ? (proj ? (void*)moe_decode_fused_kernel<MC_DTYPE_BF16, true>
                         : (void*)moe_decode_fused_kernel<MC_DTYPE_BF16, false>)
                 : (proj ? (void*)moe_decode_fused_kernel<MC_DTYPE_F32, true>
                         : (void*)moe_decode_fused_kernel<MC_DTYPE_F32, false>);
  // the dynamic shared memory limit is raised once per device and kernel
  static std::atomic<int> smem_set[4][64];
  std::atomic<int>& cur =
      smem_set[(router_dtype == MC_DTYPE_BF16 ? 0 : 1) + (proj ? 2 : 0)][ctx->device & 63];
  if (cur.load() < (int)L.total) {
    MC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 ctx->max_smem_optin - 4096));
    cur.store(ctx->max_smem_optin - 4096);
  }
  // The CTAs wait on one another, so all of them must be resident at once:
  // one CTA per SM, grid = SM count. The launch is not cooperative so that it
  // can be a programmatic dependent launch (the next kernel's CTAs start as
  // this one's retire); if another kernel held SMs, the bounded waits would
  // end with an error status instead of a hang.
  int per_sm = 0;
  MC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, L.total));
  MC_REQUIRE(per_sm >= 1, "moe_decode_layer: kernel does not fit one CTA per SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&P, (void*)&L};
  MC_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
  return mc_after_launch("moe_decode_fused_kernel");
}

extern "C" int mc_moe_decode_layer(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                                   const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                                   const void* router_w, int router_dtype,
                                   const float* expert_bias, int route_mode, float* logits,
                                   uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
                                   const mc_qweights* up, const mc_qweights* down, int n_experts,
                                   uint16_t* out, uint32_t* sync, size_t ws_words, float eps,
                                   float route_eps) {
  return mc_decode_layer_impl(ctx, h, b, norm_w, h_out, normed, router_w, router_dtype,
                              expert_bias, route_mode, logits, ids, weights, gate, up, down,
                              n_experts, out, sync, ws_words, eps, route_eps, false, nullptr,
                              nullptr, nullptr);
}

// gemv_quant(proj, h) -> b followed by moe_decode (kernels/lfm.rs:112-149,
// lfm.rs:967-1011) in one launch; see the header.
extern "C" int mc_moe_decode_layer_proj(mc_ctx* ctx, const uint16_t* h, const mc_qweights* proj,
                                        uint16_t* p_out, const uint16_t* norm_w, uint16_t* h_out,
                                        uint16_t* normed, const void* router_w, int router_dtype,
                                        const float* expert_bias, int route_mode, float* logits,
                                        uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
                                        const mc_qweights* up, const mc_qweights* down,
                                        int n_experts, uint16_t* out, uint32_t* sync,
                                        size_t ws_words, float eps, float route_eps) {
  MC_REQUIRE(proj, "moe_decode_layer_proj: null proj");
  return mc_decode_layer_impl(ctx, h, nullptr, norm_w, h_out, normed, router_w, router_dtype,
                              expert_bias, route_mode, logits, ids, weights, gate, up, down,
                              n_experts, out, sync, ws_words, eps, route_eps, false, nullptr, proj,
                              p_out);
}
