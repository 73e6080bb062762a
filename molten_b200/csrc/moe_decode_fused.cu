// One whole MoE decode layer for one token in a single persistent launch:
// residual add + RMSNorm + router + top-4 (router_addnorm_route), the four
// experts' gate/up + SwiGLU (gemv_gather_act) and down + weighted combine
// (gemv_gather_down_combine4) -- moe_decode in lfm.rs:967-1011 after the
// fused router of lfm.rs:1154-1169.
//
// B200 design. One CTA per SM (cooperative launch: all CTAs co-resident).
//  * Every CTA computes the RMSNorm itself; CTAs 0..3 also compute 16 router
//    logits each and publish them.
//  * As soon as a CTA has the 64 logits it runs the (identical) top-4 and all
//    512 threads issue its whole share of the expert weights as 16-byte
//    cp.async copies into shared memory: gate/up row pairs [p0, p1) of the
//    4*I pairs and the four experts' down rows for output rows [i0, i1),
//    ~145 KB per SM, so the layer's 21 MB are in flight at once. Gate/up rows
//    are consumed chunk by chunk as their mbarriers complete.
//  * The down rows are resident by the time a warp has its expert's act
//    vector, which every CTA reads from the other CTAs' published values.
//
// No grid barrier and no fence: published values are self-validating words
// carrying the launch's epoch tag (logits: tag32 << 32 | f32 bits; act:
// tag16 << 16 | bf16 bits), so a consumer polls exactly the words it needs
// until their tags match. The caller's workspace (u32 words, zeroed once,
// then owned by one chain of calls) holds:
//   ws[0]            epoch (advanced by the last CTA to finish)
//   ws[1]            CTAs finished (reset by the last one)
//   ws[2]            sticky error status bits: 1 logits wait gave up,
//                    2 expert id out of range, 4 gate/up copies wait,
//                    8 act wait, 16 down copies wait
//   ws[3]            CTAs that published their act rows (reset by the last
//                    CTA to finish)
//   ws[4..132)       64 tagged logits (u64)
//   ws[132..)        act rows as bf16, [slot][row] (2 per word)
// Every wait is bounded by a %globaltimer deadline; on timeout the CTA
// records the status and leaves only after its own copies have landed.
//
// Arithmetic per output is the canonical order of the separate kernels, so
// results are bit-identical to router_addnorm_route + gemv_gather_act +
// gemv_gather_down_combine4 and to the CPU oracle.
#include "gemv_common.cuh"
#include "mc_async.cuh"
#include "route_common.cuh"
#include "rownorm.cuh"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int H = 2048;
constexpr int kChunk = 16;                              // gate/up row pairs per mbarrier
constexpr unsigned long long kTimeoutNs = 200000000ull;  // 200 ms per wait

constexpr int GU_CODE = H / 2;       // 1024 B of codes per gate/up row
constexpr int GU_SB = (H / 64) * 2;  // 64 B of scales (or biases) per row
constexpr int GU_PIECES = (2 * GU_CODE + 4 * GU_SB) / 16;  // 16-byte copies per row pair
constexpr int kActWord = 132;  // first act word in the workspace

struct Layout {
  int pmax, rmax, nchunk;
  int off_gc, off_uc, off_gs, off_gb, off_us, off_ub;  // gate/up staging
  int off_dc, off_ds, off_db;                          // down staging
  int off_bar, total;
};

__host__ __device__ inline Layout make_layout(int pmax, int rmax, int I) {
  Layout L;
  L.pmax = pmax;
  L.rmax = rmax;
  L.nchunk = (pmax + kChunk - 1) / kChunk;
  const int dn_code = I / 2, dn_sb = (I / 64) * 2;
  int o = 0;
  L.off_gc = o; o += pmax * GU_CODE;
  L.off_uc = o; o += pmax * GU_CODE;
  L.off_gs = o; o += pmax * GU_SB;
  L.off_gb = o; o += pmax * GU_SB;
  L.off_us = o; o += pmax * GU_SB;
  L.off_ub = o; o += pmax * GU_SB;
  L.off_dc = o; o += 4 * rmax * dn_code;
  L.off_ds = o; o += 4 * rmax * dn_sb;
  L.off_db = o; o += 4 * rmax * dn_sb;
  o = (o + 15) & ~15;
  L.off_bar = o; o += (L.nchunk + 5) * 8;  // code chunks, scales/biases, 4 down slots
  L.total = o;
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
  int mode, E, I, n_router_ctas;
  unsigned long long* trace;
};

#define TRACE(k) \
  do { if (P.trace && t == 0) P.trace[16 * blockIdx.x + (k)] = mc_globaltimer(); } while (0)

__device__ __forceinline__ void record_error(uint32_t* sync, uint32_t bit) {
  atomicOr(sync + 2, bit);
}

__device__ __forceinline__ bool mbar_wait_deadline(uint64_t* bar, unsigned long long deadline) {
  while (!mc_mbar_test_sleep(bar, 0, 20000u))
    if (mc_globaltimer() > deadline) return false;
  return true;
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_fused_kernel(const Params P, Layout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(16) float nrow[H];
  __shared__ __align__(16) uint16_t nbf[H];
  __shared__ float red[8];
  __shared__ float zs[64];
  __shared__ uint32_t ids_s[4];
  __shared__ uint16_t wts_s[4];
  __shared__ float p_s[4][32];
  __shared__ __align__(16) uint16_t act_s[4 * 2048];  // 16-byte chunks XOR-swizzled per group
  __shared__ uint32_t flag_s;

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int I = P.I;
  const int npairs = 4 * I;
  const int p0 = (int)(((long)cta * npairs) / G), p1 = (int)(((long)(cta + 1) * npairs) / G);
  const int i0 = (int)(((long)cta * H) / G), i1 = (int)(((long)(cta + 1) * H) / G);
  const int np = p1 - p0, nr = i1 - i0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  uint32_t* sync = P.sync;
  unsigned long long* logits64 = reinterpret_cast<unsigned long long*>(sync + 4);
  uint16_t* act = reinterpret_cast<uint16_t*>(sync + kActWord);
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(sync);
  const uint32_t tag32 = epoch == 0xffffffffu ? 1u : epoch + 1u;
  const uint32_t tag16 = (tag32 % 65535u) + 1u;
  bool ok = true;
  TRACE(0);

  if (t == 0) {
    for (int c = 0; c < L.nchunk + 5; ++c) mc_mbar_init(bars + c, 1);
    mc_fence_barrier_init();
    flag_s = 0;
  }

  // ---- router row prefetch (router CTAs), then add + RMSNorm (all CTAs)
  const int e_mine = cta * kWarps + warp;
  const bool router_cta = cta < P.n_router_ctas;
  RouterRow<DT> rr;
  if (router_cta && e_mine < P.E) rr.load(P.router_w, e_mine, lane);
  float hp[8];
  if (t < 256) {
    float acc = 0.0f;
    const uint4 hv = __ldg(reinterpret_cast<const uint4*>(P.h) + t);
    uint4 bv = make_uint4(0, 0, 0, 0);
    if (P.badd) bv = __ldg(reinterpret_cast<const uint4*>(P.badd) + t);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float hf = mc_bf16_to_f32((uint16_t)(hw[i >> 1] >> (16 * (i & 1))));
      float v = hf;
      if (P.badd) v = __fadd_rn(hf, mc_bf16_to_f32((uint16_t)(bw[i >> 1] >> (16 * (i & 1)))));
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
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(P.norm_w) + t);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    float n[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float wf = mc_bf16_to_f32((uint16_t)(ww[i >> 1] >> (16 * (i & 1))));
      n[i] = mc_round_bf16(__fmul_rn(__fmul_rn(hp[i], inv), wf));
      nrow[8 * t + i] = n[i];
    }
    const uint4 nb = pack8_bf16(n);
    reinterpret_cast<uint4*>(nbf)[t] = nb;
    if (cta == 0) {
      reinterpret_cast<uint4*>(P.h_out)[t] = pack8_bf16(hp);
      reinterpret_cast<uint4*>(P.normed)[t] = nb;
    }
  }
  __syncthreads();
  TRACE(1);

  // ---- router logits: CTA c < n_router_ctas publishes experts 16c .. 16c+15
  if (router_cta && e_mine < P.E) {
    const float z = rr.dot(nrow, lane);
    if (lane == 0) {
      P.logits[e_mine] = z;
      mc_st_publish_u64(logits64 + e_mine,
                        ((unsigned long long)tag32 << 32) | (unsigned long long)__float_as_uint(z));
    }
  }
  TRACE(2);

  // ---- warp 0 of every CTA: gather the 64 tagged logits, identical top-4
  if (warp == 0) {
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    bool got = true;
    for (int i = lane; i < P.E; i += 32) {
      unsigned long long v;
      while (((v = mc_ld_poll_u64(logits64 + i)) >> 32) != tag32) {
        if (mc_globaltimer() > deadline) {
          got = false;
          break;
        }
        __nanosleep(128);
      }
      zs[i] = __uint_as_float((uint32_t)v);
    }
    got = __all_sync(0xffffffffu, got);
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
    }
  }
  __syncthreads();
  TRACE(3);
  if (flag_s) ok = false;

  // ---- one thread issues this CTA's expert rows as a few bulk (TMA) copies:
  // the small scale/bias arrays first, then the codes chunk by chunk, then
  // the down rows; the other warps start on chunks as they land.
  const int dn_code = I / 2, dn_sb = (I / 64) * 2;
  uint64_t* bar_sb = bars + L.nchunk;
  uint64_t* bar_dn = bars + L.nchunk + 1;
  // at most two expert segments: local pairs [0, qs) and [qs, np)
  const int slot0 = p0 / I;
  const int qs = min(np, (slot0 + 1) * I - p0);
  bool issued = false;  // thread 0 only
  if (ok && t == 0) {
    issued = true;
    const uint64_t pol = mc_policy_evict_normal();
    for (int c = 0; c < L.nchunk; ++c) {
      if (c == 1) {
        // scales/biases right after the first code chunk
        mc_mbar_expect_tx(bar_sb, (uint32_t)np * (4 * GU_SB));
        for (int sgi = 0; sgi < 2; ++sgi) {
          const int qa = sgi == 0 ? 0 : qs, qb = sgi == 0 ? qs : np;
          if (qa >= qb) continue;
          const int slot = (p0 + qa) / I;
          const size_t row = (size_t)ids_s[slot] * I + (p0 + qa - slot * I);
          const uint32_t n = (uint32_t)(qb - qa) * GU_SB;
          mc_bulk_g2s(smem + L.off_gs + qa * GU_SB, P.gate.scales + row * (GU_SB / 2), n, bar_sb, pol);
          mc_bulk_g2s(smem + L.off_gb + qa * GU_SB, P.gate.biases + row * (GU_SB / 2), n, bar_sb, pol);
          mc_bulk_g2s(smem + L.off_us + qa * GU_SB, P.up.scales + row * (GU_SB / 2), n, bar_sb, pol);
          mc_bulk_g2s(smem + L.off_ub + qa * GU_SB, P.up.biases + row * (GU_SB / 2), n, bar_sb, pol);
        }
      }
      const int q0 = c * kChunk, q1 = min(np, q0 + kChunk);
      if (q0 >= q1) {
        mc_mbar_arrive(bars + c);
        continue;
      }
      mc_mbar_expect_tx(bars + c, (uint32_t)(q1 - q0) * (2 * GU_CODE));
      for (int sgi = 0; sgi < 2; ++sgi) {
        const int qa = max(q0, sgi == 0 ? 0 : qs), qb = min(q1, sgi == 0 ? qs : np);
        if (qa >= qb) continue;
        const int slot = (p0 + qa) / I;
        const size_t row = (size_t)ids_s[slot] * I + (p0 + qa - slot * I);
        const uint32_t n = (uint32_t)(qb - qa) * GU_CODE;
        mc_bulk_g2s(smem + L.off_gc + qa * GU_CODE,
                    reinterpret_cast<const uint8_t*>(P.gate.codes) + row * GU_CODE, n, bars + c, pol);
        mc_bulk_g2s(smem + L.off_uc + qa * GU_CODE,
                    reinterpret_cast<const uint8_t*>(P.up.codes) + row * GU_CODE, n, bars + c, pol);
      }
    }
    if (L.nchunk < 2) {
      mc_mbar_expect_tx(bar_sb, (uint32_t)np * (4 * GU_SB));
      for (int sgi = 0; sgi < 2; ++sgi) {
        const int qa = sgi == 0 ? 0 : qs, qb = sgi == 0 ? qs : np;
        if (qa >= qb) continue;
        const int slot = (p0 + qa) / I;
        const size_t row = (size_t)ids_s[slot] * I + (p0 + qa - slot * I);
        const uint32_t n = (uint32_t)(qb - qa) * GU_SB;
        mc_bulk_g2s(smem + L.off_gs + qa * GU_SB, P.gate.scales + row * (GU_SB / 2), n, bar_sb, pol);
        mc_bulk_g2s(smem + L.off_gb + qa * GU_SB, P.gate.biases + row * (GU_SB / 2), n, bar_sb, pol);
        mc_bulk_g2s(smem + L.off_us + qa * GU_SB, P.up.scales + row * (GU_SB / 2), n, bar_sb, pol);
        mc_bulk_g2s(smem + L.off_ub + qa * GU_SB, P.up.biases + row * (GU_SB / 2), n, bar_sb, pol);
      }
    }
    for (int r = 0; r < 4; ++r) {
      if (nr == 0) {
        mc_mbar_arrive(bar_dn + r);
        continue;
      }
      mc_mbar_expect_tx(bar_dn + r, (uint32_t)nr * (dn_code + 2 * dn_sb));
      const size_t row = (size_t)ids_s[r] * H + i0;
      mc_bulk_g2s(smem + L.off_dc + r * L.rmax * dn_code,
                  reinterpret_cast<const uint8_t*>(P.down.codes) + row * dn_code, nr * dn_code,
                  bar_dn + r, pol);
      mc_bulk_g2s(smem + L.off_ds + r * L.rmax * dn_sb, P.down.scales + row * (dn_sb / 2),
                  nr * dn_sb, bar_dn + r, pol);
      mc_bulk_g2s(smem + L.off_db + r * L.rmax * dn_sb, P.down.biases + row * (dn_sb / 2),
                  nr * dn_sb, bar_dn + r, pol);
    }
  }

  TRACE(13);
  // ---- gate/up + SwiGLU on the staged rows; act published to the workspace
  if (ok) {
    float2 xs[32];
    const float xg = load_group_x<4, 2>(nbf, lane, xs);
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    bool ready = np == 0 || mbar_wait_deadline(bar_sb, deadline);
    for (int q = warp; q < np && ready; q += kWarps) {
      if (!mbar_wait_deadline(bars + q / kChunk, deadline)) {
        ready = false;
        break;
      }
      if (q == 0) TRACE(8);
      if (q + kWarps >= np) TRACE(9);
      const uint8_t* rows[2] = {smem + L.off_gc + q * GU_CODE, smem + L.off_uc + q * GU_CODE};
      const uint16_t* sc[2] = {reinterpret_cast<const uint16_t*>(smem + L.off_gs + q * GU_SB),
                               reinterpret_cast<const uint16_t*>(smem + L.off_us + q * GU_SB)};
      const uint16_t* bi[2] = {reinterpret_cast<const uint16_t*>(smem + L.off_gb + q * GU_SB),
                               reinterpret_cast<const uint16_t*>(smem + L.off_ub + q * GU_SB)};
      float sum[2];
      smem_rows_dot_q4<2>(rows, sc, bi, 32, lane, xs, xg, sum);
      if (lane == 0) {
        const float g = mc_round_bf16(sum[0]);
        const float u = mc_round_bf16(sum[1]);
        const float sl = mc_round_bf16(mc_silu(g));
        act[p0 + q] = mc_f32_to_bf16(__fmul_rn(sl, u));
      }
    }
    if (!ready && lane == 0) record_error(sync, 4u);
  }
  __syncthreads();
  TRACE(4);

  // ---- act published by every CTA (release/acquire counter, one poller)
  if (t == 0) {
    __threadfence();
    mc_red_release_add(sync + 3, 1u);
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    while (mc_ld_acquire(sync + 3) < (uint32_t)G) {
      if (mc_globaltimer() > deadline) {
        record_error(sync, 8u);
        flag_s = 1;
        break;
      }
    }
  }
  __syncthreads();
  TRACE(5);
  if (flag_s) ok = false;

  // ---- stage the act rows once per CTA (L2 -> shared, swizzled so the
  // per-lane group reads below are bank-conflict free)
  if (ok) {
    const int nchunk16 = (4 * I) / 8;  // 16-byte chunks of bf16 act
    for (int c = t; c < nchunk16; c += kThreads) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(act) + c);
      const int g = c >> 3;            // 64-value group (across slots)
      reinterpret_cast<uint4*>(act_s)[(g << 3) | ((c & 7) ^ (g & 7))] = v;
    }
  }
  __syncthreads();

  // ---- down rows + weighted combine
  if (ok) {
    const int r = warp & 3;
    const int Gd = I / 64;
    float2 xs[32];
    float xg = 0.0f;
    if (lane < Gd) {
      const int g = r * Gd + lane;
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
      xg = prescale_group_x<4>(xv, xs);
    }
    __syncwarp();
    asm volatile("" ::: "memory");
    TRACE(10);
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    const bool dn_ok = mbar_wait_deadline(bar_dn + r, deadline);
    TRACE(11);
    if (!dn_ok) {
      if (lane == 0) record_error(sync, 16u);
    } else {
      const int j0 = warp >> 2;
      const uint8_t* rows[4];
      const uint16_t* sc[4];
      const uint16_t* bi[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = min(j0 + 4 * k, nr - 1);
        rows[k] = smem + L.off_dc + (r * L.rmax + j) * dn_code;
        sc[k] = reinterpret_cast<const uint16_t*>(smem + L.off_ds + (r * L.rmax + j) * dn_sb);
        bi[k] = reinterpret_cast<const uint16_t*>(smem + L.off_db + (r * L.rmax + j) * dn_sb);
      }
      float sum[4];
      smem_rows_dot_q4<4>(rows, sc, bi, Gd, lane, xs, xg, sum);
      __syncwarp();
      asm volatile("" ::"f"(sum[0]), "f"(sum[1]), "f"(sum[2]), "f"(sum[3]) : "memory");
      TRACE(12);
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (j0 + 4 * k < nr) p_s[r][j0 + 4 * k] = mc_round_bf16(sum[k]);
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

  // ---- leave only after this CTA's bulk copies landed (immediate on the
  // normal path); the last CTA resets the counters and advances the epoch
  if (issued) {
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    for (int c = 0; c < L.nchunk + 5; ++c)
      if (!mbar_wait_deadline(bars + c, deadline)) record_error(sync, 16u);
  }
  TRACE(7);
  if (t == 0) {
    const uint32_t done = atomicAdd(sync + 1, 1u);
    if (done == (uint32_t)G - 1) {
      sync[1] = 0u;
      sync[3] = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(sync) = tag32;
    }
  }
}

}  // namespace

extern "C" size_t mc_moe_decode_workspace_words(int moe_inter) {
  return (size_t)kActWord + 4 * (size_t)(moe_inter > 0 ? moe_inter : 0);
}

extern "C" int mc_moe_decode_layer(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                                   const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                                   const void* router_w, int router_dtype,
                                   const float* expert_bias, int route_mode, float* logits,
                                   uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
                                   const mc_qweights* up, const mc_qweights* down, int n_experts,
                                   uint16_t* out, uint32_t* sync, size_t ws_words, float eps,
                                   float route_eps) {
  MC_REQUIRE(ctx, "moe_decode_layer: null context");
  int rc;
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
  // a down row's scales (I/64 bf16) are one bulk copy: 16-byte size and start
  MC_REQUIRE(I % 512 == 0, "moe_decode_layer: expert width %d must be a multiple of 512", I);
  MC_REQUIRE(ws_words >= mc_moe_decode_workspace_words(I),
             "moe_decode_layer: workspace of %zu words < %zu", ws_words,
             mc_moe_decode_workspace_words(I));
  MC_REQUIRE(h && norm_w && h_out && normed && router_w && logits && ids && weights && out && sync,
             "moe_decode_layer: null pointer");
  MC_REQUIRE(router_dtype == MC_DTYPE_BF16 || router_dtype == MC_DTYPE_F32,
             "moe_decode_layer: router dtype %d", router_dtype);
  MC_REQUIRE(route_mode == MC_ROUTE_SOFTMAX_RENORM || route_mode == MC_ROUTE_SIGMOID_BIAS,
             "moe_decode_layer: route mode %d", route_mode);
  const void* a16[] = {h,            norm_w,       h_out,      normed,     router_w,
                       gate->scales, gate->biases, up->scales, up->biases, down->scales,
                       down->biases, sync};
  for (const void* p : a16)
    MC_REQUIRE(mc_aligned(p, 16), "moe_decode_layer: buffers must be 16-byte aligned");
  MC_REQUIRE(!b || mc_aligned(b, 16), "moe_decode_layer: b must be 16-byte aligned");
  MC_REQUIRE((const void*)h_out != (const void*)h && (const void*)h_out != (const void*)b &&
                 (const void*)normed != (const void*)h && (const void*)normed != (const void*)b,
             "moe_decode_layer: h_out/normed must not alias h or b");
  const int G = ctx->num_sms;
  const int pmax = (4 * I + G - 1) / G + 1, rmax = (H + G - 1) / G + 1;
  MC_REQUIRE(rmax <= 32 && G >= (n_experts + kWarps - 1) / kWarps,
             "moe_decode_layer: too few SMs (%d)", G);
  const Layout L = make_layout(pmax, rmax, I);
  MC_REQUIRE(L.total + 16 * 1024 <= ctx->max_smem_optin,
             "moe_decode_layer: %d B of staging exceeds shared memory", L.total);
  Params P{h, b, norm_w, h_out, normed, router_w, expert_bias, logits, ids, weights, *gate, *up,
           *down, out, sync, eps, route_eps, route_mode, n_experts, I,
           (n_experts + kWarps - 1) / kWarps,
           ctx->trace && ctx->trace_len >= 16 * G ? ctx->trace : nullptr};
  void* fn = router_dtype == MC_DTYPE_BF16 ? (void*)moe_decode_fused_kernel<MC_DTYPE_BF16>
                                           : (void*)moe_decode_fused_kernel<MC_DTYPE_F32>;
  MC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&P, (void*)&L};
  MC_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
  return mc_after_launch("moe_decode_fused_kernel");
}
