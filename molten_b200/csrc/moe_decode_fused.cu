// moe_decode (lfm.rs:967-1011) behind the fused router (lfm.rs:1154-1169) as
// ONE persistent cooperative launch for one token (batch 1): add + RMSNorm +
// router + top-4 (router_addnorm_route), the four experts' gate/up GEMVs with
// SwiGLU (gemv_gather_act) and their down GEMVs with the weighted combine
// (gemv_gather_down_combine4), bit-identical to those three kernels.
//
// One CTA per SM, 16 warps. Timeline of a launch:
//  * every CTA adds h + b and normalises the row (each needs the normed row);
//    warp 0 of CTAs 0..E-1 has prefetched one router row and publishes that
//    expert's logit, epoch-tagged, to the workspace;
//  * warp 0 of every CTA polls the E tagged logits and picks the same top-4;
//  * every thread issues L2 prefetches for its CTA's slice of the 4 experts'
//    down rows, then each warp streams its gate/up row pairs straight from
//    HBM (16-byte non-allocating loads, the next pair's loads issued before
//    the current pair is reduced) and publishes bf16 act values;
//  * after a release/acquire count of the CTAs that published, each CTA loads
//    the act rows and computes its down rows from L2 (4 rows per warp in
//    flight) and the weighted combine.
// No bulk copies and no shared staging of weights: the weight stream is the
// plain load pattern that reaches HBM speed on this part.
//
// Published values are self-validating words carrying the launch's epoch tag
// (logits: tag32 << 32 | f32 bits). The caller's workspace (u32 words, zeroed
// once, then owned by one chain of calls) holds:
//   ws[0]            epoch (advanced by the last CTA to finish)
//   ws[1]            CTAs finished (reset by the last one)
//   ws[2]            sticky error status bits: 1 logits wait gave up,
//                    2 expert id out of range, 8 act wait
//   ws[3]            CTAs that published their act rows (reset by the last
//                    CTA to finish)
//   ws[4]            router warps that published their logit (reset likewise)
//   ws[5..8)         reserved
//   ws[8..136)       64 tagged logits (u64)
//   ws[136..)        act rows as bf16, [slot][row] (2 per word)
// Every wait is bounded by a %globaltimer deadline; waiting lanes back off
// between polls (a few thousand lanes spinning on the same lines slow the
// writers down).
//
// Arithmetic per output is the canonical order of the separate kernels, so
// results are bit-identical to router_addnorm_route + gemv_gather_act +
// gemv_gather_down_combine4 and to the CPU oracle.
#include "gemv_common.cuh"
#include "mc_async.cuh"
#include "route_common.cuh"
#include "rownorm.cuh"

namespace {

constexpr int kThreads = 384;  // 12 warps, 3 per scheduler: up to 168 registers per thread
                               // (the register file is split per scheduler), room for
                               // kPairs row pairs in flight per warp
constexpr int kWarps = kThreads / 32;
constexpr int kPairs = 4;      // gate/up row pairs each warp has in flight
constexpr int kDnRows = 5;     // down rows per warp (12 warps, 3 per expert)
constexpr int H = 2048;
constexpr unsigned long long kTimeoutNs = 200000000ull;  // 200 ms per wait
constexpr int kLogitWord = 8;  // first tagged-logit word in the workspace
constexpr int kActWord = 136;  // first act word in the workspace

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
};

#define TRACE(k) \
  do { if (P.trace && t == 0) P.trace[16 * blockIdx.x + (k)] = mc_globaltimer(); } while (0)

__device__ __forceinline__ void record_error(uint32_t* sync, uint32_t bit) {
  atomicOr(sync + 2, bit);
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// One gate/up row pair of the stacked experts: codes (group `lane`) and the
// raw bf16 scale/bias words, loaded ahead of use.
struct PairLoad {
  QGroup<4> g, u;
  uint16_t gs, gb, us, ub;
  __device__ __forceinline__ void load(const Params& P, size_t row, int lane) {
    g.load(reinterpret_cast<const uint8_t*>(P.gate.codes) + row * (H / 2), lane);
    u.load(reinterpret_cast<const uint8_t*>(P.up.codes) + row * (H / 2), lane);
    gs = __ldg(P.gate.scales + row * (H / 64) + lane);
    gb = __ldg(P.gate.biases + row * (H / 64) + lane);
    us = __ldg(P.up.scales + row * (H / 64) + lane);
    ub = __ldg(P.up.biases + row * (H / 64) + lane);
  }
};

template <int DT>
__global__ void __maxnreg__(168) moe_decode_fused_kernel(const Params P) {
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
  uint32_t* sync = P.sync;
  unsigned long long* logits64 = reinterpret_cast<unsigned long long*>(sync + kLogitWord);
  uint16_t* act = reinterpret_cast<uint16_t*>(sync + kActWord);
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(sync);
  const uint32_t tag32 = epoch == 0xffffffffu ? 1u : epoch + 1u;
  bool ok = true;
  TRACE(0);
  if (t == 0) flag_s = 0;

  // ---- router row prefetch (warp 0 of CTA e < E), then add + RMSNorm (all CTAs)
  const bool router_warp = warp == 0 && cta < P.E;
  RouterRow<DT> rr;
  if (router_warp) rr.load(P.router_w, cta, lane);
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

  // ---- router logit of expert `cta` (warp 0), published epoch-tagged
  if (router_warp) {
    const float z = rr.dot(nrow, lane);
    if (lane == 0) {
      P.logits[cta] = z;
      mc_st_publish_u64(logits64 + cta,
                        ((unsigned long long)tag32 << 32) | (unsigned long long)__float_as_uint(z));
      __threadfence();
      mc_red_release_add(sync + 4, 1u);
    }
  }
  TRACE(2);

  // ---- gate/up activations prescaled once (all warps), meanwhile warp 0
  // gathers the tagged logits
  float2 xs[32];
  const float xg = load_group_x<4, 2>(nbf, lane, xs);
  if (warp == 0) {
    // lane 0 waits (backing off) until all E router warps have published;
    // then lane l reads logits 2l, 2l+1 in one 16-byte load (tags checked)
    const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
    bool got = true;
    if (lane == 0) {
      while (mc_ld_acquire(sync + 4) < (uint32_t)P.E) {
        if (mc_globaltimer() > deadline) {
          got = false;
          break;
        }
        __nanosleep(64);
      }
    }
    got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
    if (got && 2 * lane < P.E) {
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

  const int dn_code = I / 2, Gd = I / 64;
  if (ok) {
    // ---- L2 prefetch of this CTA's down rows (codes, scales, biases) of the
    // 4 experts: contiguous row ranges, one 128-byte line per thread
    const int code_lines = (nr * dn_code + 127) / 128, sb_lines = (nr * Gd * 2 + 127) / 128;
    const int per_e = code_lines + 2 * sb_lines;
    for (int l = t; l < 4 * per_e; l += kThreads) {
      const int r = l / per_e, k = l % per_e;
      const size_t row = (size_t)ids_s[r] * H + i0;
      if (k < code_lines) {
        prefetch_l2(reinterpret_cast<const uint8_t*>(P.down.codes) + row * dn_code + 128 * k);
      } else {
        const int kk = k - code_lines;
        const uint16_t* base = kk < sb_lines ? P.down.scales : P.down.biases;
        prefetch_l2(reinterpret_cast<const uint8_t*>(base + row * Gd) + 128 * (kk % sb_lines));
      }
    }

    // ---- gate/up + SwiGLU: warp w takes pairs w, w+12, w+24, w+36 of this CTA
    // (kPairs at a time), every load issued before the first reduction
    auto pair_row = [&](int q) -> size_t {
      const int slot = (p0 + q) / I;
      return (size_t)ids_s[slot] * I + (p0 + q - slot * I);
    };
    for (int base = 0; base < np; base += kWarps * kPairs) {
      PairLoad pl[kPairs];
#pragma unroll
      for (int k = 0; k < kPairs; ++k) {
        const int q = base + warp + kWarps * k;
        if (q < np) pl[k].load(P, pair_row(q), lane);
      }
#pragma unroll
      for (int k = 0; k < kPairs; ++k) {
        const int q = base + warp + kWarps * k;
        if (q >= np) break;
        float acc_g = 0.0f, acc_u = 0.0f;
        acc_g = __fadd_rn(acc_g, __fmaf_rn(mc_bf16_to_f32(pl[k].gs), pl[k].g.qx(xs),
                                           __fmul_rn(mc_bf16_to_f32(pl[k].gb), xg)));
        acc_u = __fadd_rn(acc_u, __fmaf_rn(mc_bf16_to_f32(pl[k].us), pl[k].u.qx(xs),
                                           __fmul_rn(mc_bf16_to_f32(pl[k].ub), xg)));
        const float gsum = mc_warp_butterfly(acc_g);
        const float usum = mc_warp_butterfly(acc_u);
        if (lane == 0) {
          const float g = mc_round_bf16(gsum);
          const float u = mc_round_bf16(usum);
          const float sl = mc_round_bf16(mc_silu(g));
          act[p0 + q] = mc_f32_to_bf16(__fmul_rn(sl, u));
        }
      }
    }
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
      __nanosleep(32);
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
  TRACE(10);

  // ---- down rows (from L2, 4 rows per warp in flight) + weighted combine
  if (ok && warp < 12) {
    const int r = warp & 3;
    float2 dxs[1][32];
    float dxg[1] = {0.0f};
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
      dxg[0] = prescale_group_x<4>(xv, dxs[0]);
    }
    const int j0 = warp >> 2;  // 0..2: rows j0, j0+3, ... of expert slot r
    const uint8_t* rows[kDnRows];
    const uint16_t* sc[kDnRows];
    const uint16_t* bi[kDnRows];
#pragma unroll
    for (int k = 0; k < kDnRows; ++k) {
      const int j = min(j0 + 3 * k, nr - 1);
      const size_t row = (size_t)ids_s[r] * H + i0 + j;
      rows[k] = reinterpret_cast<const uint8_t*>(P.down.codes) + row * dn_code;
      sc[k] = P.down.scales + row * Gd;
      bi[k] = P.down.biases + row * Gd;
    }
    if (nr > 0) {
      float sum[kDnRows];
      rows_dot<4, 1, kDnRows>(rows, sc, bi, Gd, lane, dxs, dxg, sum);
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < kDnRows; ++k)
          if (j0 + 3 * k < nr) p_s[r][j0 + 3 * k] = mc_round_bf16(sum[k]);
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

  // ---- the last CTA to finish resets the counters and advances the epoch
  TRACE(7);
  if (t == 0) {
    const uint32_t done = atomicAdd(sync + 1, 1u);
    if (done == (uint32_t)G - 1) {
      sync[1] = 0u;
      sync[3] = 0u;
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
  // each CTA: <= 15 down rows (3 warps x kDnRows per expert), <= 12 x kPairs
  // gate/up pairs per pass, one router warp per expert among the CTAs
  MC_REQUIRE((H + G - 1) / G <= 3 * kDnRows && G >= n_experts,
             "moe_decode_layer: too few SMs (%d)", G);
  Params P{h, b, norm_w, h_out, normed, router_w, expert_bias, logits, ids, weights, *gate, *up,
           *down, out, sync, eps, route_eps, route_mode, n_experts, I,
           ctx->trace && ctx->trace_len >= 16 * G ? ctx->trace : nullptr};
  void* fn = router_dtype == MC_DTYPE_BF16 ? (void*)moe_decode_fused_kernel<MC_DTYPE_BF16>
                                           : (void*)moe_decode_fused_kernel<MC_DTYPE_F32>;
  int per_sm = 0;  // every CTA must be resident at once (cross-CTA waits)
  MC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, 0));
  MC_REQUIRE(per_sm >= 1, "moe_decode_layer: kernel does not fit one CTA per SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&P};
  MC_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
  return mc_after_launch("moe_decode_fused_kernel");
}
