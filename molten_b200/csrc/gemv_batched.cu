// Batched decode GEMV for tall matrices at batch >= 2 (the Q6 LM head +
// argmax of a batched decode step, tall Q4 projections): gemv_quant /
// gemv_head_argmax (kernels/lfm.rs:112-149, 826-848) when several tokens
// share one weight pass.
//
// gemv_kernel gives every token its own pass over the weights, so at batch B
// the codes are read and decoded B times. Here a warp owns 32 rows, lane l
// row l, and up to T tokens: each 64-code group of the lane's row is decoded
// once (mask + OR 2^23, subtract 2^23) and its fma chains then run once per
// token against that token's pre-scaled activations, which all CTAs' lanes
// read from shared memory as broadcasts.
//
// Results are bit-identical to gemv_kernel / gemv_ring_kernel and to the
// oracle: per (row, token) the group dot, the term fma(s, qx, b * xg) and the
// lane value 0 + term are computed with the same operations in the same
// order, and the 32-lane xor butterfly of the canonical order (levels 16, 8,
// 4, 2, 1) is replayed inside the lane by visiting the groups in 5-bit
// bit-reversed order: the pairs a butterfly level adds are the pairs this
// nested loop adds at the same depth (float addition commutes, so which of
// the two is "own" does not matter). Groups at or past K/64 contribute +0,
// as the idle lanes of the butterfly do.
//
// Short matrices split K over up to 8 warps per row block (each one subtree
// of the butterfly, the subtrees then added in its order) so that a 2048-row
// projection still fills the SMs. K <= 2048 (one group per lane in the
// canonical order); larger K and unaligned operands stay on gemv_kernel.
#include <atomic>

#include "gemv_common.cuh"

namespace {

constexpr int kWarpsB = 8;
constexpr int kThreadsB = kWarpsB * 32;
constexpr int kMaxG = 32;

// Per token: 32 groups x 32 pre-scaled activation pairs, then 32 group sums.
template <int T>
struct BatchedShape {
  static constexpr uint32_t kPairs = kMaxG * 32 * 8;
  static constexpr uint32_t kSmem = T * (kPairs + kMaxG * 4);
};

// Pair m of group g of token t sits at slot m ^ 2*(g & 15) of the group's 32
// (bit 0 of m kept, so pairs 2p, 2p+1 stay adjacent for one 16-byte load):
// the prescale pass writes one group per lane, and the plain layout would put
// all 32 lanes' stores in one bank.
__device__ __forceinline__ int pair_slot(int g, int m) { return m ^ ((g & 15) << 1); }

// One group's codes of the lane's row.
template <int BITS>
struct RawGroup {
  uint4 v[BITS == 6 ? 3 : 2];
  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + (BITS == 6 ? 48 : 32) * g;
    v[0] = mc_ldg_stream(p);
    v[1] = mc_ldg_stream(p + 16);
    if (BITS == 6) v[2] = mc_ldg_stream(p + 32);
  }
};

// Decoded codes of one group: q[i] = (code_a * 2^ea, code_b * 2^eb), the
// exact values the f32x2 add of q4_wordpair_fma / q6_packet_fma produces,
// in the order those functions feed them to their fma chains.
//   Q4: i = 8p + j: word pair p (quarter p), step j (.x word 2p, .y word 2p+1)
//   Q6: i = 2m (codes 4m, 4m+1) and 2m+1 (codes 4m+2, 4m+3) of packet m
__device__ __forceinline__ uint64_t magic_pair(uint32_t lo, uint32_t hi) {
  const unsigned long long NEG = 0xCB000000CB000000ull;  // (-2^23, -2^23)
  unsigned long long q;
  asm("mov.b64 %0, {%1, %2};" : "=l"(q) : "r"(lo), "r"(hi));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(q), "l"(NEG));
  return q;
}

__device__ __forceinline__ void decode_q4(const RawGroup<4>& r, uint64_t* q) {
  const uint32_t W[8] = {r.v[0].x, r.v[0].y, r.v[0].z, r.v[0].w,
                         r.v[1].x, r.v[1].y, r.v[1].z, r.v[1].w};
  const uint32_t MAG = MC_MAGIC;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t wa = W[2 * p], wb = W[2 * p + 1];
    const uint32_t sa = wa >> 12, sb = wb >> 12;
#define MC_Q4_DEC(J, A, B, M)                                                            \
  {                                                                                      \
    uint32_t lo, hi;                                                                     \
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(lo) : "r"(A), "n"(M), "r"(MAG));         \
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(hi) : "r"(B), "n"(M), "r"(MAG));         \
    q[8 * p + (J)] = magic_pair(lo, hi);                                                 \
  }
    MC_Q4_DEC(0, wa, wb, 0xF)
    MC_Q4_DEC(1, wa, wb, 0xF0)
    MC_Q4_DEC(2, wa, wb, 0xF00)
    MC_Q4_DEC(3, wa, wb, 0xF000)
    MC_Q4_DEC(4, wa, wb, 0xF0000)
    MC_Q4_DEC(5, sa, sb, 0xF00)
    MC_Q4_DEC(6, sa, sb, 0xF000)
    MC_Q4_DEC(7, sa, sb, 0xF0000)
#undef MC_Q4_DEC
  }
}

template <int OFF>
__device__ __forceinline__ void decode_q6_packet(uint32_t lo, uint32_t hi, uint64_t& q01,
                                                 uint64_t& q23) {
  const uint32_t MAG = MC_MAGIC;
  constexpr uint32_t selP = (OFF) | ((OFF + 1) << 4) | ((OFF + 2) << 8) | ((OFF + 3) << 12);
  constexpr uint32_t selQ = (OFF + 1) | ((OFF + 2) << 4) | ((OFF + 3) << 8) | ((OFF + 3) << 12);
  uint32_t P, Q, c0, c1, c2, c3;
  if (OFF == 0) {
    P = lo;
  } else {
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(P) : "r"(lo), "r"(hi), "n"(selP));
  }
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(Q) : "r"(lo), "r"(hi), "n"(selQ));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(c0) : "r"(P), "n"(0x3F), "r"(MAG));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(c1) : "r"(P), "n"(0xFC0), "r"(MAG));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(c2) : "r"(P), "n"(0x3F000), "r"(MAG));
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(c3) : "r"(Q), "n"(0xFC00), "r"(MAG));
  q01 = magic_pair(c0, c1);
  q23 = magic_pair(c2, c3);
}

__device__ __forceinline__ void decode_q6(const RawGroup<6>& r, uint64_t* q) {
  const uint32_t W[12] = {r.v[0].x, r.v[0].y, r.v[0].z, r.v[0].w, r.v[1].x, r.v[1].y,
                          r.v[1].z, r.v[1].w, r.v[2].x, r.v[2].y, r.v[2].z, r.v[2].w};
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int base = 3 * m;
    const int wi = base >> 2;
    const int wj = wi + 1 < 12 ? wi + 1 : 11;
    switch (base & 3) {
      case 0: decode_q6_packet<0>(W[wi], W[wj], q[2 * m], q[2 * m + 1]); break;
      case 1: decode_q6_packet<1>(W[wi], W[wj], q[2 * m], q[2 * m + 1]); break;
      case 2: decode_q6_packet<2>(W[wi], W[wj], q[2 * m], q[2 * m + 1]); break;
      default: decode_q6_packet<3>(W[wi], W[wj], q[2 * m], q[2 * m + 1]); break;
    }
  }
}

__device__ __forceinline__ void fma2(unsigned long long& acc, uint64_t q, float2 x) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(acc)
      : "l"(q), "l"(*reinterpret_cast<const unsigned long long*>(&x)));
}

// qx of one token: the four quarter chains of the canonical order over the
// decoded group (xp = the token's 32 pre-scaled pairs of this group, slots
// permuted by pair_slot), then (c0 + c1) + (c2 + c3) per parity, even + odd.
template <int BITS>
__device__ __forceinline__ float token_qx(const uint64_t* q, const float2* xp, int g) {
  unsigned long long c[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float4 x2 = *reinterpret_cast<const float4*>(xp + pair_slot(g, i));
    // Q4: pairs i, i+1 belong to quarter i / 8; Q6: packet i / 2, quarter i / 8
    fma2(c[i >> 3], q[i], make_float2(x2.x, x2.y));
    fma2(c[i >> 3], q[i + 1], make_float2(x2.z, x2.w));
  }
  return quarters_qx(reinterpret_cast<const float2*>(c));
}

// Rows [32*rb, 32*rb + 32) x tokens [t0, t0 + nt): MODE 0 stores
// y[token][row] = bf16(row . x[token]); MODE 1 folds the argmax of the
// bf16-rounded values into keys[token] (zero on entry).
template <int BITS, int MODE, int T>
__global__ void __launch_bounds__(kThreadsB, 1)
gemv_batched_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                    const uint16_t* __restrict__ biases, const uint16_t* __restrict__ x,
                    uint16_t* __restrict__ y, unsigned long long* __restrict__ keys, int N, int K,
                    int batch, int ks_log2) {
  extern __shared__ __align__(16) uint8_t smb[];
  float2* xs_s = reinterpret_cast<float2*>(smb);
  float* xg_s = reinterpret_cast<float*>(smb + T * BatchedShape<T>::kPairs);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = K / 64;
  const int t0 = blockIdx.y * T;
  const int nt = min(T, batch - t0);
  const size_t row_bytes = (size_t)K * BITS / 8;

  // the first row block's codes into L2 before the wait (weights are never
  // written by the previous kernel)
  {
    const int row = (blockIdx.x * kWarpsB + warp) * 32 + lane;
    if (row < N) {
      const uint8_t* r = codes + (size_t)row * row_bytes;
      for (size_t off = 0; off < row_bytes; off += 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(r + off));
    }
  }
  mc_pdl_launch_dependents();
  mc_pdl_wait();

  // pre-scaled activations of the CTA's tokens: one (token, group) per thread
  for (int i = threadIdx.x; i < T * kMaxG; i += kThreadsB) {
    const int tt = i / kMaxG, g = i % kMaxG;
    float2 tmp[32];
    float xg = 0.0f;
    if (tt < nt && g < G) {
      xg = load_group_x<BITS>(x + (size_t)(t0 + tt) * K, g, tmp);
    } else {
#pragma unroll
      for (int m = 0; m < 32; ++m) tmp[m] = make_float2(0.0f, 0.0f);
    }
    float2* dst = xs_s + (size_t)i * 32;
#pragma unroll
    for (int m = 0; m < 32; ++m) dst[pair_slot(g, m)] = tmp[m];
    xg_s[i] = xg;
  }
  __syncthreads();

  float best_v[T];
  uint32_t best_i[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    best_v[t] = -INFINITY;
    best_i[t] = 0;
  }

  // K split: KS = 2^ks_log2 warps share a row block, part p taking the
  // groups whose visit index s has s >> (5 - ks_log2) == p -- one subtree of
  // the butterfly -- and the parts are then added in the butterfly's order
  // (balanced tree over p). A CTA covers kWarpsB / KS row blocks per pass;
  // every warp of the CTA runs the same number of passes.
  const int KS = 1 << ks_log2;
  const int part = warp & (KS - 1);
  const int rbl = warp >> ks_log2;
  const int rb_per_cta = kWarpsB >> ks_log2;
  const int s_lo = part << (5 - ks_log2), s_hi = (part + 1) << (5 - ks_log2);
  // loop bounds of the visit digits i1..i4 (i0 always runs 0..1)
  int lo[5], hi[5];
#pragma unroll
  for (int d = 1; d < 5; ++d) {
    const bool fixed = d >= 5 - ks_log2;
    lo[d] = fixed ? (s_lo >> d) & 1 : 0;
    hi[d] = fixed ? lo[d] + 1 : 2;
  }
  __shared__ float part_s[kWarpsB][T][32];

  const int nrb = (N + 31) / 32;
  for (int base = blockIdx.x * rb_per_cta; base < nrb; base += gridDim.x * rb_per_cta) {
    const int rb = base + rbl;
    const int row = rb * 32 + lane;
    const bool on = row < N;
    const int rr = on ? row : N - 1;
    const uint8_t* crow = codes + (size_t)rr * row_bytes;
    const uint16_t* srow = scales + (size_t)rr * G;
    const uint16_t* brow = biases + (size_t)rr * G;

    // group visit s = i0 + 2 i1 + 4 i2 + 8 i3 + 16 i4 is group bitrev5(s);
    // the next group's codes and scale / bias load while this one computes
    RawGroup<BITS> cur, nxt;
    uint16_t s_cur = 0, b_cur = 0, s_nxt = 0, b_nxt = 0;
    {
      const int g0 = (int)(__brev((unsigned)s_lo) >> 27);
      if (g0 < G) {
        cur.load(crow, g0);
        s_cur = __ldg(srow + g0);
        b_cur = __ldg(brow + g0);
      }
    }
    float l1[T], l2[T], l3[T], l4[T], l5[T];
#pragma unroll 1
    for (int i4 = lo[4]; i4 < hi[4]; ++i4) {
#pragma unroll 1
      for (int i3 = lo[3]; i3 < hi[3]; ++i3) {
#pragma unroll 1
        for (int i2 = lo[2]; i2 < hi[2]; ++i2) {
#pragma unroll 1
          for (int i1 = lo[1]; i1 < hi[1]; ++i1) {
#pragma unroll
            for (int i0 = 0; i0 < 2; ++i0) {
              const int s = i0 + 2 * i1 + 4 * i2 + 8 * i3 + 16 * i4;
              const int g = 16 * i0 + 8 * i1 + 4 * i2 + 2 * i3 + i4;
              const int gn = (int)(__brev((unsigned)(s + 1)) >> 27);
              if (s + 1 < s_hi && gn < G) {
                nxt.load(crow, gn);
                s_nxt = __ldg(srow + gn);
                b_nxt = __ldg(brow + gn);
              }
              float term[T];
              if (g < G) {
                uint64_t q[32];
                if (BITS == 6)
                  decode_q6(reinterpret_cast<const RawGroup<6>&>(cur), q);
                else
                  decode_q4(reinterpret_cast<const RawGroup<4>&>(cur), q);
                const float sc = mc_bf16_to_f32(s_cur), bi = mc_bf16_to_f32(b_cur);
#pragma unroll
                for (int t = 0; t < T; ++t) {
                  const int i = t * kMaxG + g;
                  const float qx = token_qx<BITS>(q, xs_s + (size_t)i * 32, g);
                  term[t] = __fadd_rn(0.0f, __fmaf_rn(sc, qx, __fmul_rn(bi, xg_s[i])));
                }
              } else {
#pragma unroll
                for (int t = 0; t < T; ++t) term[t] = 0.0f;
              }
#pragma unroll
              for (int t = 0; t < T; ++t) l1[t] = i0 ? __fadd_rn(l1[t], term[t]) : term[t];
              cur = nxt;
              s_cur = s_nxt;
              b_cur = b_nxt;
            }
#pragma unroll
            for (int t = 0; t < T; ++t) l2[t] = i1 != lo[1] ? __fadd_rn(l2[t], l1[t]) : l1[t];
          }
#pragma unroll
          for (int t = 0; t < T; ++t) l3[t] = i2 != lo[2] ? __fadd_rn(l3[t], l2[t]) : l2[t];
        }
#pragma unroll
        for (int t = 0; t < T; ++t) l4[t] = i3 != lo[3] ? __fadd_rn(l4[t], l3[t]) : l3[t];
      }
#pragma unroll
      for (int t = 0; t < T; ++t) l5[t] = i4 != lo[4] ? __fadd_rn(l5[t], l4[t]) : l4[t];
    }

    if (KS > 1) {
      // the parts' subtree sums, added level by level (p, p ^ 1), (.., .. ^ 2), ..
#pragma unroll
      for (int t = 0; t < T; ++t) part_s[warp][t][lane] = l5[t];
      __syncthreads();
      if (part == 0) {
#pragma unroll
        for (int t = 0; t < T; ++t) {
          float v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] = q < KS ? part_s[warp + q][t][lane] : 0.0f;
#pragma unroll
          for (int w = 8; w > 1; w >>= 1)
            if (w <= KS) {
#pragma unroll
              for (int q = 0; q < w / 2; ++q) v[q] = __fadd_rn(v[2 * q], v[2 * q + 1]);
            }
          l5[t] = v[0];
        }
      }
      __syncthreads();
    }
    if (part == 0) {
      if (MODE == 0) {
#pragma unroll
        for (int t = 0; t < T; ++t)
          if (on && t < nt) y[(size_t)(t0 + t) * N + row] = mc_f32_to_bf16(l5[t]);
      } else {
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float v = mc_round_bf16(l5[t]);
          if (on && mc_better(v, (uint32_t)row, best_v[t], best_i[t])) {
            best_v[t] = v;
            best_i[t] = (uint32_t)row;
          }
        }
      }
    }
  }

  if (MODE == 1) {
    __shared__ float bv_s[kWarpsB][T];
    __shared__ uint32_t bi_s[kWarpsB][T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float v = best_v[t];
      uint32_t i = best_i[t];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, off);
        if (mc_better(ov, oi, v, i)) {
          v = ov;
          i = oi;
        }
      }
      if (lane == 0) {
        bv_s[warp][t] = v;
        bi_s[warp][t] = i;
      }
    }
    __syncthreads();
    if (threadIdx.x < nt) {
      const int t = threadIdx.x;
      float v = bv_s[0][t];
      uint32_t i = bi_s[0][t];
      for (int w = 1; w < kWarpsB; ++w)
        if (mc_better(bv_s[w][t], bi_s[w][t], v, i)) {
          v = bv_s[w][t];
          i = bi_s[w][t];
        }
      atomicMax(keys + t0 + t, mc_argmax_key(v, i));
    }
  }
}

template <int BITS, int MODE, int T>
int launch_batched(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                   unsigned long long* keys, int batch) {
  auto fn = gemv_batched_kernel<BITS, MODE, T>;
  constexpr uint32_t smem = BatchedShape<T>::kSmem;
  static std::atomic<bool> ready[64];
  const int dev = ctx->device & 63;
  if (!ready[dev].load()) {
    MC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    ready[dev].store(true);
  }
  const int groups = (batch + T - 1) / T;
  const int nrb = (w->out_features + 31) / 32;
  // split K over up to 8 warps per row block until the warps fill one CTA per SM
  int ks_log2 = 0;
  while (ks_log2 < 3 && ((long)nrb * groups << ks_log2) < (long)ctx->num_sms * kWarpsB) ++ks_log2;
  const int rb_per_cta = kWarpsB >> ks_log2;
  const int need = (nrb + rb_per_cta - 1) / rb_per_cta;
  // one CTA per SM in all: the token groups share the SMs
  int gx = (ctx->num_sms + groups - 1) / groups;
  if (gx > need) gx = need;
  if (gx < 1) gx = 1;
  MC_CUDA(mc_launch_pdl(fn, dim3(gx, groups), dim3(kThreadsB), smem, ctx->stream,
                        reinterpret_cast<const uint8_t*>(w->codes), w->scales, w->biases, x, y,
                        keys, w->out_features, w->in_features, batch, ks_log2));
  return mc_after_launch("gemv_batched_kernel");
}

template <int BITS, int MODE>
int dispatch_batched(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                     unsigned long long* keys, int batch) {
  if (batch <= 2) return launch_batched<BITS, MODE, 2>(ctx, w, x, y, keys, batch);
  if (batch <= 4) return launch_batched<BITS, MODE, 4>(ctx, w, x, y, keys, batch);
  return launch_batched<BITS, MODE, 8>(ctx, w, x, y, keys, batch);
}

}  // namespace

// Used by mc_gemv_quant / mc_gemv_head_argmax (gemv.cu) for K <= 2048 and
// batch >= 2 on tall matrices (at least 32 rows per warp slot of one CTA per
// SM), batch >= 8 on any. Returns 1 when the call does not qualify (the
// caller then uses gemv_kernel), else MC_OK or an error code.
int mc_gemv_batched(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                    unsigned long long* keys, int batch, int mode) {
  if (batch < 2 || w->group_size != 64 || w->in_features > 64 * kMaxG) return 1;
  // short matrices (the 2048-row projection) from batch 8: measured on B200 at
  // batch 8 / 32, 12.0 / 39.9 us per-token vs 10.5 / 17.9 us here (K split 8)
  if ((long)w->out_features < (long)ctx->num_sms * kWarpsB * 32 && batch < 8) return 1;
  if ((int)BatchedShape<8>::kSmem + 4096 > ctx->max_smem_optin) return 1;
  if (!mc_aligned(w->codes, 16) || !mc_aligned(x, 16)) return 1;
  if (w->bits == 6)
    return mode ? dispatch_batched<6, 1>(ctx, w, x, y, keys, batch)
                : dispatch_batched<6, 0>(ctx, w, x, y, keys, batch);
  return mode ? dispatch_batched<4, 1>(ctx, w, x, y, keys, batch)
              : dispatch_batched<4, 0>(ctx, w, x, y, keys, batch);
}
