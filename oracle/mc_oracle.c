/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the quantized MoE matmul path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference leg may load this library, and only as the checker or the
 * timed CPU baseline. The product (molten_b200/) never calls it.
 *
 * PARITY UNPINNED: the reference (zhangshuibai/molten) is Rust + Metal and
 * cannot run on this machine, and it ships no tests, fixtures or golden
 * vectors for this path. This file restates the reference's arithmetic from
 * its Metal sources (file:line cited per function, paths inside the
 * reference project) and fixes every fp32 reduction order so that the CUDA
 * kernels can be checked bit for bit. Where the reference's order is that of
 * Apple's simd_sum (unspecified), the canonical order below is this
 * project's choice, shared with the CUDA kernels and stated at the top of
 * molten_b200/csrc/gemv_common.cuh. It is pinned by hand-computable known answers in
 * tests/test_oracle.py and by the committed fixtures in tests/golden/.
 *
 * Build: oracle/build.py (gcc -O3 -fopenmp -ffp-contract=off; fmaf only where named).
 *
 * Conventions (weights.rs:7-20, quant.rs:1-3, lfm.metal:185-199):
 *   Q4: codes u32[N][K/8], 8 codes per word, low nibble first.
 *   Q6: codes are a little-endian bit stream, code k at bits 6k..6k+5
 *       (MLX's 4-codes-in-3-bytes packing).
 *   scales, biases: bf16[N][K/64]; w = s*q + b.
 *   Activations bf16; accumulation fp32.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ numerics */

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float or_bf16_to_f32(uint16_t h) { return f_of(((uint32_t)h) << 16); }

/* round to nearest even; NaN -> quiet NaN (MLX bfloat cast). */
uint16_t or_f32_to_bf16(float f) {
  uint32_t u = u_of(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float rb(float f) { return or_bf16_to_f32(or_f32_to_bf16(f)); }
static float bf(uint16_t h) { return or_bf16_to_f32(h); }

/* exp(x): Cody-Waite reduction by ln2 (LN2_HI = 22713/2^15), degree-7 Taylor
 * polynomial in Horner form, 2^n applied as two power-of-two factors. The
 * same steps as the CUDA side's mc_exp, written again here. */
float or_exp(float x) {
  const float LOG2E = 1.44269502162933349609375f;
  const float LN2_HI = 0.693145751953125f;
  const float LN2_LO = 1.42860682030941723212e-06f;
  if (x != x) return x;
  if (x > 88.8f) return f_of(0x7f800000u);
  if (x < -104.0f) return 0.0f;
  float n = rintf(x * LOG2E);
  float r = fmaf(-n, LN2_HI, x);
  r = fmaf(-n, LN2_LO, r);
  float p = 1.98412698412698412698e-04f;
  p = fmaf(p, r, 1.38888888888888888889e-03f);
  p = fmaf(p, r, 8.33333333333333333333e-03f);
  p = fmaf(p, r, 4.16666666666666666667e-02f);
  p = fmaf(p, r, 1.66666666666666666667e-01f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ni = (int)n;
  int n1 = ni / 2;
  int n2 = ni - n1;
  float s1 = f_of((uint32_t)(n1 + 127) << 23);
  float s2 = f_of((uint32_t)(n2 + 127) << 23);
  return (p * s1) * s2;
}

/* elementwise.metal:11-13 / lfm.metal:1442-1443: g / (1 + exp(-g)). */
float or_silu(float g) { return g / (1.0f + or_exp(-g)); }
/* lfm.metal:629-630. */
float or_sigmoid(float z) { return 1.0f / (1.0f + or_exp(-z)); }

/* lfm.metal:1200-1207. */
uint64_t or_argmax_key(float v, uint32_t i) {
  uint32_t u = u_of(v);
  if ((u << 1) == 0u) u = 0u;
  uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)o << 32) | (uint64_t)(~i);
}

/* lfm.metal:1119-1124. */
static int better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

/* 32-lane xor butterfly (masks 16, 8, 4, 2, 1); every lane ends with the
 * same bits because fp32 addition is commutative. */
static float butterfly32(float* v) {
  for (int m = 16; m >= 1; m >>= 1) {
    float t[32];
    for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ m];
    memcpy(v, t, sizeof t);
  }
  return v[0];
}

/* ------------------------------------------------------ quantized GEMV row
 *
 * Reference: dot_word_q4 + GEMV_Q4_BODY, lfm.metal:102-139 (per 8-code word
 * s*(q.x) + b*(sum x)); decode_q6/_reg lfm.metal:186-243.
 * Canonical order (this project's; Apple's simd_sum order is unspecified):
 *   - lane l (0..31) owns groups g = l, l+32, ... and keeps acc_l, starting
 *     at +0.0f;
 *   - per group (64 codes): four quarters p of 16 codes (i = 16p..16p+15
 *     within the group), each with two chains cE[p] and cO[p] -- Q4: codes
 *     of the even and odd 32-bit word (bit 3 of k), Q6: even and odd k --
 *     each starting at +0 and cX[p] = fmaf(q_k * 2^e_k, x_k * 2^-e_k, cX[p])
 *     in increasing k, where e_k is the bit position the GPU leaves code k
 *     at (E4 / E6 below; the product is exact, the power-of-two pre-scaling
 *     of x is what the GPU reads);
 *     cX = (cX[0] + cX[1]) + (cX[2] + cX[3]); qx = cE + cO;
 *   - xg_g = x_{64g} + x_{64g+1} + ... (left to right) -- shared by all rows;
 *   - term = fmaf(s_g, qx, b_g * xg_g); acc_l = acc_l + term;
 *   - row sum = 32-lane xor butterfly of acc_l.
 */
static const int E4[8] = {0, 4, 8, 12, 16, 8, 12, 16};
static const int E6[4] = {0, 6, 12, 10};

static void prescale(const float* x, int K, int bits, float* xs, float* xg) {
  for (int k = 0; k < K; ++k) {
    int e = bits == 4 ? E4[k & 7] : E6[k & 3];
    xs[k] = x[k] * ldexpf(1.0f, -e);
  }
  for (int g = 0; g < K / 64; ++g) {
    float s = x[64 * g];
    for (int i = 1; i < 64; ++i) s = s + x[64 * g + i];
    xg[g] = s;
  }
}

static inline uint32_t code_at(const uint8_t* row, int bits, int k) {
  if (bits == 4) {
    uint32_t w;
    memcpy(&w, row + 4 * (k >> 3), 4);
    return (w >> (4 * (k & 7))) & 15u;
  }
  /* 6-bit little-endian stream */
  int bit = 6 * k;
  uint32_t lo = row[bit >> 3];
  /* a code at bit offset 0 or 2 of its byte does not reach the next byte
   * (and for the last code of a row that byte is outside the row) */
  uint32_t hi = (bit & 7) > 2 ? row[(bit >> 3) + 1] : 0;
  uint32_t v = lo | (hi << 8);
  return (v >> (bit & 7)) & 63u;
}

static float row_dot(const uint8_t* row, const uint16_t* s, const uint16_t* b,
                     int bits, int K, const float* xs, const float* xg) {
  float acc[32];
  for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
  const int G = K / 64;
  for (int g = 0; g < G; ++g) {
    float cE[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cO[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int i = 0; i < 64; ++i) {
      int k = 64 * g + i;
      uint32_t q = code_at(row, bits, k);
      int e = bits == 4 ? E4[k & 7] : E6[k & 3];
      float qf = (float)(q << e);
      /* Q4: chain by word parity (bit 3 of k); Q6: by code parity */
      int odd = bits == 4 ? (k >> 3) & 1 : k & 1;
      int p = i >> 4;
      if (odd) cO[p] = fmaf(qf, xs[k], cO[p]);
      else cE[p] = fmaf(qf, xs[k], cE[p]);
    }
    float sE = (cE[0] + cE[1]) + (cE[2] + cE[3]);
    float sO = (cO[0] + cO[1]) + (cO[2] + cO[3]);
    float qx = sE + sO;
    float term = fmaf(bf(s[g]), qx, bf(b[g]) * xg[g]);
    acc[g & 31] = acc[g & 31] + term;
  }
  return butterfly32(acc);
}

static size_t row_bytes(int bits, int K) { return (size_t)K * bits / 8; }

/* gemv_quant (kernels/lfm.rs:112-149): y[b][n] = bf16(row_dot). acc_out
 * (nullable) receives the fp32 sums. x: bf16 [B][K]. */
void or_gemv_quant(const void* codes, const uint16_t* scales, const uint16_t* biases,
                   int bits, int N, int K, const uint16_t* x, int B,
                   uint16_t* y, float* acc_out) {
  float* xf = (float*)malloc(sizeof(float) * K);
  float* xs = (float*)malloc(sizeof(float) * K);
  float* xg = (float*)malloc(sizeof(float) * (K / 64));
  const int G = K / 64;
  for (int bb = 0; bb < B; ++bb) {
    for (int k = 0; k < K; ++k) xf[k] = bf(x[(size_t)bb * K + k]);
    prescale(xf, K, bits, xs, xg);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = (const uint8_t*)codes + (size_t)n * row_bytes(bits, K);
      float v = row_dot(row, scales + (size_t)n * G, biases + (size_t)n * G, bits, K, xs, xg);
      if (acc_out) acc_out[(size_t)bb * N + n] = v;
      if (y) y[(size_t)bb * N + n] = or_f32_to_bf16(v);
    }
  }
  free(xf); free(xs); free(xg);
}

/* gemv_head_argmax + token_tail (kernels/lfm.rs:826-888; lfm.metal:1215-1291):
 * logits are bf16-rounded, the winner is "value desc, index asc" (ties to the
 * lowest token id), reported as the 64-bit key and the token. */
void or_head_argmax(const void* codes, const uint16_t* scales, const uint16_t* biases,
                    int bits, int N, int K, const uint16_t* x, int B,
                    uint64_t* keys, uint32_t* tokens) {
  float* xf = (float*)malloc(sizeof(float) * K);
  float* xs = (float*)malloc(sizeof(float) * K);
  float* xg = (float*)malloc(sizeof(float) * (K / 64));
  float* lg = (float*)malloc(sizeof(float) * N);
  const int G = K / 64;
  for (int bb = 0; bb < B; ++bb) {
    for (int k = 0; k < K; ++k) xf[k] = bf(x[(size_t)bb * K + k]);
    prescale(xf, K, bits, xs, xg);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint8_t* row = (const uint8_t*)codes + (size_t)n * row_bytes(bits, K);
      lg[n] = rb(row_dot(row, scales + (size_t)n * G, biases + (size_t)n * G, bits, K, xs, xg));
    }
    float bv = -INFINITY;
    uint32_t bi = 0;
    for (int n = 0; n < N; ++n)
      if (better(lg[n], (uint32_t)n, bv, bi)) { bv = lg[n]; bi = (uint32_t)n; }
    if (keys) keys[bb] = or_argmax_key(bv, bi);
    if (tokens) tokens[bb] = bi;
  }
  free(xf); free(xs); free(xg); free(lg);
}

/* argmax_bf16 (kernels/lfm.rs:794-820; lfm.metal:1126-1192): ties to the
 * lowest index; the result does not depend on the partition. */
void or_argmax_bf16(const uint16_t* logits, int n, int B, uint32_t* out) {
  for (int bb = 0; bb < B; ++bb) {
    float bv = -INFINITY;
    uint32_t bi = 0;
    for (int i = 0; i < n; ++i) {
      float v = bf(logits[(size_t)bb * n + i]);
      if (better(v, (uint32_t)i, bv, bi)) { bv = v; bi = (uint32_t)i; }
    }
    out[bb] = bi;
  }
}

/* ------------------------------------------------------- add + RMSNorm
 * lfm_norm_row_v8_tg lfm.metal:306-366 (bf16 residual add, fp32 sum of
 * squares, total/H + eps, bf16 output). Canonical order: 256 partials, partial
 * t = fmaf chain over k = 8t..8t+7; 8 warps of 32 partials each reduced by the
 * xor butterfly; total = ((p0 + p1) + p2) ... + p7; inv = 1/sqrtf(total/H +
 * eps) (IEEE sqrt and divide); n_k = bf16((h'_k * inv) * w_k). H = 2048.
 * b (the residual addend) may be NULL (treated as all zeros, h' = h). */
void or_add_rmsnorm(const uint16_t* h, const uint16_t* b, const uint16_t* w, int H,
                    float eps, uint16_t* hout, uint16_t* nout) {
  float* hp = (float*)malloc(sizeof(float) * H);
  for (int k = 0; k < H; ++k) {
    float v = b ? bf(h[k]) + bf(b[k]) : bf(h[k]);
    hp[k] = rb(v);
    if (hout) hout[k] = or_f32_to_bf16(v);
  }
  const int T = 256, per = H / 256;
  float part[256];
  for (int t = 0; t < T; ++t) {
    float a = 0.0f;
    for (int i = 0; i < per; ++i) { float v = hp[per * t + i]; a = fmaf(v, v, a); }
    part[t] = a;
  }
  float total = 0.0f;
  for (int wp = 0; wp < 8; ++wp) total = total + butterfly32(part + 32 * wp);
  float inv = 1.0f / sqrtf(total / (float)H + eps);
  for (int k = 0; k < H; ++k) nout[k] = or_f32_to_bf16((hp[k] * inv) * bf(w[k]));
  free(hp);
}

/* --------------------------------------------------------- router GEMV
 * lfm_router_lane_sum_tg_fixed lfm.metal:728-771 (lane-strided fp32 dot,
 * simd_sum). Canonical order: lane l owns k = 256j + 8l + i (j outer, i
 * inner), acc = fmaf(W_k, n_k, acc) from +0; 32-lane xor butterfly.
 * w_dtype 0 = bf16 router (BASELINE cfg1), 1 = f32 router (reference model).
 * K must be a multiple of 256. */
void or_router_logits(const uint16_t* normed, const void* W, int w_dtype, int E, int K,
                      float* logits) {
  for (int e = 0; e < E; ++e) {
    float acc[32];
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      for (int j = 0; j < K / 256; ++j)
        for (int i = 0; i < 8; ++i) {
          int k = 256 * j + 8 * l + i;
          float wv = w_dtype == 0 ? bf(((const uint16_t*)W)[(size_t)e * K + k])
                                  : ((const float*)W)[(size_t)e * K + k];
          a = fmaf(wv, bf(normed[k]), a);
        }
      acc[l] = a;
    }
    logits[e] = butterfly32(acc);
  }
}

/* --------------------------------------------------------------- top-4
 * Selection: lfm_topk_warp_b lfm.metal:619-675 and lfm_moe_route_batch
 * :1558-1602 -- repeat TOPK times: the unused candidate with the greatest
 * value, an exact tie to the lower expert id.
 * mode 0 (softmax_renorm, BASELINE cfg1/cfg3): value = raw logit (softmax is
 *   monotone); weights = softmax over all experts renormalised over the
 *   selected ones, computed as e_r = exp(z_r - z_top1), den = ((e0+e1)+e2)+e3,
 *   w_r = bf16(e_r / den) (the full-softmax denominator cancels).
 * mode 1 (sigmoid_bias, the reference model): s = sigmoid(z); value = s +
 *   bias; den = eps; den += s_r in rank order; w_r = bf16(s_r / den). */
void or_route_topk(const float* z, int E, int topk, int mode, const float* bias,
                   float eps, uint32_t* ids, uint16_t* wts) {
  float val[256], s[256];
  int used[256];
  for (int e = 0; e < E; ++e) {
    used[e] = 0;
    if (mode == 0) { s[e] = z[e]; val[e] = z[e]; }
    else { s[e] = or_sigmoid(z[e]); val[e] = s[e] + (bias ? bias[e] : 0.0f); }
  }
  uint32_t ch[8];
  for (int r = 0; r < topk; ++r) {
    float bv = -INFINITY; uint32_t bi = 0xffffffffu;
    for (int e = 0; e < E; ++e) {
      if (used[e]) continue;
      if (better(val[e], (uint32_t)e, bv, bi)) { bv = val[e]; bi = (uint32_t)e; }
    }
    if (bi == 0xffffffffu) bi = 0;
    ch[r] = bi; used[bi] = 1;
  }
  if (mode == 0) {
    float ex[8], den = 0.0f;
    for (int r = 0; r < topk; ++r) { ex[r] = or_exp(z[ch[r]] - z[ch[0]]); den = den + ex[r]; }
    for (int r = 0; r < topk; ++r) { ids[r] = ch[r]; wts[r] = or_f32_to_bf16(ex[r] / den); }
  } else {
    float den = eps;
    for (int r = 0; r < topk; ++r) den = den + s[ch[r]];
    for (int r = 0; r < topk; ++r) { ids[r] = ch[r]; wts[r] = or_f32_to_bf16(s[ch[r]] / den); }
  }
}

/* router_addnorm_route (kernels/lfm.rs:266-311; lfm.metal:773-854), batch B
 * independent rows. h, b (nullable), out rows bf16 [B][H]; logits f32 [B][E];
 * ids u32 [B][4]; wts bf16 [B][4]. */
void or_router_addnorm_route(const uint16_t* h, const uint16_t* b, const uint16_t* norm_w,
                             const void* W, int w_dtype, const float* ebias, int mode,
                             int E, int H, float eps, float route_eps, int B,
                             uint16_t* hout, uint16_t* normed, float* logits,
                             uint32_t* ids, uint16_t* wts) {
  for (int bb = 0; bb < B; ++bb) {
    const size_t o = (size_t)bb * H;
    or_add_rmsnorm(h + o, b ? b + o : NULL, norm_w, H, eps, hout + o, normed + o);
    or_router_logits(normed + o, W, w_dtype, E, H, logits + (size_t)bb * E);
    or_route_topk(logits + (size_t)bb * E, E, 4, mode, ebias, route_eps, ids + 4 * bb,
                  wts + 4 * bb);
  }
}

/* gemv_gather_act (kernels/lfm.rs:421-460; lfm.metal:1392-1445): for slot r
 * and row i, rows ids[r]*I + i of the stacked [E*I, H] gate/up weights;
 * act = bf16(bf16(silu(bf16(gate))) * bf16(up)). x: bf16 [B][H];
 * ids [B][4]; act bf16 [B][4][I]. */
void or_gemv_gather_act(const void* gc, const uint16_t* gs, const uint16_t* gb,
                        const void* uc, const uint16_t* us, const uint16_t* ub,
                        int I, int H, const uint16_t* x, const uint32_t* ids, int B,
                        uint16_t* act) {
  float* xf = (float*)malloc(sizeof(float) * H);
  float* xs = (float*)malloc(sizeof(float) * H);
  float* xg = (float*)malloc(sizeof(float) * (H / 64));
  const int G = H / 64;
  const size_t rb_ = row_bytes(4, H);
  for (int bb = 0; bb < B; ++bb) {
    for (int k = 0; k < H; ++k) xf[k] = bf(x[(size_t)bb * H + k]);
    prescale(xf, H, 4, xs, xg);
    for (int r = 0; r < 4; ++r) {
      const size_t e = ids[4 * bb + r];
#pragma omp parallel for schedule(static)
      for (int i = 0; i < I; ++i) {
        const size_t row = e * I + i;
        float g = row_dot((const uint8_t*)gc + row * rb_, gs + row * G, gb + row * G, 4, H, xs, xg);
        float u = row_dot((const uint8_t*)uc + row * rb_, us + row * G, ub + row * G, 4, H, xs, xg);
        float sl = rb(or_silu(rb(g)));
        act[((size_t)bb * 4 + r) * I + i] = or_f32_to_bf16(sl * rb(u));
      }
    }
  }
  free(xf); free(xs); free(xg);
}

/* gemv_gather_down_combine4 (kernels/lfm.rs:499-533; lfm.metal:1503-1554):
 * p_r = bf16(row_dot(down row ids[r]*H + i, act_r)); out = bf16(sum over r in
 * rank order, from 0, of bf16(w_r * p_r)). act bf16 [B][4][I]; out [B][H]. */
void or_gemv_gather_down_combine4(const void* dc, const uint16_t* ds, const uint16_t* db,
                                  int H, int I, const uint16_t* act, const uint32_t* ids,
                                  const uint16_t* wts, int B, uint16_t* out) {
  float* xf = (float*)malloc(sizeof(float) * 4 * I);
  float* xs = (float*)malloc(sizeof(float) * 4 * I);
  float* xg = (float*)malloc(sizeof(float) * 4 * (I / 64));
  const int G = I / 64;
  const size_t rb_ = row_bytes(4, I);
  for (int bb = 0; bb < B; ++bb) {
    for (int r = 0; r < 4; ++r) {
      for (int k = 0; k < I; ++k) xf[r * I + k] = bf(act[((size_t)bb * 4 + r) * I + k]);
      prescale(xf + r * I, I, 4, xs + r * I, xg + r * G);
    }
#pragma omp parallel for schedule(static)
    for (int i = 0; i < H; ++i) {
      float tot = 0.0f;
      for (int r = 0; r < 4; ++r) {
        const size_t row = (size_t)ids[4 * bb + r] * H + i;
        float p = rb(row_dot((const uint8_t*)dc + row * rb_, ds + row * G, db + row * G, 4, I,
                             xs + r * I, xg + r * G));
        tot = tot + rb(bf(wts[4 * bb + r]) * p);
      }
      out[(size_t)bb * H + i] = or_f32_to_bf16(tot);
    }
  }
  free(xf); free(xs); free(xg);
}

/* ---------------------------- decode neighbours of the MoE block (Q/K/V, conv, dense FFN) */

/* proj3_gemv_scatter (kernels/lfm.rs:150-205 -> lfm_proj3_gemv_scatter_bf16
 * lfm.metal:1020-1068): the Q, K and V GEMVs of one row x (K = 2048) in the
 * canonical row order; q[i] = bf16(Q_i . x), k[i] = bf16(K_i . x), and V row
 * i goes to the cache slot v_cache[((i / 64) * max_seq + pos) * 64 + i % 64]
 * (v_cache bf16 [nv / 64][max_seq][64]; nothing else of it is written). */
void or_proj3_gemv_scatter(const void* qc, const uint16_t* qs, const uint16_t* qb,
                           const void* kc, const uint16_t* ks, const uint16_t* kb,
                           const void* vc, const uint16_t* vs, const uint16_t* vb,
                           int nq, int nk, int nv, int K, const uint16_t* x, uint16_t* q,
                           uint16_t* k, uint16_t* v_cache, int max_seq, int pos) {
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(nv > 0 ? nv : 1));
  or_gemv_quant(qc, qs, qb, 4, nq, K, x, 1, q, NULL);
  or_gemv_quant(kc, ks, kb, 4, nk, K, x, 1, k, NULL);
  or_gemv_quant(vc, vs, vb, 4, nv, K, x, 1, tmp, NULL);
  for (int i = 0; i < nv; ++i)
    v_cache[((size_t)(i / 64) * max_seq + pos) * 64 + i % 64] = tmp[i];
  free(tmp);
}

/* conv3_gemv (kernels/lfm.rs:207-246 -> lfm_conv3_gemv_split_bf16
 * lfm.metal:1070-1110): rows c, H + c, 2H + c of the [3H][K] projection give
 * b, c, x for channel c (each bf16-rounded); with the two-tap state
 * (v0 = state[c], v1 = state[H + c]) and taps w[c][0..2]:
 *   v2 = bf16(b * x); z = bf16((w0 * v0 + w1 * v1) + w2 * v2) (no fused
 *   multiply-add, left to right: this project's order, the reference's is
 *   its compiler's); out[c] = bf16(c * z);
 *   new_state[c] = state[H + c]; new_state[H + c] = v2. */
void or_conv3_gemv(const void* codes, const uint16_t* scales, const uint16_t* biases, int H,
                   int K, const uint16_t* x, const uint16_t* w, const uint16_t* state,
                   uint16_t* out, uint16_t* new_state) {
  uint16_t* p = (uint16_t*)malloc(sizeof(uint16_t) * 3 * (size_t)H);
  or_gemv_quant(codes, scales, biases, 4, 3 * H, K, x, 1, p, NULL);
  for (int ch = 0; ch < H; ++ch) {
    const float b = bf(p[ch]), c = bf(p[H + ch]), xv = bf(p[2 * H + ch]);
    const float v0 = bf(state[ch]), v1 = bf(state[H + ch]);
    const float v2 = rb(b * xv);
    const float z = (bf(w[3 * ch]) * v0 + bf(w[3 * ch + 1]) * v1) + bf(w[3 * ch + 2]) * v2;
    out[ch] = or_f32_to_bf16(c * rb(z));
    new_state[H + ch] = or_f32_to_bf16(v2);
    new_state[ch] = state[H + ch];
  }
  free(p);
}

/* gemv_gu_act (kernels/lfm.rs:462-495 -> lfm_gemv_q4_gu_act_bf16
 * lfm.metal:1447-1498): the dense FFN front half, act[b][n] =
 * bf16(bf16(silu(bf16(gate_n . x))) * bf16(up_n . x)). x bf16 [B][K]. */
void or_gemv_gu_act(const void* gc, const uint16_t* gs, const uint16_t* gb, const void* uc,
                    const uint16_t* us, const uint16_t* ub, int N, int K, const uint16_t* x,
                    int B, uint16_t* act) {
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N * B);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N * B);
  or_gemv_quant(gc, gs, gb, 4, N, K, x, B, g, NULL);
  or_gemv_quant(uc, us, ub, 4, N, K, x, B, u, NULL);
  for (size_t i = 0; i < (size_t)N * B; ++i)
    act[i] = or_f32_to_bf16(rb(or_silu(bf(g[i]))) * bf(u[i]));
  free(g); free(u);
}

/* ------------------------------------------------- sampling draw
 * Contract: docs/PROTOCOL.md:48-75 and lfm_sample.metal:1-27 (w = pen(v)/T;
 * kept set {w >= tau}: top-k ties kept, then the smallest top-p prefix with
 * its boundary tie group; Gumbel-max draw with Philox4x32-10, counter
 * (id/4, pos, "SAMP", 0), key (seed lo, seed hi); ties to the lower id).
 * The threshold follows this project's exact integer definition (the GPU
 * finds the same one by radix selection): top-k by counts; top-p by
 * per-token masses m_i = rint(exp(w_i - max w) * 2^40) summed in 64 bits,
 * target ceil(rint(top_p * 2^32) * Z / 2^32) with Z the mass of the top-k
 * kept set (or of the whole vocabulary). log, Philox and the Gumbel
 * transform are written again here with the same steps as the CUDA side
 * (molten_b200/csrc/mc_numerics.cuh). */

/* log: x = 2^e m, m in [sqrt(1/2), sqrt(2)); 2 atanh((m-1)/(m+1)) by its odd
 * series to s^11; e ln2 with fdlibm's logf split of ln2. */
float or_log(float x) {
  uint32_t u = u_of(x);
  if (x != x || x < 0.0f) return f_of(0x7fc00000u);
  if (x == 0.0f) return f_of(0xff800000u);
  if (u >= 0x7f800000u) return x;
  int e = 0;
  if (u < 0x00800000u) { x = x * 8388608.0f; u = u_of(x); e = -23; }
  e += (int)(u >> 23) - 127;
  uint32_t mu = (u & 0x007fffffu) | 0x3f800000u;
  if (mu > 0x3fb504f3u) { mu -= 0x00800000u; e += 1; }
  const float m = f_of(mu);
  const float s = (m + -1.0f) / (m + 1.0f);
  const float z = s * s;
  float p = 9.09090936183929443359e-02f;
  p = fmaf(p, z, 1.11111111938953399658e-01f);
  p = fmaf(p, z, 1.42857149243354797363e-01f);
  p = fmaf(p, z, 2.00000002980232238770e-01f);
  p = fmaf(p, z, 3.33333343267440795898e-01f);
  const float two_s = s + s;
  const float lm = fmaf(two_s * z, p, two_s);
  const float ef = (float)e;
  return fmaf(ef, 6.9313812256e-01f, fmaf(ef, 9.0580006145e-06f, lm));
}

/* Philox4x32-10 (Salmon et al., SC 2011). */
static void or_philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

void or_philox4x32_10(uint32_t* c, uint32_t k0, uint32_t k1) { or_philox(c, k0, k1); }

uint32_t or_sample_word(uint32_t id, uint32_t pos, uint32_t seed_lo, uint32_t seed_hi) {
  uint32_t c[4] = {id >> 2, pos, 0x53414D50u, 0u};
  or_philox(c, seed_lo, seed_hi);
  return c[id & 3u];
}

/* Gumbel(0, 1) of a uniform word (lfm_sample.metal:129-142 semantics). */
float or_gumbel(uint32_t x) {
  const float v = ((float)x + 0.5f) * 2.3283064365386963e-10f;
  float e;
  if (v < 0.015625f) {
    e = v * (1.0f + v * (0.5f + v * (0.33333334f + v * 0.25f)));
  } else {
    float t = 1.0f + -v;
    if (t < 2.9802322387695312e-08f) t = 2.9802322387695312e-08f;
    e = -or_log(t);
  }
  return -or_log(e);
}

static uint32_t fkey(float v) {
  uint32_t u = u_of(v);
  if ((u << 1) == 0u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
static float kfloat(uint32_t k) { return f_of((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

/* lfm_sample.metal:96-105. */
float or_sample_w(float v, int seen, float inv_temp, float penalty, float inv_penalty) {
  if (seen) v = v > 0.0f ? v * inv_penalty : v * penalty;
  uint32_t u = u_of(v * inv_temp);
  if ((u << 1) == 0u) u = 0u;
  return f_of(u);
}

static uint64_t token_mass(float w, float M) {
  const float e = or_exp(w - M);
  if (e != e) return 0u;
  return (uint64_t)llrintf(e * 1099511627776.0f);
}

typedef struct { uint32_t key; uint64_t mass; } or_km;

static int cmp_key_desc(const void* a, const void* b) {
  const uint32_t x = ((const or_km*)a)->key, y = ((const or_km*)b)->key;
  return x < y ? 1 : (x > y ? -1 : 0);
}

/* The draw: returns the argmax key (value w + G desc, id asc) of the kept
 * tokens and the threshold key in *tau_out (0: every token kept). top_k 0
 * or >= V is off; top_p >= 1 is off. */
uint64_t or_sample_draw(const uint16_t* logits, int V, const uint32_t* seen, float temperature,
                        uint32_t top_k, float top_p, float penalty, uint64_t seed, uint32_t pos,
                        uint32_t* tau_out) {
  const float inv_temp = 1.0f / temperature, inv_pen = 1.0f / penalty;
  const int use_pen = penalty != 1.0f && seen != NULL;
  if (top_k >= (uint32_t)V) top_k = 0;
  float* w = (float*)malloc(sizeof(float) * V);
  uint32_t* keys = (uint32_t*)malloc(sizeof(uint32_t) * V);
  uint32_t mk = 0;
  for (int i = 0; i < V; ++i) {
    const int sn = use_pen && ((seen[i >> 5] >> (i & 31)) & 1u);
    w[i] = or_sample_w(bf(logits[i]), sn, inv_temp, penalty, inv_pen);
    keys[i] = fkey(w[i]);
    if (keys[i] > mk) mk = keys[i];
  }
  uint32_t tau = 0;
  if (top_k != 0 || top_p < 1.0f) {
    const float M = kfloat(mk);
    or_km* srt = (or_km*)malloc(sizeof(or_km) * V);
    for (int i = 0; i < V; ++i) {
      srt[i].key = keys[i];
      srt[i].mass = token_mass(w[i], M);
    }
    qsort(srt, V, sizeof(or_km), cmp_key_desc);
    uint32_t tau_k = 0;
    if (top_k) tau_k = srt[top_k - 1].key;  /* the k-th largest; ties kept */
    tau = tau_k;
    if (top_p < 1.0f) {
      uint64_t Z = 0;
      for (int i = 0; i < V && srt[i].key >= tau_k; ++i) Z += srt[i].mass;
      const uint64_t pf = (uint64_t)llrintf(top_p * 4294967296.0f);
      const unsigned __int128 prod = (unsigned __int128)pf * Z + 0xffffffffu;
      uint64_t target = (uint64_t)(prod >> 32);
      if (target == 0) target = 1;
      /* the largest key whose mass at or above it reaches the target: walk
       * the distinct keys downwards, each tie group added whole */
      uint64_t cum = 0;
      tau = srt[V - 1].key;
      for (int j = 0; j < V;) {
        int j2 = j;
        while (j2 < V && srt[j2].key == srt[j].key) cum += srt[j2++].mass;
        if (cum >= target) { tau = srt[j].key; break; }
        j = j2;
      }
    }
    free(srt);
  }
  uint64_t best = 0;
  const uint32_t slo = (uint32_t)seed, shi = (uint32_t)(seed >> 32);
  for (int i = 0; i < V; ++i) {
    if (keys[i] < tau) continue;
    const float g = or_gumbel(or_sample_word((uint32_t)i, pos, slo, shi));
    const uint64_t k = or_argmax_key(w[i] + g, (uint32_t)i);
    if (k > best) best = k;
  }
  if (tau_out) *tau_out = tau;
  free(w); free(keys);
  return best;
}

/* ------------------------------------------------------------- prefill */

/* moe_route_batch (kernels/lfm.rs:536-555; lfm.metal:1558-1602). */
void or_moe_route_batch(const float* logits, int m, int E, int mode, const float* bias,
                        float eps, uint32_t* ids, uint16_t* gw) {
  for (int t = 0; t < m; ++t)
    or_route_topk(logits + (size_t)t * E, E, 4, mode, bias, eps, ids + 4 * (size_t)t,
                  gw + 4 * (size_t)t);
}

/* moe_count_slots / moe_offsets / moe_sorted (lfm.metal:1604-1686): per-expert
 * counts, exclusive scan, and the stable token-major, rank-major scatter:
 * ids_sorted[pos] = t, slotpos[t*topk + r] = pos. */
void or_moe_sort(const uint32_t* ids, int m, int topk, int E, uint32_t* counts,
                 uint32_t* offsets, uint32_t* ids_sorted, uint32_t* slotpos) {
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (size_t i = 0; i < (size_t)m * topk; ++i) counts[ids[i]]++;
  uint32_t acc = 0;
  for (int e = 0; e < E; ++e) { offsets[e] = acc; acc += counts[e]; }
  uint32_t* pos = (uint32_t*)malloc(sizeof(uint32_t) * E);
  memcpy(pos, offsets, sizeof(uint32_t) * E);
  for (int t = 0; t < m; ++t)
    for (int r = 0; r < topk; ++r) {
      uint32_t e = ids[(size_t)t * topk + r];
      uint32_t p = pos[e]++;
      ids_sorted[p] = (uint32_t)t;
      slotpos[(size_t)t * topk + r] = p;
    }
  free(pos);
}

/* dequantize<bfloat16, 8, 4> quant_nax.metal:2947-2953: w = bf16(s*q + b)
 * (s*q is exact in fp32, so the one rounding is of the sum). out bf16 [N][K]. */
void or_dequant_q4(const uint32_t* codes, const uint16_t* scales, const uint16_t* biases,
                   int N, int K, uint16_t* out) {
  const int G = K / 64;
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      uint32_t w = codes[(size_t)n * (K / 8) + k / 8];
      float q = (float)((w >> (4 * (k & 7))) & 15u);
      float s = bf(scales[(size_t)n * G + k / 64]), b = bf(biases[(size_t)n * G + k / 64]);
      out[(size_t)n * K + k] = or_f32_to_bf16(fmaf(s, q, b));
    }
}

/* Grouped Q4 GEMM reference (quant.rs:228-266 -> lfm_qmm_t_body
 * quant_nax.metal:4091-4234): for sorted row i of expert e,
 * C[i][n] = bf16(sum_k A[i][k] * Wdeq[e*N + n][k]) with fp32 accumulation in
 * increasing k from 0.0f (the tensor-op order on the GPU differs, hence a
 * tolerance). A rows are given already in sorted order (gx / act).
 * Each output keeps that one sequential chain; only the loop nest around it
 * is arranged for speed (the dequantised expert transposed to [K][N], blocks
 * of rows sharing each pass over it, row blocks spread over OpenMP threads),
 * so the result does not depend on the thread count. */
#define OR_RB 8
void or_gemm_q4_grouped(const uint16_t* A, int S, int K, const uint32_t* codes,
                        const uint16_t* scales, const uint16_t* biases, int N,
                        const uint32_t* counts, const uint32_t* offsets, int E,
                        uint16_t* C, float* Cacc) {
  uint16_t* wd = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N * K);
  float* wt = (float*)malloc(sizeof(float) * (size_t)N * K);  /* [K][N] */
  for (int e = 0; e < E; ++e) {
    if (counts[e] == 0) continue;
    or_dequant_q4(codes + (size_t)e * N * (K / 8), scales + (size_t)e * N * (K / 64),
                  biases + (size_t)e * N * (K / 64), N, K, wd);
    for (int n = 0; n < N; ++n)
      for (int k = 0; k < K; ++k) wt[(size_t)k * N + n] = bf(wd[(size_t)n * K + k]);
    const long i0 = offsets[e], rows = counts[e];
    const long nblk = (rows + OR_RB - 1) / OR_RB;
#pragma omp parallel for schedule(dynamic, 1)
    for (long blk = 0; blk < nblk; ++blk) {
      const long r0 = i0 + blk * OR_RB;
      const int rb = (int)((rows - blk * OR_RB) < OR_RB ? (rows - blk * OR_RB) : OR_RB);
      float* acc = (float*)calloc((size_t)OR_RB * N, sizeof(float));
      float af[OR_RB];
      for (int k = 0; k < K; ++k) {
        const float* wrow = wt + (size_t)k * N;
        for (int r = 0; r < rb; ++r) af[r] = bf(A[(size_t)(r0 + r) * K + k]);
        for (int r = 0; r < rb; ++r) {
          float* ar = acc + (size_t)r * N;
          const float a = af[r];
          for (int n = 0; n < N; ++n) ar[n] = ar[n] + a * wrow[n];
        }
      }
      for (int r = 0; r < rb; ++r)
        for (int n = 0; n < N; ++n) {
          const float a = acc[(size_t)r * N + n];
          if (Cacc) Cacc[(size_t)(r0 + r) * N + n] = a;
          C[(size_t)(r0 + r) * N + n] = or_f32_to_bf16(a);
        }
      free(acc);
    }
  }
  (void)S;
  free(wd); free(wt);
}

/* silu_mul_bf16 (elementwise.metal:7-15). */
void or_silu_mul(const uint16_t* g, const uint16_t* u, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = or_f32_to_bf16(rb(or_silu(bf(g[i]))) * bf(u[i]));
}

/* gather_rows_bf16 (elementwise.metal:19-52). */
void or_gather_rows(const uint16_t* table, const uint32_t* ids, int rows, int H,
                    uint16_t* out) {
  for (int r = 0; r < rows; ++r)
    memcpy(out + (size_t)r * H, table + (size_t)ids[r] * H, sizeof(uint16_t) * H);
}

/* moe_combine_rows (kernels/lfm.rs:701-756; lfm.metal:859-940):
 * out[t][h] = bf16(sum_r (from 0, rank order) bf16(gw[t][r] * ed[slotpos][h])). */
void or_moe_combine(const uint16_t* ed, const uint32_t* slotpos, const uint16_t* gw, int m,
                    int topk, int H, uint16_t* out) {
  for (int t = 0; t < m; ++t)
    for (int h = 0; h < H; ++h) {
      float s = 0.0f;
      for (int r = 0; r < topk; ++r) {
        uint32_t p = slotpos[(size_t)t * topk + r];
        s = s + rb(bf(gw[(size_t)t * topk + r]) * bf(ed[(size_t)p * H + h]));
      }
      out[(size_t)t * H + h] = or_f32_to_bf16(s);
    }
}

/* Whole prefill MoE FFN for a chunk (moe_prefill lfm.rs:847-965, without the
 * router GEMV: the logits are an input, as in BASELINE cfg3). x: bf16 [m][H];
 * logits f32 [m][E]; weights stacked [E*I][H] (gate, up) and [E*H][I] (down).
 * Outputs: ids/gw [m][4]; out bf16 [m][H]. Intermediates optional (NULL). */
void or_moe_prefill(const uint16_t* x, const float* logits, int m, int E, int H, int I,
                    int mode, const float* bias,
                    const uint32_t* gc, const uint16_t* gs, const uint16_t* gb,
                    const uint32_t* uc, const uint16_t* us, const uint16_t* ub,
                    const uint32_t* dc, const uint16_t* ds, const uint16_t* db,
                    uint32_t* ids, uint16_t* gw, uint32_t* ids_sorted, uint32_t* slotpos,
                    uint16_t* act_out, uint16_t* ed_out, uint16_t* out) {
  const size_t S = (size_t)m * 4;
  uint32_t* counts = (uint32_t*)malloc(sizeof(uint32_t) * E);
  uint32_t* offsets = (uint32_t*)malloc(sizeof(uint32_t) * E);
  uint16_t* gx = (uint16_t*)malloc(sizeof(uint16_t) * S * H);
  uint16_t* g = (uint16_t*)malloc(sizeof(uint16_t) * S * I);
  uint16_t* u = (uint16_t*)malloc(sizeof(uint16_t) * S * I);
  uint16_t* act = (uint16_t*)malloc(sizeof(uint16_t) * S * I);
  uint16_t* ed = (uint16_t*)malloc(sizeof(uint16_t) * S * H);
  or_moe_route_batch(logits, m, E, mode, bias, 1e-6f, ids, gw);
  or_moe_sort(ids, m, 4, E, counts, offsets, ids_sorted, slotpos);
  or_gather_rows(x, ids_sorted, (int)S, H, gx);
  or_gemm_q4_grouped(gx, (int)S, H, gc, gs, gb, I, counts, offsets, E, g, NULL);
  or_gemm_q4_grouped(gx, (int)S, H, uc, us, ub, I, counts, offsets, E, u, NULL);
  or_silu_mul(g, u, S * I, act);
  or_gemm_q4_grouped(act, (int)S, I, dc, ds, db, H, counts, offsets, E, ed, NULL);
  or_moe_combine(ed, slotpos, gw, m, 4, H, out);
  if (act_out) memcpy(act_out, act, sizeof(uint16_t) * S * I);
  if (ed_out) memcpy(ed_out, ed, sizeof(uint16_t) * S * H);
  free(counts); free(offsets); free(gx); free(g); free(u); free(act); free(ed);
}
