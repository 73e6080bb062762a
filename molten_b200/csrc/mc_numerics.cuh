// Canonical arithmetic shared by every decode kernel of this library.
//
// The decode path must produce bit-identical top-4 expert ids and argmax
// tokens run after run and against the CPU restatement in oracle/. That only
// holds if every fp32 operation on the way is fixed: which products are
// fused, the order of every sum, and the exp/sqrt/div used. This header fixes
// the pieces that are not plain IEEE add/mul/fma:
//
//   * bf16 <-> f32 conversion (round-to-nearest-even, as MLX's bfloat cast);
//   * mc_exp: our own exp (Cody-Waite reduction by ln2, degree-7 Taylor
//     polynomial in Horner form, exponent reconstruction in two steps) so the
//     GPU and the oracle compute SiLU, sigmoid and softmax weights identically
//     (CUDA's expf and glibc's expf differ in the last ulp);
//   * the argmax key of lfm.metal:1200-1207 (value desc, index asc).
//
// The reduction orders themselves are documented next to each kernel.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

#define MC_HD __host__ __device__ __forceinline__

// bf16 bits -> f32 (exact).
MC_HD float mc_bf16_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(((uint32_t)h) << 16);
#else
  union { uint32_t u; float f; } v; v.u = ((uint32_t)h) << 16; return v.f;
#endif
}

MC_HD uint32_t mc_f32_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  union { uint32_t u; float f; } v; v.f = f; return v.u;
#endif
}

MC_HD float mc_bits_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  union { uint32_t u; float f; } v; v.u = u; return v.f;
#endif
}

// f32 -> bf16 bits, round to nearest even; NaN becomes a quiet NaN.
MC_HD uint16_t mc_f32_to_bf16(float f) {
  uint32_t u = mc_f32_bits(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// f32 rounded through bf16 and back (the value a bfloat store + reload sees).
MC_HD float mc_round_bf16(float f) { return mc_bf16_to_f32(mc_f32_to_bf16(f)); }

#ifdef __CUDA_ARCH__
#define MC_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#define MC_MUL(a, b) __fmul_rn((a), (b))
#define MC_ADD(a, b) __fadd_rn((a), (b))
#define MC_DIV(a, b) __fdiv_rn((a), (b))
#define MC_SQRT(a) __fsqrt_rn(a)
#define MC_RINT(a) rintf(a)
#else
#include <math.h>
#define MC_FMA(a, b, c) fmaf((a), (b), (c))
#define MC_MUL(a, b) ((a) * (b))
#define MC_ADD(a, b) ((a) + (b))
#define MC_DIV(a, b) ((a) / (b))
#define MC_SQRT(a) sqrtf(a)
#define MC_RINT(a) rintf(a)
#endif

// exp(x) for float x.
// Method: x = n*ln2 + r with n = rint(x*log2(e)) and the Cody-Waite split
// ln2 = LN2_HI + LN2_LO, where LN2_HI = 22713/32768 has 15 significant bits
// so n*LN2_HI is exact for |n| < 512; then exp(r) by the Taylor series of
// degree 7 (coefficients 1/k!) for |r| <= ln2/2, whose truncation error is
// below 0.15 ulp; finally 2^n applied as two exact power-of-two factors so
// results that land in the subnormal range round once.
MC_HD float mc_exp(float x) {
  const float LOG2E = 1.44269502162933349609375f;       // float(log2(e))
  const float LN2_HI = 0.693145751953125f;              // 22713 / 2^15
  const float LN2_LO = 1.42860682030941723212e-06f;     // ln2 - LN2_HI
  if (!(x == x)) return x;                              // NaN
  if (x > 88.8f) return mc_bits_f32(0x7f800000u);       // +inf
  if (x < -104.0f) return 0.0f;
  const float n = MC_RINT(MC_MUL(x, LOG2E));
  float r = MC_FMA(-n, LN2_HI, x);
  r = MC_FMA(-n, LN2_LO, r);
  float p = 1.98412698412698412698e-04f;                // 1/5040
  p = MC_FMA(p, r, 1.38888888888888888889e-03f);        // 1/720
  p = MC_FMA(p, r, 8.33333333333333333333e-03f);        // 1/120
  p = MC_FMA(p, r, 4.16666666666666666667e-02f);        // 1/24
  p = MC_FMA(p, r, 1.66666666666666666667e-01f);        // 1/6
  p = MC_FMA(p, r, 0.5f);
  p = MC_FMA(p, r, 1.0f);
  p = MC_FMA(p, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni / 2;
  const int n2 = ni - n1;
  const float s1 = mc_bits_f32((uint32_t)(n1 + 127) << 23);
  const float s2 = mc_bits_f32((uint32_t)(n2 + 127) << 23);
  return MC_MUL(MC_MUL(p, s1), s2);
}

// SiLU as MLX/lfm.metal write it: g / (1 + exp(-g)).
MC_HD float mc_silu(float g) { return MC_DIV(g, MC_ADD(1.0f, mc_exp(-g))); }

// Logistic sigmoid, lfm.metal:629-630: 1 / (1 + exp(-z)).
MC_HD float mc_sigmoid(float z) { return MC_DIV(1.0f, MC_ADD(1.0f, mc_exp(-z))); }

// Orderable 64-bit argmax key (lfm.metal:1200-1207): a larger key is a larger
// value, or an equal value at a lower index; -0 folds to +0.
MC_HD unsigned long long mc_argmax_key(float v, uint32_t i) {
  uint32_t u = mc_f32_bits(v);
  if ((u << 1) == 0u) u = 0u;
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(~i);
}

MC_HD uint32_t mc_key_token(unsigned long long key) { return ~(uint32_t)(key & 0xffffffffull); }

// Candidate merge of lfm.metal:1119-1124: value desc, index asc.
MC_HD bool mc_better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// Bit positions the decode GEMVs leave each code at when they turn it into a
// float with the 2^23 magic (see gemv_common.cuh). Code k of a 4-bit word sits
// at bit E4[k % 8] of its register, so the kernels multiply it by x * 2^-E4.
// The products are exact, so the canonical sum is simply
// acc = fma(q * 2^e, x * 2^-e, acc) for each code in order.
#define MC_E4_0 0
#define MC_E4_1 4
#define MC_E4_2 8
#define MC_E4_3 12
#define MC_E4_4 16
#define MC_E4_5 8
#define MC_E4_6 12
#define MC_E4_7 16
// 6-bit codes: position within the 4-code (3-byte) packet.
#define MC_E6_0 0
#define MC_E6_1 6
#define MC_E6_2 12
#define MC_E6_3 10

// ---------------------------------------------------------------- sampling
// Pieces of the sampled draw (sample.cu), restated in the CPU oracle.

// log(x) for float x > 0.
// Method: x = 2^e * m with m in [sqrt(1/2), sqrt(2)); log(m) = 2 atanh(s) with
// s = (m - 1) / (m + 1), |s| <= 0.1716, summed as the odd series
// 2s (1 + s^2/3 + s^4/5 + ... + s^10/11) (truncation below 2e-11); then
// e * ln2 added with ln2 split into a high part with trailing zero bits and a
// low part, as fdlibm's logf splits it (ln2_hi = 0x3f317180, ln2_lo =
// 0x3717f7d1). Subnormal inputs are scaled by 2^23 first. 0 gives -inf,
// negative or NaN inputs NaN, +inf itself.
MC_HD float mc_log(float x) {
  uint32_t u = mc_f32_bits(x);
  if (!(x == x) || x < 0.0f) return mc_bits_f32(0x7fc00000u);
  if (x == 0.0f) return mc_bits_f32(0xff800000u);
  if (u >= 0x7f800000u) return x;
  int e = 0;
  if (u < 0x00800000u) {
    x = MC_MUL(x, 8388608.0f);  // 2^23, exact
    u = mc_f32_bits(x);
    e = -23;
  }
  e += (int)(u >> 23) - 127;
  uint32_t mu = (u & 0x007fffffu) | 0x3f800000u;  // m in [1, 2)
  if (mu > 0x3fb504f3u) {                           // m > sqrt(2): use m / 2
    mu -= 0x00800000u;
    e += 1;
  }
  const float m = mc_bits_f32(mu);
  const float s = MC_DIV(MC_ADD(m, -1.0f), MC_ADD(m, 1.0f));
  const float z = MC_MUL(s, s);
  float p = 9.09090936183929443359e-02f;             // 1/11
  p = MC_FMA(p, z, 1.11111111938953399658e-01f);     // 1/9
  p = MC_FMA(p, z, 1.42857149243354797363e-01f);     // 1/7
  p = MC_FMA(p, z, 2.00000002980232238770e-01f);     // 1/5
  p = MC_FMA(p, z, 3.33333343267440795898e-01f);     // 1/3
  const float two_s = MC_ADD(s, s);
  const float lm = MC_FMA(MC_MUL(two_s, z), p, two_s);
  const float ef = (float)e;
  const float LN2_HI = 6.9313812256e-01f;  // 0x3f317180
  const float LN2_LO = 9.0580006145e-06f;  // 0x3717f7d1
  return MC_FMA(ef, LN2_HI, MC_FMA(ef, LN2_LO, lm));
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): ten rounds of two 32x32->64 multiplies with the
// round key bumped by the Weyl constants.
MC_HD void mc_philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const unsigned long long p0 = (unsigned long long)0xD2511F53u * c[0];
    const unsigned long long p1 = (unsigned long long)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Philox counter word 2 of the draw ("SAMP").
#define MC_SAMPLE_DOMAIN 0x53414D50u

// The 32-bit uniform word of token `id` for the draw at position `pos`:
// word id % 4 of Philox4x32-10 with counter (id / 4, pos, "SAMP", 0) and key
// (seed mod 2^32, seed / 2^32).
MC_HD uint32_t mc_sample_word(uint32_t id, uint32_t pos, uint32_t seed_lo, uint32_t seed_hi) {
  uint32_t c[4] = {id >> 2, pos, MC_SAMPLE_DOMAIN, 0u};
  mc_philox4x32_10(c, seed_lo, seed_hi);
  return c[id & 3u];
}

// Gumbel(0, 1) from a 32-bit uniform word: V = (x + 0.5) / 2^32, E = -log(1 - V)
// (an Exp(1) variate; for V < 1/64 from the series V + V^2/2 + V^3/3 + V^4/4,
// which keeps full relative precision for the small E whose G wins), G = -log(E).
MC_HD float mc_gumbel(uint32_t x) {
  const float v = MC_MUL(MC_ADD((float)x, 0.5f), 2.3283064365386963e-10f);
  float e;
  if (v < 0.015625f) {
    e = MC_MUL(v, MC_ADD(1.0f, MC_MUL(v, MC_ADD(0.5f, MC_MUL(v, MC_ADD(0.33333334f,
                                                                      MC_MUL(v, 0.25f)))))));
  } else {
    float t = MC_ADD(1.0f, -v);
    if (t < 2.9802322387695312e-08f) t = 2.9802322387695312e-08f;  // 2^-25
    e = -mc_log(t);
  }
  return -mc_log(e);
}

// Orderable 32-bit key of a float (larger key, larger value; -0 folds to +0),
// the high word of mc_argmax_key, and back.
MC_HD uint32_t mc_fkey(float v) {
  uint32_t u = mc_f32_bits(v);
  if ((u << 1) == 0u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
MC_HD float mc_kfloat(uint32_t k) {
  return mc_bits_f32((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Processed logit of the draw: w = pen(v) * inv_temp with pen(v) = v *
// inv_penalty (v > 0) or v * penalty (v <= 0) for seen tokens; -0 folds to +0.
MC_HD float mc_sample_w(float v, bool seen, float inv_temp, float penalty, float inv_penalty) {
  if (seen) v = v > 0.0f ? MC_MUL(v, inv_penalty) : MC_MUL(v, penalty);
  uint32_t u = mc_f32_bits(MC_MUL(v, inv_temp));
  if ((u << 1) == 0u) u = 0u;
  return mc_bits_f32(u);
}
