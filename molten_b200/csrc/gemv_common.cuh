// Register-level pieces of the decode GEMVs: turning packed codes into floats
// and the canonical per-group dot product.
//
// Canonical row order (mirrored by oracle/mc_oracle.c row_dot):
//   lane l of a warp owns the 64-code groups g = l, l+32, ...; per group two
//   chains, even codes and odd codes, each acc = fma(q*2^e, x*2^-e, acc) in
//   increasing k; qx = even + odd; term = fma(s, qx, b * xg) with xg the
//   left-to-right sum of the group's 64 activations; the lane's terms are
//   added in increasing g starting from +0; the row sum is the 32-lane xor
//   butterfly. (Reference arithmetic: dot_word_q4 / GEMV_Q4_BODY,
//   lfm.metal:102-139: s*(q.x) + b*(sum x).)
//
// Code -> float without I2F: OR-ing a code that sits at bit e (e+width <= 23)
// into the mantissa of 2^23 gives the float 2^23 + q*2^e; subtracting 2^23 is
// exact. The activation is pre-scaled by 2^-e so the fused product is q*x
// exactly. Two codes per packed f32x2 add/fma (sm_100a FADD2/FFMA2).
#pragma once
#include "mc_internal.cuh"

// 8 codes of one Q4 word against 4 activation pairs (x pre-scaled by E4).
__device__ __forceinline__ void q4_word_fma(uint32_t w, float2 x0, float2 x1, float2 x2,
                                            float2 x3, float2& acc) {
  const float2 neg = make_float2(-MC_MAGIC_F, -MC_MAGIC_F);
  const uint32_t w8 = w >> 8;
  float2 q01 = make_float2(__uint_as_float((w & 0x0000000Fu) | MC_MAGIC),
                           __uint_as_float((w & 0x000000F0u) | MC_MAGIC));
  float2 q23 = make_float2(__uint_as_float((w & 0x00000F00u) | MC_MAGIC),
                           __uint_as_float((w & 0x0000F000u) | MC_MAGIC));
  float2 q45 = make_float2(__uint_as_float((w & 0x000F0000u) | MC_MAGIC),
                           __uint_as_float((w & 0x00F00000u) | MC_MAGIC));
  float2 q67 = make_float2(__uint_as_float((w8 & 0x000F0000u) | MC_MAGIC),
                           __uint_as_float((w8 & 0x00F00000u) | MC_MAGIC));
  q01 = __fadd2_rn(q01, neg);
  q23 = __fadd2_rn(q23, neg);
  q45 = __fadd2_rn(q45, neg);
  q67 = __fadd2_rn(q67, neg);
  acc = __ffma2_rn(q01, x0, acc);
  acc = __ffma2_rn(q23, x1, acc);
  acc = __ffma2_rn(q45, x2, acc);
  acc = __ffma2_rn(q67, x3, acc);
}

// One Q4 group: 8 words (two uint4) against 32 pre-scaled activation pairs.
__device__ __forceinline__ float q4_group_qx(uint4 a, uint4 b, const float2* xs) {
  float2 acc = make_float2(0.0f, 0.0f);
  q4_word_fma(a.x, xs[0], xs[1], xs[2], xs[3], acc);
  q4_word_fma(a.y, xs[4], xs[5], xs[6], xs[7], acc);
  q4_word_fma(a.z, xs[8], xs[9], xs[10], xs[11], acc);
  q4_word_fma(a.w, xs[12], xs[13], xs[14], xs[15], acc);
  q4_word_fma(b.x, xs[16], xs[17], xs[18], xs[19], acc);
  q4_word_fma(b.y, xs[20], xs[21], xs[22], xs[23], acc);
  q4_word_fma(b.z, xs[24], xs[25], xs[26], xs[27], acc);
  q4_word_fma(b.w, xs[28], xs[29], xs[30], xs[31], acc);
  return __fadd_rn(acc.x, acc.y);
}

// One 4-code Q6 packet starting at byte `off` (0..3) of (lo, hi).
template <int OFF>
__device__ __forceinline__ void q6_packet_fma(uint32_t lo, uint32_t hi, float2 x01, float2 x23,
                                              float2& acc) {
  const float2 neg = make_float2(-MC_MAGIC_F, -MC_MAGIC_F);
  constexpr uint32_t selP = (OFF) | ((OFF + 1) << 4) | ((OFF + 2) << 8) | ((OFF + 3) << 12);
  constexpr uint32_t selQ = (OFF + 1) | ((OFF + 2) << 4) | ((OFF + 3) << 8) | ((OFF + 3) << 12);
  const uint32_t P = __byte_perm(lo, hi, selP);
  const uint32_t Q = __byte_perm(lo, hi, selQ);
  float2 c01 = make_float2(__uint_as_float((P & 0x0000003Fu) | MC_MAGIC),
                           __uint_as_float((P & 0x00000FC0u) | MC_MAGIC));
  float2 c23 = make_float2(__uint_as_float((P & 0x0003F000u) | MC_MAGIC),
                           __uint_as_float((Q & 0x0000FC00u) | MC_MAGIC));
  c01 = __fadd2_rn(c01, neg);
  c23 = __fadd2_rn(c23, neg);
  acc = __ffma2_rn(c01, x01, acc);
  acc = __ffma2_rn(c23, x23, acc);
}

// One Q6 group: 48 bytes (three uint4) against 32 pre-scaled activation pairs.
__device__ __forceinline__ float q6_group_qx(uint4 a, uint4 b, uint4 c, const float2* xs) {
  const uint32_t W[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int base = 3 * m;
    const int wi = base >> 2;
    const int wj = wi + 1 < 12 ? wi + 1 : 11;
    switch (base & 3) {
      case 0: q6_packet_fma<0>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      case 1: q6_packet_fma<1>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      case 2: q6_packet_fma<2>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      default: q6_packet_fma<3>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
    }
  }
  return __fadd_rn(acc.x, acc.y);
}

// Scale exponent of code k for the given bit width (matches MC_E4_* / MC_E6_*).
template <int BITS>
__device__ __forceinline__ int code_shift(int k) {
  if (BITS == 4) {
    const int j = k & 7;
    return j < 6 ? 4 * j : (j == 6 ? 16 : 20);
  } else {
    const int j = k & 3;
    return j == 0 ? 0 : (j == 1 ? 6 : (j == 2 ? 12 : 10));
  }
}

// Loads one group's 64 bf16 activations (128 bytes at x + 64*g), writes the
// pre-scaled pairs and returns the group's left-to-right activation sum.
template <int BITS>
__device__ __forceinline__ float load_group_x(const uint16_t* __restrict__ x, int g, float2* xs) {
  const uint4* src = reinterpret_cast<const uint4*>(x + 64 * g);
  float sum = 0.0f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 v = __ldg(src + c);
    const uint32_t wds[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int k0 = 8 * c + 2 * h;
      const float lo = __uint_as_float(wds[h] << 16);
      const float hi = __uint_as_float(wds[h] & 0xffff0000u);
      sum = (k0 == 0) ? lo : __fadd_rn(sum, lo);
      sum = __fadd_rn(sum, hi);
      xs[k0 / 2] = make_float2(__fmul_rn(lo, mc_pow2_neg(code_shift<BITS>(k0))),
                               __fmul_rn(hi, mc_pow2_neg(code_shift<BITS>(k0 + 1))));
    }
  }
  return sum;
}

// Per-group code bytes.
template <int BITS>
struct QGroup;
template <>
struct QGroup<4> {
  uint4 v[2];
  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + 32 * g;
    v[0] = mc_ldg_stream(p);
    v[1] = mc_ldg_stream(p + 16);
  }
  __device__ __forceinline__ float qx(const float2* xs) const { return q4_group_qx(v[0], v[1], xs); }
};
template <>
struct QGroup<6> {
  uint4 v[3];
  __device__ __forceinline__ void load(const uint8_t* row, int g) {
    const uint8_t* p = row + 48 * g;
    v[0] = mc_ldg_stream(p);
    v[1] = mc_ldg_stream(p + 16);
    v[2] = mc_ldg_stream(p + 32);
  }
  __device__ __forceinline__ float qx(const float2* xs) const {
    return q6_group_qx(v[0], v[1], v[2], xs);
  }
};

// Lane-level accumulation of one row (canonical order), returns the
// butterflied row sum (identical in all lanes).
template <int BITS, int GPL, int R>
__device__ __forceinline__ void rows_dot(const uint8_t* const* rows, const uint16_t* const* sc,
                                         const uint16_t* const* bi, int G, int lane,
                                         const float2 (*xs)[32], const float* xg, float* out) {
  QGroup<BITS> q[R][GPL];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      const int g = lane + 32 * j;
      if (g < G) q[r][j].load(rows[r], g);
    }
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    acc[r] = 0.0f;
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      const int g = lane + 32 * j;
      if (g < G) {
        const float s = mc_bf16_to_f32(__ldg(sc[r] + g));
        const float b = mc_bf16_to_f32(__ldg(bi[r] + g));
        const float qx = q[r][j].qx(xs[j]);
        acc[r] = __fadd_rn(acc[r], __fmaf_rn(s, qx, __fmul_rn(b, xg[j])));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) out[r] = mc_warp_butterfly(acc[r]);
}

