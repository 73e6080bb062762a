// Register-level pieces of the decode GEMVs: turning packed codes into floats
// and the canonical per-group dot product.
//
// Canonical row order (mirrored by oracle/mc_oracle.c row_dot):
//   lane l of a warp owns the 64-code groups g = l, l+32, ...; a group is
//   four quarters of 16 codes and each quarter p has two chains
//   c = fma(q*2^e, x*2^-e, c) in increasing k, both starting at +0 -- for
//   Q4 the codes of the quarter's even word (bit 3 of k clear) and of its
//   odd word; for Q6 even and odd k --; per parity the quarter chains are
//   combined (c0 + c1) + (c2 + c3), and qx = even + odd (four independent
//   chains of 8 instead of one of 32: the group dot is latency bound);
//   term = fma(s, qx, b * xg) with xg the
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

__device__ __forceinline__ float2 mc_u64_as_float2(uint64_t v) {
  float2 f;
  f.x = __uint_as_float((uint32_t)v);
  f.y = __uint_as_float((uint32_t)(v >> 32));
  return f;
}

// 16 codes of two adjacent Q4 words (wa = word 2m, wb = word 2m+1 of a group)
// against 8 activation pairs xs[j] = (x[16m+j], x[16m+8+j]) pre-scaled by E4.
// Per code pair: two lop3 (mask the code at its bit position, OR the 2^23
// exponent), one f32x2 add (-2^23) and one f32x2 fma into acc (.x takes word
// 2m's codes, .y word 2m+1's, each in increasing k). Codes 5..7 (bits 20..31)
// would reach the exponent, so they are taken from w >> 12. Written as PTX:
// the compiler's own version of the same operations issued ~1.4x slower
// (lop3, f32x2 add and fma each issue at half rate, so the instruction
// count per code is what bounds the decode GEMVs).
__device__ __forceinline__ void q4_wordpair_fma(uint32_t wa, uint32_t wb, const float2* xs,
                                                float2& acc) {
  const unsigned long long NEG = 0xCB000000CB000000ull;  // (-2^23, -2^23)
  const uint32_t MAG = MC_MAGIC;
  const uint32_t sa = wa >> 12, sb = wb >> 12;
  unsigned long long a = *reinterpret_cast<const unsigned long long*>(&acc);
#define MC_Q4_STEP(J, A, B, M)                                                             \
  {                                                                                        \
    uint32_t lo, hi;                                                                       \
    unsigned long long q;                                                                  \
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(lo) : "r"(A), "n"(M), "r"(MAG));           \
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(hi) : "r"(B), "n"(M), "r"(MAG));           \
    asm("mov.b64 %0, {%1, %2};" : "=l"(q) : "r"(lo), "r"(hi));                            \
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(q), "l"(NEG));                          \
    asm("fma.rn.f32x2 %0, %1, %2, %0;"                                                     \
        : "+l"(a)                                                                          \
        : "l"(q), "l"(*reinterpret_cast<const unsigned long long*>(xs + (J))));            \
  }
  MC_Q4_STEP(0, wa, wb, 0xF)
  MC_Q4_STEP(1, wa, wb, 0xF0)
  MC_Q4_STEP(2, wa, wb, 0xF00)
  MC_Q4_STEP(3, wa, wb, 0xF000)
  MC_Q4_STEP(4, wa, wb, 0xF0000)
  MC_Q4_STEP(5, sa, sb, 0xF00)
  MC_Q4_STEP(6, sa, sb, 0xF000)
  MC_Q4_STEP(7, sa, sb, 0xF0000)
#undef MC_Q4_STEP
  acc = *reinterpret_cast<const float2*>(&a);
}

// (c0 + c1) + (c2 + c3) per parity, then even + odd.
__device__ __forceinline__ float quarters_qx(const float2* c) {
  const float2 s = __fadd2_rn(__fadd2_rn(c[0], c[1]), __fadd2_rn(c[2], c[3]));
  return __fadd_rn(s.x, s.y);
}

// One Q4 group: 8 words (two uint4) against 32 pre-scaled activation pairs;
// word pair p is quarter p.
__device__ __forceinline__ float q4_group_qx(uint4 a, uint4 b, const float2* xs) {
  float2 c[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) c[p] = make_float2(0.0f, 0.0f);
  q4_wordpair_fma(a.x, a.y, xs + 0, c[0]);
  q4_wordpair_fma(a.z, a.w, xs + 8, c[1]);
  q4_wordpair_fma(b.x, b.y, xs + 16, c[2]);
  q4_wordpair_fma(b.z, b.w, xs + 24, c[3]);
  return quarters_qx(c);
}

// One 4-code Q6 packet starting at byte OFF (0..3) of (lo, hi): P holds the
// packet's bytes OFF..OFF+3 (codes at bits 0, 6, 12, 18), Q bytes OFF+1..
// (code 3 at bits 10..15, below the exponent); per code one lop3 (mask, OR
// 2^23), per code pair one f32x2 add (-2^23) and one f32x2 fma into acc
// (.x even codes, .y odd codes). Written as PTX for the same reason as
// q4_wordpair_fma.
template <int OFF>
__device__ __forceinline__ void q6_packet_fma(uint32_t lo, uint32_t hi, float2 x01, float2 x23,
                                              float2& acc) {
  const unsigned long long NEG = 0xCB000000CB000000ull;
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
  unsigned long long a = *reinterpret_cast<const unsigned long long*>(&acc), q01, q23;
  asm("mov.b64 %0, {%1, %2};" : "=l"(q01) : "r"(c0), "r"(c1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(q23) : "r"(c2), "r"(c3));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(q01) : "l"(q01), "l"(NEG));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(q23) : "l"(q23), "l"(NEG));
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(a)
      : "l"(q01), "l"(*reinterpret_cast<const unsigned long long*>(&x01)));
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(a)
      : "l"(q23), "l"(*reinterpret_cast<const unsigned long long*>(&x23)));
  acc = *reinterpret_cast<const float2*>(&a);
}

// One Q6 group: 48 bytes (three uint4) against 32 pre-scaled activation pairs.
__device__ __forceinline__ float q6_group_qx(uint4 a, uint4 b, uint4 c, const float2* xs) {
  const uint32_t W[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
  float2 q[4];  // packets 4p..4p+3 (codes 16p..16p+15) are quarter p
#pragma unroll
  for (int p = 0; p < 4; ++p) q[p] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int base = 3 * m;
    const int wi = base >> 2;
    const int wj = wi + 1 < 12 ? wi + 1 : 11;
    float2& acc = q[m >> 2];
    switch (base & 3) {
      case 0: q6_packet_fma<0>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      case 1: q6_packet_fma<1>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      case 2: q6_packet_fma<2>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
      default: q6_packet_fma<3>(W[wi], W[wj], xs[2 * m], xs[2 * m + 1], acc); break;
    }
  }
  return quarters_qx(q);
}

// Scale exponent of code k for the given bit width (matches MC_E4_* / MC_E6_*).
template <int BITS>
__device__ __forceinline__ int code_shift(int k) {
  if (BITS == 4) {
    const int j = k & 7;
    return j < 5 ? 4 * j : 4 * (j - 3);
  } else {
    const int j = k & 3;
    return j == 0 ? 0 : (j == 1 ? 6 : (j == 2 ? 12 : 10));
  }
}

// Pre-scales one group's 64 activations into the pair layout the code
// kernels consume and returns the group's left-to-right activation sum.
// Q4: xs[8m + j] = (x[16m+j], x[16m+8+j]) * 2^-E4[j]; Q6: xs[i] =
// (x[2i], x[2i+1]) * 2^-E6.
template <int BITS>
__device__ __forceinline__ float prescale_group_x(const float* xv, float2* xs) {
  float sum = xv[0];
#pragma unroll
  for (int k = 1; k < 64; ++k) sum = __fadd_rn(sum, xv[k]);
  if (BITS == 4) {
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        xs[8 * m + j] = make_float2(__fmul_rn(xv[16 * m + j], mc_pow2_neg(code_shift<4>(j))),
                                    __fmul_rn(xv[16 * m + 8 + j], mc_pow2_neg(code_shift<4>(j))));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      xs[i] = make_float2(__fmul_rn(xv[2 * i], mc_pow2_neg(code_shift<6>(2 * i))),
                          __fmul_rn(xv[2 * i + 1], mc_pow2_neg(code_shift<6>(2 * i + 1))));
  }
  return sum;
}

// Loads one group's 64 bf16 activations (128 bytes at x + 64*g), writes the
// pre-scaled pairs and returns the group's left-to-right activation sum.
// SRC 0: read-only global (__ldg); 1: global written earlier in the same
// kernel by other CTAs (__ldcg, L2); 2: shared memory holding the row with
// the 16-byte chunks of group g at g*8 + (c ^ (g & 7)) (XOR swizzle: lanes
// reading the same chunk of consecutive groups hit different banks; the
// plain layout is an 8-way conflict that stalls the whole shared-memory pipe).
template <int BITS, int SRC = 0>
__device__ __forceinline__ float load_group_x(const uint16_t* __restrict__ x, int g, float2* xs) {
  const uint4* src = reinterpret_cast<const uint4*>(x + 64 * g);
  float xv[64];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 v = SRC == 0 ? __ldg(src + c) : (SRC == 1 ? __ldcg(src + c) : src[c ^ (g & 7)]);
    const uint32_t wds[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      xv[8 * c + 2 * h] = __uint_as_float(wds[h] << 16);
      xv[8 * c + 2 * h + 1] = __uint_as_float(wds[h] & 0xffff0000u);
    }
  }
  return prescale_group_x<BITS>(xv, xs);
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


// R Q4 rows staged in shared memory (codes, scales, biases contiguous per
// row); one group per lane (K <= 2048); same canonical order as rows_dot.
template <int R>
__device__ __forceinline__ void smem_rows_dot_q4(const uint8_t* const* rows,
                                                 const uint16_t* const* sc,
                                                 const uint16_t* const* bi, int G, int lane,
                                                 const float2* xs, float xg, float* out) {
  uint4 a[R], b[R];
  float s[R], bb[R];
  const bool on = lane < G;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (on) {
      const uint4* p = reinterpret_cast<const uint4*>(rows[r] + 32 * lane);
      a[r] = p[0];
      b[r] = p[1];
      s[r] = mc_bf16_to_f32(sc[r][lane]);
      bb[r] = mc_bf16_to_f32(bi[r][lane]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float acc = 0.0f;
    if (on) acc = __fadd_rn(acc, __fmaf_rn(s[r], q4_group_qx(a[r], b[r], xs), __fmul_rn(bb[r], xg)));
    out[r] = mc_warp_butterfly(acc);
  }
}
