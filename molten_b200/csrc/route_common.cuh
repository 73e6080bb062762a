// Router row dot product and warp top-4, shared by the routing kernels and
// the fused decode layer.
#pragma once
#include "mc_internal.cuh"

// Router logit of one expert row (canonical order, oracle or_router_logits):
// lane l owns k = 256j + 8l + i (j outer, i inner), fma chain from +0, then
// the 32-lane butterfly. n: the normalized row as floats.
template <int DT>
struct RouterRow;

template <>
struct RouterRow<MC_DTYPE_BF16> {
  uint4 w[8];
  __device__ __forceinline__ void load(const void* W, int e, int lane) {
    const uint4* row = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(W) +
                                                      (size_t)e * 2048);
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = __ldg(row + 32 * j + lane);
  }
  __device__ __forceinline__ float dot(const float* n, int lane) const {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t ww[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
      const float4 n0 = *reinterpret_cast<const float4*>(n + 256 * j + 8 * lane);
      const float4 n1 = *reinterpret_cast<const float4*>(n + 256 * j + 8 * lane + 4);
      const float nv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
        acc = __fmaf_rn(mc_bf16_to_f32((uint16_t)(ww[i >> 1] >> (16 * (i & 1)))), nv[i], acc);
    }
    return mc_warp_butterfly(acc);
  }
};

template <>
struct RouterRow<MC_DTYPE_F32> {
  float4 w[16];
  __device__ __forceinline__ void load(const void* W, int e, int lane) {
    const float4* row =
        reinterpret_cast<const float4*>(reinterpret_cast<const float*>(W) + (size_t)e * 2048);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      w[2 * j] = __ldg(row + 64 * j + 2 * lane);
      w[2 * j + 1] = __ldg(row + 64 * j + 2 * lane + 1);
    }
  }
  __device__ __forceinline__ float dot(const float* n, int lane) const {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 n0 = *reinterpret_cast<const float4*>(n + 256 * j + 8 * lane);
      const float4 n1 = *reinterpret_cast<const float4*>(n + 256 * j + 8 * lane + 4);
      const float4 a = w[2 * j], b = w[2 * j + 1];
      acc = __fmaf_rn(a.x, n0.x, acc);
      acc = __fmaf_rn(a.y, n0.y, acc);
      acc = __fmaf_rn(a.z, n0.z, acc);
      acc = __fmaf_rn(a.w, n0.w, acc);
      acc = __fmaf_rn(b.x, n1.x, acc);
      acc = __fmaf_rn(b.y, n1.y, acc);
      acc = __fmaf_rn(b.z, n1.z, acc);
      acc = __fmaf_rn(b.w, n1.w, acc);
    }
    return mc_warp_butterfly(acc);
  }
};

// Orderable 32-bit key of a candidate: a larger value has a larger key, +0
// and -0 share one key (they compare equal), a NaN gets 0 like a used or
// absent entry (never better than a number; -inf maps to 0x007fffff).
__device__ __forceinline__ uint32_t top4_key(float v) {
  if (v != v) return 0u;
  const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Warp top-4 over E <= 64 logits (lane owns experts lane and lane+32), the
// selection and weight rules of oracle or_route_topk: each round takes the
// largest value, the lowest index among equal values, and index 0 when no
// candidate is left. A round is two warp reductions (max of the keys, then
// min of the indices holding it). Results valid in lane 0.
__device__ __forceinline__ void warp_top4(const float* z, int E, int mode, const float* bias,
                                          float route_eps, uint32_t* ids_out,
                                          uint16_t* w_out) {
  const int lane = threadIdx.x & 31;
  float s0 = -INFINITY, s1 = -INFINITY, v0 = -INFINITY, v1 = -INFINITY;
  const bool has0 = lane < E, has1 = lane + 32 < E;
  if (has0) {
    const float zz = z[lane];
    s0 = mode == MC_ROUTE_SOFTMAX_RENORM ? zz : mc_sigmoid(zz);
    v0 = mode == MC_ROUTE_SOFTMAX_RENORM ? zz : __fadd_rn(s0, bias ? bias[lane] : 0.0f);
  }
  if (has1) {
    const float zz = z[lane + 32];
    s1 = mode == MC_ROUTE_SOFTMAX_RENORM ? zz : mc_sigmoid(zz);
    v1 = mode == MC_ROUTE_SOFTMAX_RENORM ? zz : __fadd_rn(s1, bias ? bias[lane + 32] : 0.0f);
  }
  uint32_t k0 = has0 ? top4_key(v0) : 0u, k1 = has1 ? top4_key(v1) : 0u;
  uint32_t ch[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, k0 > k1 ? k0 : k1);
    uint32_t pick = 0u;
    if (m != 0u) {
      const uint32_t cand = k0 == m ? (uint32_t)lane : (k1 == m ? (uint32_t)lane + 32u : 64u);
      pick = __reduce_min_sync(0xffffffffu, cand);
    }
    if (pick == (uint32_t)lane) k0 = 0u;
    if (pick == (uint32_t)lane + 32u) k1 = 0u;
    ch[r] = pick;
  }
  float raw[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float a = __shfl_sync(0xffffffffu, s0, ch[r] & 31);
    const float b = __shfl_sync(0xffffffffu, s1, ch[r] & 31);
    raw[r] = ch[r] < 32 ? a : b;
  }
  // weights: every lane forms the same numerators and denominator (in rank
  // order), lane r < 4 divides for rank r, lane 0 collects
  float num[4], den;
  if (mode == MC_ROUTE_SOFTMAX_RENORM) {
    den = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      num[r] = mc_exp(__fadd_rn(raw[r], -raw[0]));
      den = __fadd_rn(den, num[r]);
    }
  } else {
    den = route_eps;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      num[r] = raw[r];
      den = __fadd_rn(den, raw[r]);
    }
  }
  const float mine = lane == 0 ? num[0] : lane == 1 ? num[1] : lane == 2 ? num[2] : num[3];
  const uint32_t wb = mc_f32_to_bf16(__fdiv_rn(mine, den));
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const uint32_t w = __shfl_sync(0xffffffffu, wb, r);
    if (lane == 0) {
      ids_out[r] = ch[r];
      w_out[r] = (uint16_t)w;
    }
  }
}

