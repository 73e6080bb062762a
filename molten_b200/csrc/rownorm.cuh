// Row-level add + RMSNorm for hidden = 2048 with 256 threads, shared by the
// norm, token-tail and router kernels.
#pragma once
#include "mc_internal.cuh"

// --------------------------------------------------------- add + RMSNorm row
// Canonical order (oracle or_add_rmsnorm): thread t of 256 owns elements
// 8t..8t+7 (fma chain of squares), warp butterfly, the 8 warp partials added
// in order, inv = 1/sqrt(total/H + eps), n = bf16((h' * inv) * w).
__device__ __forceinline__ void addnorm_row_2048(const uint16_t* __restrict__ h,
                                                 const uint16_t* __restrict__ badd,
                                                 const uint16_t* __restrict__ w, float eps,
                                                 float* hp8, float* n8, float* red) {
  const int t = threadIdx.x;
  const uint4 hv = __ldg(reinterpret_cast<const uint4*>(h) + t);
  uint4 bv = make_uint4(0, 0, 0, 0);
  if (badd) bv = __ldg(reinterpret_cast<const uint4*>(badd) + t);
  const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + t);
  const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
  const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
  const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float hf = mc_bf16_to_f32((uint16_t)(hw[i >> 1] >> (16 * (i & 1))));
    float v = hf;
    if (badd) v = __fadd_rn(hf, mc_bf16_to_f32((uint16_t)(bw[i >> 1] >> (16 * (i & 1)))));
    hp8[i] = mc_round_bf16(v);
    acc = __fmaf_rn(hp8[i], hp8[i], acc);
  }
  acc = mc_warp_butterfly(acc);
  if ((t & 31) == 0) red[t >> 5] = acc;
  __syncthreads();
  float total = red[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) total = __fadd_rn(total, red[j]);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(total, 1.0f / 2048.0f), eps)));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float wf = mc_bf16_to_f32((uint16_t)(ww[i >> 1] >> (16 * (i & 1))));
    n8[i] = mc_round_bf16(__fmul_rn(__fmul_rn(hp8[i], inv), wf));
  }
}

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint4 r;
  r.x = (uint32_t)mc_f32_to_bf16(v[0]) | ((uint32_t)mc_f32_to_bf16(v[1]) << 16);
  r.y = (uint32_t)mc_f32_to_bf16(v[2]) | ((uint32_t)mc_f32_to_bf16(v[3]) << 16);
  r.z = (uint32_t)mc_f32_to_bf16(v[4]) | ((uint32_t)mc_f32_to_bf16(v[5]) << 16);
  r.w = (uint32_t)mc_f32_to_bf16(v[6]) | ((uint32_t)mc_f32_to_bf16(v[7]) << 16);
  return r;
}

