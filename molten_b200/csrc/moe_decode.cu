// Decode expert kernels: the gate/up gather GEMV fused with SwiGLU
// (lfm_gemv_q4_gather_act_bf16, lfm.metal:1392-1445) and the down gather GEMV
// fused with the weighted combine (lfm_gemv_q4_gather_down_combine4_bf16,
// lfm.metal:1503-1554).
//
// The expert ids are read on the device, so both kernels can be captured in
// a CUDA graph behind the router without a host round trip. Weights are the
// stacked [E*I][H] (gate, up) and [E*H][I] (down) Q4 matrices; each warp
// streams whole rows with the canonical row order of gemv_common.cuh.
#include "gemv_common.cuh"

namespace {

constexpr int kWarps = 8;

// grid (4 * I/(16*ITER), batch): CTA = (slot, 16*ITER rows); warp = 2 rows
// of gate and up per 16-row tile, ITER tiles one after the other, so the
// token's activations are pre-scaled once per warp for 4*ITER row dots.
template <int ITER>
__global__ void __launch_bounds__(kWarps * 32)
gather_act_kernel(const uint32_t* __restrict__ gc, const uint16_t* __restrict__ gs,
                  const uint16_t* __restrict__ gb, const uint32_t* __restrict__ uc,
                  const uint16_t* __restrict__ us, const uint16_t* __restrict__ ub,
                  const uint16_t* __restrict__ x, const uint32_t* __restrict__ ids,
                  uint16_t* __restrict__ act, int I, int E) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  constexpr int K = 2048, G = 32, R = 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int tiles = I / (16 * ITER);
  const int slot = blockIdx.x / tiles;
  const int base = (blockIdx.x % tiles) * 16 * ITER + warp * R;
  const uint32_t e = ids[4 * b + slot];
  uint16_t* out = act + ((size_t)b * 4 + slot) * I;
  if (e >= (uint32_t)E) {
    // Out-of-range id (corrupt routing): defined zeros, no weight read.
#pragma unroll
    for (int it = 0; it < ITER; ++it)
      if (lane < R) out[base + 16 * it + lane] = 0;
    return;
  }
  float2 xs[1][32];
  float xg[1];
  xg[0] = load_group_x<4>(x + (size_t)b * K, lane, xs[0]);
#pragma unroll 1
  for (int it = 0; it < ITER; ++it) {
    const int i0 = base + 16 * it;
    const uint8_t* rows[2 * R];
    const uint16_t* sc[2 * R];
    const uint16_t* bi[2 * R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const size_t row = (size_t)e * I + i0 + r;
      rows[r] = reinterpret_cast<const uint8_t*>(gc) + row * (K / 2);
      sc[r] = gs + row * G;
      bi[r] = gb + row * G;
      rows[R + r] = reinterpret_cast<const uint8_t*>(uc) + row * (K / 2);
      sc[R + r] = us + row * G;
      bi[R + r] = ub + row * G;
    }
    float sum[2 * R];
    rows_dot<4, 1, 2 * R>(rows, sc, bi, G, lane, xs, xg, sum);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (lane == r) {
        const float g = mc_round_bf16(sum[r]);
        const float u = mc_round_bf16(sum[R + r]);
        const float s = mc_round_bf16(mc_silu(g));
        out[i0 + r] = mc_f32_to_bf16(__fmul_rn(s, u));
      }
    }
  }
}

// grid (H/(8*ITER), batch): CTA = 8*ITER output rows; warp w = slot (w & 3)
// for rows (w >> 2)*4 .. +3 of each 8-row tile, ITER tiles one after the
// other (the slot's act row pre-scaled once per warp); then 8*ITER threads
// combine in rank order.
template <int ITER>
__global__ void __launch_bounds__(kWarps * 32)
down_combine_kernel(const uint32_t* __restrict__ dc, const uint16_t* __restrict__ ds,
                    const uint16_t* __restrict__ db, const uint16_t* __restrict__ act,
                    const uint32_t* __restrict__ ids, const uint16_t* __restrict__ wts,
                    uint16_t* __restrict__ out, int H, int I, int E) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  constexpr int R = 4;
  __shared__ float p[4][8 * ITER];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int slot = warp & 3;
  const int c0 = blockIdx.x * 8 * ITER;
  const int r0 = (warp >> 2) * R;
  const int G = I / 64;
  const uint32_t e = ids[4 * b + slot];
  if (e < (uint32_t)E) {
    float2 xs[1][32];
    float xg[1] = {0.0f};
    if (lane < G) xg[0] = load_group_x<4>(act + ((size_t)b * 4 + slot) * I, lane, xs[0]);
#pragma unroll 1
    for (int it = 0; it < ITER; ++it) {
      const uint8_t* rows[R];
      const uint16_t* sc[R];
      const uint16_t* bi[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const size_t row = (size_t)e * H + c0 + 8 * it + r0 + r;
        rows[r] = reinterpret_cast<const uint8_t*>(dc) + row * (I / 2);
        sc[r] = ds + row * G;
        bi[r] = db + row * G;
      }
      float sum[R];
      rows_dot<4, 1, R>(rows, sc, bi, G, lane, xs, xg, sum);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) p[slot][8 * it + r0 + r] = mc_round_bf16(sum[r]);
      }
    }
  } else if (lane == 0) {
#pragma unroll
    for (int it = 0; it < ITER; ++it)
#pragma unroll
      for (int r = 0; r < R; ++r) p[slot][8 * it + r0 + r] = 0.0f;
  }
  __syncthreads();
  if (threadIdx.x < 8 * ITER) {
    float tot = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r)
      tot = __fadd_rn(tot, mc_round_bf16(__fmul_rn(mc_bf16_to_f32(wts[4 * b + r]),
                                                   p[r][threadIdx.x])));
    out[(size_t)b * H + c0 + threadIdx.x] = mc_f32_to_bf16(tot);
  }
}

}  // namespace

extern "C" int mc_gemv_gather_act(mc_ctx* ctx, const mc_qweights* gate, const mc_qweights* up,
                                  const uint16_t* x, const uint32_t* ids, uint16_t* act,
                                  int n_experts, int batch) {
  MC_REQUIRE(ctx, "gemv_gather_act: null context");
  int rc = mc_check_gemv_weights(gate, "gemv_gather_act gate");
  if (rc) return rc;
  rc = mc_check_gemv_weights(up, "gemv_gather_act up");
  if (rc) return rc;
  MC_REQUIRE(gate->bits == 4 && up->bits == 4, "gemv_gather_act: gate/up must be 4-bit");
  MC_REQUIRE(gate->in_features == 2048 && up->in_features == 2048,
             "gemv_gather_act: hidden must be 2048");
  MC_REQUIRE(n_experts >= 4 && gate->out_features % n_experts == 0 &&
                 up->out_features == gate->out_features,
             "gemv_gather_act: stacked gate/up rows %d not a multiple of n_experts %d",
             gate->out_features, n_experts);
  const int I = gate->out_features / n_experts;
  MC_REQUIRE(I % 16 == 0, "gemv_gather_act: expert width %d must be a multiple of 16", I);
  MC_REQUIRE(x && ids && act && mc_aligned(x, 16), "gemv_gather_act: bad x/ids/act");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_gather_act: batch %d", batch);
  // a warp takes 2 row tiles from batch 4 and 4 from batch 8 (measured best
  // on B200: more tiles amortise the pre-scale, fewer keep the grid filled)
  if (batch >= 8 && I % 64 == 0) {
    const dim3 grid(4 * (I / 64), batch);
    MC_CUDA(mc_launch_pdl(gather_act_kernel<4>, grid, dim3(kWarps * 32), 0, ctx->stream,
                          gate->codes, gate->scales, gate->biases, up->codes, up->scales,
                          up->biases, x, ids, act, I, n_experts));
  } else if (batch >= 4 && I % 32 == 0) {
    const dim3 grid(4 * (I / 32), batch);
    MC_CUDA(mc_launch_pdl(gather_act_kernel<2>, grid, dim3(kWarps * 32), 0, ctx->stream,
                          gate->codes, gate->scales, gate->biases, up->codes, up->scales,
                          up->biases, x, ids, act, I, n_experts));
  } else {
    const dim3 grid(4 * (I / 16), batch);
    MC_CUDA(mc_launch_pdl(gather_act_kernel<1>, grid, dim3(kWarps * 32), 0, ctx->stream,
                          gate->codes, gate->scales, gate->biases, up->codes, up->scales,
                          up->biases, x, ids, act, I, n_experts));
  }
  return mc_after_launch("gather_act_kernel");
}

extern "C" int mc_gemv_gather_down_combine4(mc_ctx* ctx, const mc_qweights* down,
                                            const uint16_t* act, const uint32_t* ids,
                                            const uint16_t* weights, uint16_t* out,
                                            int n_experts, int batch) {
  MC_REQUIRE(ctx, "gemv_gather_down_combine4: null context");
  int rc = mc_check_gemv_weights(down, "gemv_gather_down_combine4");
  if (rc) return rc;
  MC_REQUIRE(down->bits == 4, "gemv_gather_down_combine4: down must be 4-bit");
  const int I = down->in_features;
  MC_REQUIRE(I % 64 == 0 && I <= 2048, "gemv_gather_down_combine4: expert width %d", I);
  MC_REQUIRE(n_experts >= 4 && down->out_features % n_experts == 0,
             "gemv_gather_down_combine4: stacked down rows %d not a multiple of n_experts %d",
             down->out_features, n_experts);
  const int H = down->out_features / n_experts;
  MC_REQUIRE(H % 8 == 0, "gemv_gather_down_combine4: hidden %d must be a multiple of 8", H);
  MC_REQUIRE(act && ids && weights && out && mc_aligned(act, 16),
             "gemv_gather_down_combine4: bad act/ids/weights/out");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_gather_down_combine4: batch %d", batch);
  // two tiles per warp from batch 4 (four: 166 registers, one CTA fewer per
  // SM, measured slower)
  if (batch >= 4 && H % 16 == 0) {
    const dim3 grid(H / 16, batch);
    MC_CUDA(mc_launch_pdl(down_combine_kernel<2>, grid, dim3(kWarps * 32), 0, ctx->stream,
                          down->codes, down->scales, down->biases, act, ids, weights, out, H, I,
                          n_experts));
  } else {
    const dim3 grid(H / 8, batch);
    MC_CUDA(mc_launch_pdl(down_combine_kernel<1>, grid, dim3(kWarps * 32), 0, ctx->stream,
                          down->codes, down->scales, down->biases, act, ids, weights, out, H, I,
                          n_experts));
  }
  return mc_after_launch("down_combine_kernel");
}
