// Routing: the fused residual add + RMSNorm + router GEMV + top-4 of the
// decode step (lfm_router_addnorm_route_f32, lfm.metal:773-854), the unfused
// router GEMV + route_token pair (lfm.metal:417-428, 686-703) and the prefill
// per-token top-4 (lfm_moe_route_batch, lfm.metal:1558-1602).
//
// Fused kernel: grid (E/8, batch), 256 threads. Every CTA recomputes the row
// norm (12 KB of bf16 rows, L2-resident after the first CTA) so no CTA waits
// for another; warp w then computes the logit of expert 8*blockIdx.x + w.
// Each CTA publishes its logits, fences and bumps the batch row's counter;
// the CTA that observes the final count runs the warp top-4 and resets the
// counter -- the reference's last-finisher pattern, with no inter-CTA wait.
#include "mc_internal.cuh"
#include "rownorm.cuh"
#include "route_common.cuh"

namespace {

template <int DT>
__global__ void __launch_bounds__(256)
router_addnorm_route_kernel(const uint16_t* __restrict__ h, const uint16_t* __restrict__ badd,
                            const uint16_t* __restrict__ norm_w, uint16_t* __restrict__ h_out,
                            uint16_t* __restrict__ normed, const void* __restrict__ W,
                            const float* __restrict__ ebias, int mode, float* logits,
                            uint32_t* __restrict__ ids, uint16_t* __restrict__ wts,
                            uint32_t* counter, int E, float eps, float route_eps) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  __shared__ __align__(16) float nrow[2048];
  __shared__ float red[8];
  __shared__ uint32_t last_s;
  __shared__ float zs[64];
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  // Issue this warp's router row before the norm so its latency overlaps.
  RouterRow<DT> rr;
  if (e < E) rr.load(W, e, lane);
  const size_t o = (size_t)b * 2048;
  float hp[8], n[8];
  addnorm_row_2048(h + o, badd ? badd + o : nullptr, norm_w, eps, hp, n, red);
  *reinterpret_cast<float4*>(nrow + 8 * threadIdx.x) = make_float4(n[0], n[1], n[2], n[3]);
  *reinterpret_cast<float4*>(nrow + 8 * threadIdx.x + 4) = make_float4(n[4], n[5], n[6], n[7]);
  if (blockIdx.x == 0) {
    reinterpret_cast<uint4*>(h_out + o)[threadIdx.x] = pack8_bf16(hp);
    reinterpret_cast<uint4*>(normed + o)[threadIdx.x] = pack8_bf16(n);
  }
  __syncthreads();
  if (e < E) {
    const float z = rr.dot(nrow, lane);
    if (lane == 0) {
      logits[(size_t)b * E + e] = z;
      __threadfence();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(counter + b, 1u);
    last_s = (done == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (last_s == 0u) return;
  __threadfence();
  if (warp == 0) {
    for (int i = lane; i < E; i += 32) zs[i] = __ldcg(logits + (size_t)b * E + i);
    __syncwarp();
    warp_top4(zs, E, mode, ebias, route_eps, ids + 4 * b, wts + 4 * b);
    if (lane == 0) counter[b] = 0u;
  }
}

template <int DT>
__global__ void __launch_bounds__(256)
router_gemv_kernel(const void* __restrict__ W, const uint16_t* __restrict__ x,
                   float* __restrict__ logits, int E) {
  __shared__ __align__(16) float nrow[2048];
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + (size_t)b * 2048) + threadIdx.x);
  const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 8; ++i)
    nrow[8 * threadIdx.x + i] = mc_bf16_to_f32((uint16_t)(vw[i >> 1] >> (16 * (i & 1))));
  __syncthreads();
  if (e < E) {
    RouterRow<DT> rr;
    rr.load(W, e, lane);
    const float z = rr.dot(nrow, lane);
    if (lane == 0) logits[(size_t)b * E + e] = z;
  }
}

// One warp per token row of logits.
__global__ void __launch_bounds__(256)
route_rows_kernel(const float* __restrict__ logits, int rows, int E, int mode,
                  const float* __restrict__ ebias, float route_eps, uint32_t* __restrict__ ids,
                  uint16_t* __restrict__ wts) {
  __shared__ float zs[8][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= rows) return;
  for (int i = lane; i < E; i += 32) zs[warp][i] = __ldg(logits + (size_t)t * E + i);
  __syncwarp();
  warp_top4(zs[warp], E, mode, ebias, route_eps, ids + 4 * (size_t)t, wts + 4 * (size_t)t);
}

}  // namespace

extern "C" int mc_router_addnorm_route(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                                       const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                                       const void* router_w, int router_dtype,
                                       const float* expert_bias, int route_mode, float* logits,
                                       uint32_t* ids, uint16_t* weights, uint32_t* counter,
                                       int n_experts, int hidden, float eps, float route_eps,
                                       int batch) {
  MC_REQUIRE(ctx, "router_addnorm_route: null context");
  MC_REQUIRE(hidden == 2048, "router_addnorm_route: hidden must be 2048 (got %d)", hidden);
  MC_REQUIRE(n_experts >= 4 && n_experts <= 64,
             "router_addnorm_route: n_experts must be in [4, 64] (got %d)", n_experts);
  MC_REQUIRE(h && norm_w && h_out && normed && router_w && logits && ids && weights && counter,
             "router_addnorm_route: null pointer");
  MC_REQUIRE(router_dtype == MC_DTYPE_BF16 || router_dtype == MC_DTYPE_F32,
             "router_addnorm_route: router dtype %d", router_dtype);
  MC_REQUIRE(route_mode == MC_ROUTE_SOFTMAX_RENORM || route_mode == MC_ROUTE_SIGMOID_BIAS,
             "router_addnorm_route: route mode %d", route_mode);
  MC_REQUIRE(mc_aligned(h, 16) && (!b || mc_aligned(b, 16)) && mc_aligned(norm_w, 16) &&
                 mc_aligned(h_out, 16) && mc_aligned(normed, 16) && mc_aligned(router_w, 16),
             "router_addnorm_route: rows must be 16-byte aligned");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "router_addnorm_route: batch %d", batch);
  // CTA 0 writes h_out/normed while the other CTAs still read h and b, so the
  // outputs must be other buffers (the reference keeps x and x_alt for this).
  MC_REQUIRE((const void*)h_out != (const void*)h && (const void*)h_out != (const void*)b &&
                 (const void*)normed != (const void*)h && (const void*)normed != (const void*)b,
             "router_addnorm_route: h_out/normed must not alias h or b");
  const dim3 grid((n_experts + 7) / 8, batch);
  if (router_dtype == MC_DTYPE_BF16)
    MC_CUDA(mc_launch_pdl(router_addnorm_route_kernel<MC_DTYPE_BF16>, grid, dim3(256), 0, ctx->stream,
        h, b, norm_w, h_out, normed, router_w, expert_bias, route_mode, logits, ids, weights,
        counter, n_experts, eps, route_eps));
  else
    MC_CUDA(mc_launch_pdl(router_addnorm_route_kernel<MC_DTYPE_F32>, grid, dim3(256), 0, ctx->stream,
        h, b, norm_w, h_out, normed, router_w, expert_bias, route_mode, logits, ids, weights,
        counter, n_experts, eps, route_eps));
  return mc_after_launch("router_addnorm_route_kernel");
}

extern "C" int mc_gemv_router(mc_ctx* ctx, const void* router_w, int router_dtype,
                              const uint16_t* x, float* logits, int n_experts, int hidden,
                              int batch) {
  MC_REQUIRE(ctx, "gemv_router: null context");
  MC_REQUIRE(hidden == 2048, "gemv_router: hidden must be 2048 (got %d)", hidden);
  MC_REQUIRE(n_experts >= 1 && n_experts <= 4096, "gemv_router: n_experts %d", n_experts);
  MC_REQUIRE(router_w && x && logits, "gemv_router: null pointer");
  MC_REQUIRE(router_dtype == MC_DTYPE_BF16 || router_dtype == MC_DTYPE_F32,
             "gemv_router: router dtype %d", router_dtype);
  MC_REQUIRE(mc_aligned(router_w, 16) && mc_aligned(x, 16), "gemv_router: 16-byte alignment");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_router: batch %d", batch);
  const dim3 grid((n_experts + 7) / 8, batch);
  if (router_dtype == MC_DTYPE_BF16)
    router_gemv_kernel<MC_DTYPE_BF16><<<grid, 256, 0, ctx->stream>>>(router_w, x, logits, n_experts);
  else
    router_gemv_kernel<MC_DTYPE_F32><<<grid, 256, 0, ctx->stream>>>(router_w, x, logits, n_experts);
  return mc_after_launch("router_gemv_kernel");
}

static int launch_route_rows(mc_ctx* ctx, const float* logits, int rows, int n_experts,
                             int route_mode, const float* expert_bias, float route_eps,
                             uint32_t* ids, uint16_t* w, const char* what) {
  MC_REQUIRE(ctx, "%s: null context", what);
  MC_REQUIRE(logits && ids && w, "%s: null pointer", what);
  MC_REQUIRE(n_experts >= 4 && n_experts <= 64, "%s: n_experts must be in [4, 64] (got %d)", what,
             n_experts);
  MC_REQUIRE(route_mode == MC_ROUTE_SOFTMAX_RENORM || route_mode == MC_ROUTE_SIGMOID_BIAS,
             "%s: route mode %d", what, route_mode);
  MC_REQUIRE(rows >= 0, "%s: rows %d", what, rows);
  if (rows == 0) return MC_OK;
  route_rows_kernel<<<(rows + 7) / 8, 256, 0, ctx->stream>>>(logits, rows, n_experts, route_mode,
                                                             expert_bias, route_eps, ids, w);
  return mc_after_launch("route_rows_kernel");
}

extern "C" int mc_route_token(mc_ctx* ctx, const float* logits, int n_experts, int route_mode,
                              const float* expert_bias, float route_eps, uint32_t* ids,
                              uint16_t* weights, int batch) {
  return launch_route_rows(ctx, logits, batch, n_experts, route_mode, expert_bias, route_eps, ids,
                           weights, "route_token");
}

extern "C" int mc_moe_route_batch(mc_ctx* ctx, const float* logits, int m, int n_experts,
                                  int route_mode, const float* expert_bias, float route_eps,
                                  uint32_t* ids, uint16_t* gw) {
  return launch_route_rows(ctx, logits, m, n_experts, route_mode, expert_bias, route_eps, ids, gw,
                           "moe_route_batch");
}
