// Decode GEMVs: Q4/Q6 projection GEMV (gemv_quant), the fused Q6 head +
// argmax (gemv_head_argmax), the token tail, the two-stage bf16 argmax and the
// add + RMSNorm row kernel.
//
// Layout in HBM: weights stay in MLX's packed form; one warp owns a row at a
// time, lane l reads its group's 32 (Q4) or 48 (Q6) contiguous code bytes
// with 16-byte streaming loads, so a warp's loads cover the row contiguously.
// Each warp keeps R rows in flight for memory-level parallelism. The
// activation row lives in registers (pre-scaled pairs, see gemv_common.cuh).
#include "gemv_common.cuh"
#include "rownorm.cuh"

namespace {

constexpr int kWarps = 8;

template <int BITS>
__host__ __device__ constexpr size_t row_bytes(int K) {
  return (size_t)K * BITS / 8;
}

// y[b][n] = bf16(row n . x[b]); grid.y = batch row.
// MODE 0: store bf16 y. MODE 1: fold argmax over bf16-rounded values into
// keys[b] (head).
template <int BITS, int GPL, int R, int MODE>
__global__ void __launch_bounds__(kWarps * 32)
gemv_kernel(const uint32_t* __restrict__ codes, const uint16_t* __restrict__ scales,
            const uint16_t* __restrict__ biases, const uint16_t* __restrict__ x,
            uint16_t* __restrict__ y, unsigned long long* __restrict__ keys, int N, int K) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int G = K / 64;
  const uint16_t* xb = x + (size_t)b * K;
  // the first rows' codes, scales and biases into L2 while the previous
  // kernel may still run (weights are never written by it), then the wait
  // before x is read
  {
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    const size_t rb = row_bytes<BITS>(K);
    const int lines = (int)(rb / 128);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = row0 + r;
      if (n < N) {
        const uint8_t* row = reinterpret_cast<const uint8_t*>(codes) + (size_t)n * rb;
        for (int l = lane; l < lines; l += 32)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(row + 128 * l));
        if (lane == 0) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(scales + (size_t)n * G));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(biases + (size_t)n * G));
        }
      }
    }
  }
  mc_pdl_launch_dependents();
  mc_pdl_wait();

  float2 xs[GPL][32];
  float xg[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    const int g = lane + 32 * j;
    if (g < G) xg[j] = load_group_x<BITS>(xb, g, xs[j]);
    else xg[j] = 0.0f;
  }

  float best_v = -INFINITY;
  uint32_t best_i = 0;
  const int stride = gridDim.x * kWarps * R;
  for (int row0 = (blockIdx.x * kWarps + warp) * R; row0 < N; row0 += stride) {
    const uint8_t* rows[R];
    const uint16_t* sc[R];
    const uint16_t* bi[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = min(row0 + r, N - 1);
      rows[r] = reinterpret_cast<const uint8_t*>(codes) + (size_t)n * row_bytes<BITS>(K);
      sc[r] = scales + (size_t)n * G;
      bi[r] = biases + (size_t)n * G;
    }
    float sum[R];
    rows_dot<BITS, GPL, R>(rows, sc, bi, G, lane, xs, xg, sum);
    if (MODE == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (lane == r && row0 + r < N) y[(size_t)b * N + row0 + r] = mc_f32_to_bf16(sum[r]);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float v = mc_round_bf16(sum[r]);
        if (row0 + r < N && mc_better(v, (uint32_t)(row0 + r), best_v, best_i)) {
          best_v = v;
          best_i = (uint32_t)(row0 + r);
        }
      }
    }
  }
  if (MODE == 1) {
    __shared__ float sv[kWarps];
    __shared__ uint32_t si[kWarps];
    if (lane == 0) {
      sv[warp] = best_v;
      si[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = sv[0];
      uint32_t i = si[0];
      for (int w = 1; w < kWarps; ++w)
        if (mc_better(sv[w], si[w], v, i)) {
          v = sv[w];
          i = si[w];
        }
      atomicMax(keys + b, mc_argmax_key(v, i));
    }
  }
}

__global__ void __launch_bounds__(256)
add_rmsnorm_kernel(const uint16_t* __restrict__ h, const uint16_t* __restrict__ badd,
                   const uint16_t* __restrict__ w, uint16_t* __restrict__ hout,
                   uint16_t* __restrict__ nout, float eps) {
  __shared__ float red[8];
  const size_t o = (size_t)blockIdx.x * 2048;
  float hp[8], n[8];
  addnorm_row_2048(h + o, badd ? badd + o : nullptr, w, eps, hp, n, red);
  if (hout) reinterpret_cast<uint4*>(hout + o)[threadIdx.x] = pack8_bf16(hp);
  reinterpret_cast<uint4*>(nout + o)[threadIdx.x] = pack8_bf16(n);
}

// Token tail (lfm.metal:1291-1386): key -> token, clear the key, and with an
// embedding table the next input row and its RMSNorm. One CTA per batch row.
__global__ void __launch_bounds__(256)
token_tail_kernel(unsigned long long* __restrict__ keys, uint32_t* __restrict__ out_tok,
                  const uint16_t* __restrict__ embed, int vocab,
                  const uint16_t* __restrict__ norm_w, uint16_t* __restrict__ x_next,
                  uint16_t* __restrict__ normed_next, float eps) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  __shared__ uint32_t tok_s;
  __shared__ float red[8];
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    const unsigned long long key = keys[b];
    const uint32_t tok = mc_key_token(key);
    keys[b] = 0ull;
    out_tok[b] = tok;
    tok_s = tok;
  }
  if (embed == nullptr) return;
  __syncthreads();
  const uint32_t tok = tok_s;
  const size_t o = (size_t)b * 2048;
  if (tok >= (uint32_t)vocab) {
    // No valid token (an all-NaN head): leave defined zeros, read nothing.
    reinterpret_cast<uint4*>(x_next + o)[threadIdx.x] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(normed_next + o)[threadIdx.x] = make_uint4(0, 0, 0, 0);
    return;
  }
  float hp[8], n[8];
  addnorm_row_2048(embed + (size_t)tok * 2048, nullptr, norm_w, eps, hp, n, red);
  reinterpret_cast<uint4*>(x_next + o)[threadIdx.x] = pack8_bf16(hp);
  reinterpret_cast<uint4*>(normed_next + o)[threadIdx.x] = pack8_bf16(n);
}

// Two-stage argmax over stored bf16 logits (lfm.metal:1126-1192); the merge is
// a total order so the partition does not change the result.
__global__ void __launch_bounds__(256)
argmax_bf16_kernel(const uint16_t* __restrict__ logits, int n, uint32_t* __restrict__ out) {
  __shared__ float sv[8];
  __shared__ uint32_t si[8];
  const int b = blockIdx.x;
  const uint16_t* row = logits + (size_t)b * n;
  float bv = -INFINITY;
  uint32_t bi = 0;
  for (int i = threadIdx.x; i < n; i += 256) {
    const float v = mc_bf16_to_f32(row[i]);
    if (mc_better(v, (uint32_t)i, bv, bi)) {
      bv = v;
      bi = (uint32_t)i;
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (mc_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sv[0];
    uint32_t i = si[0];
    for (int w = 1; w < 8; ++w)
      if (mc_better(sv[w], si[w], v, i)) {
        v = sv[w];
        i = si[w];
      }
    out[b] = i;
  }
}

__global__ void eval_math_kernel(int op, const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  float r;
  switch (op) {
    case 0: r = mc_exp(v); break;
    case 1: r = mc_silu(v); break;
    case 2: r = mc_sigmoid(v); break;
    default: r = mc_round_bf16(v); break;
  }
  y[i] = r;
}

template <int BITS, int GPL, int R, int MODE>
int launch_gemv(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                unsigned long long* keys, int batch) {
  const int N = w->out_features, K = w->in_features;
  const int rows_per_cta = kWarps * R;
  int grid = (N + rows_per_cta - 1) / rows_per_cta;
  const int cap = ctx->num_sms * 8;
  if (grid > cap) grid = cap;
  MC_CUDA(mc_launch_pdl(gemv_kernel<BITS, GPL, R, MODE>, dim3(grid, batch), dim3(kWarps * 32), 0,
                        ctx->stream,
      w->codes, w->scales, w->biases, x, y, keys, N, K));
  return mc_after_launch("gemv_kernel");
}

template <int MODE>
int dispatch_gemv(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                  unsigned long long* keys, int batch) {
  const int G = w->in_features / 64;
  // few rows: one row per warp, so every SM gets work (2048 rows at R = 4
  // would fill 64 CTAs)
  const bool few = (long)w->out_features * batch < (long)ctx->num_sms * kWarps * 4;
  if (w->bits == 4) {
    if (G <= 32) {
      if (few) return launch_gemv<4, 1, 1, MODE>(ctx, w, x, y, keys, batch);
      return launch_gemv<4, 1, 4, MODE>(ctx, w, x, y, keys, batch);
    }
    return launch_gemv<4, 2, 2, MODE>(ctx, w, x, y, keys, batch);
  }
  if (G <= 32) {
    if (few) return launch_gemv<6, 1, 1, MODE>(ctx, w, x, y, keys, batch);
    return launch_gemv<6, 1, 2, MODE>(ctx, w, x, y, keys, batch);
  }
  return launch_gemv<6, 2, 1, MODE>(ctx, w, x, y, keys, batch);
}

}  // namespace

extern "C" int mc_gemv_quant(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                             int batch) {
  MC_REQUIRE(ctx, "gemv_quant: null context");
  int rc = mc_check_gemv_weights_k(w, "gemv_quant", 16384);
  if (rc) return rc;
  MC_REQUIRE(x && y, "gemv_quant: null x or y");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_quant: batch %d out of range", batch);
  MC_REQUIRE(mc_aligned(x, 16), "gemv_quant: x must be 16-byte aligned");
  if (w->in_features > 4096) {  // the dense FFN's down projection (K = 11776)
    MC_REQUIRE(w->bits == 4, "gemv_quant: %d-bit rows wider than 4096 are not built", w->bits);
    return mc_gemv_q4_wide(ctx, w, x, y, batch);
  }
  rc = mc_gemv_ring(ctx, w, x, y, nullptr, batch, 0);
  if (rc != 1) return rc;
  rc = mc_gemv_batched(ctx, w, x, y, nullptr, batch, 0);
  if (rc != 1) return rc;
  return dispatch_gemv<0>(ctx, w, x, y, nullptr, batch);
}

extern "C" int mc_gemv_head_argmax(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x,
                                   unsigned long long* keys, int batch) {
  MC_REQUIRE(ctx, "gemv_head_argmax: null context");
  int rc = mc_check_gemv_weights(w, "gemv_head_argmax");
  if (rc) return rc;
  MC_REQUIRE(x && keys, "gemv_head_argmax: null x or keys");
  MC_REQUIRE(mc_aligned(keys, 8), "gemv_head_argmax: keys must be 8-byte aligned");
  MC_REQUIRE(mc_aligned(x, 16), "gemv_head_argmax: x must be 16-byte aligned");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_head_argmax: batch %d out of range", batch);
  rc = mc_gemv_ring(ctx, w, x, nullptr, keys, batch, 1);
  if (rc != 1) return rc;
  rc = mc_gemv_batched(ctx, w, x, nullptr, keys, batch, 1);
  if (rc != 1) return rc;
  return dispatch_gemv<1>(ctx, w, x, nullptr, keys, batch);
}

extern "C" int mc_token_tail(mc_ctx* ctx, unsigned long long* keys, uint32_t* out_tok,
                             const uint16_t* embed, int vocab, const uint16_t* norm_w,
                             uint16_t* x_next, uint16_t* normed_next, int hidden, float eps,
                             int batch) {
  MC_REQUIRE(ctx, "token_tail: null context");
  MC_REQUIRE(keys && out_tok, "token_tail: null keys or out_tok");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "token_tail: batch %d out of range", batch);
  if (embed) {
    MC_REQUIRE(hidden == 2048, "token_tail: hidden must be 2048 (got %d)", hidden);
    MC_REQUIRE(vocab >= 1, "token_tail: vocab %d", vocab);
    MC_REQUIRE(norm_w && x_next && normed_next, "token_tail: null row buffers");
    MC_REQUIRE(mc_aligned(embed, 16) && mc_aligned(norm_w, 16) && mc_aligned(x_next, 16) &&
                   mc_aligned(normed_next, 16),
               "token_tail: row buffers must be 16-byte aligned");
  }
  MC_CUDA(mc_launch_pdl(token_tail_kernel, dim3(batch), dim3(256), 0, ctx->stream, keys, out_tok, embed, vocab, norm_w, x_next,
                                                    normed_next, eps));
  return mc_after_launch("token_tail_kernel");
}

extern "C" int mc_argmax_bf16(mc_ctx* ctx, const uint16_t* logits, int n, uint32_t* out,
                              int batch) {
  MC_REQUIRE(ctx, "argmax_bf16: null context");
  MC_REQUIRE(logits && out, "argmax_bf16: null pointer");
  MC_REQUIRE(n >= 1, "argmax_bf16: n %d", n);
  MC_REQUIRE(batch >= 1 && batch <= 65535, "argmax_bf16: batch %d out of range", batch);
  argmax_bf16_kernel<<<batch, 256, 0, ctx->stream>>>(logits, n, out);
  return mc_after_launch("argmax_bf16_kernel");
}

extern "C" int mc_add_rmsnorm(mc_ctx* ctx, const uint16_t* h, const uint16_t* b, const uint16_t* w,
                              uint16_t* hout, uint16_t* nout, int hidden, float eps, int batch) {
  MC_REQUIRE(ctx, "add_rmsnorm: null context");
  MC_REQUIRE(hidden == 2048, "add_rmsnorm: hidden must be 2048 (got %d)", hidden);
  MC_REQUIRE(h && w && nout, "add_rmsnorm: null pointer");
  MC_REQUIRE(mc_aligned(h, 16) && mc_aligned(w, 16) && mc_aligned(nout, 16) &&
                 (!b || mc_aligned(b, 16)) && (!hout || mc_aligned(hout, 16)),
             "add_rmsnorm: rows must be 16-byte aligned");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "add_rmsnorm: batch %d out of range", batch);
  add_rmsnorm_kernel<<<batch, 256, 0, ctx->stream>>>(h, b, w, hout, nout, eps);
  return mc_after_launch("add_rmsnorm_kernel");
}

extern "C" int mc_eval_math(mc_ctx* ctx, int op, const float* x, float* y, int n) {
  MC_REQUIRE(ctx, "eval_math: null context");
  MC_REQUIRE(x && y && n >= 0, "eval_math: bad arguments");
  MC_REQUIRE(op >= 0 && op <= 3, "eval_math: op %d", op);
  if (n == 0) return MC_OK;
  eval_math_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(op, x, y, n);
  return mc_after_launch("eval_math_kernel");
}

