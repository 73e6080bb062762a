// Decode neighbours of the MoE block: Q4 GEMVs with small epilogues, on the
// canonical row order of gemv_common.cuh (bit-identical to the CPU oracle).
//
//  * proj3_gemv_scatter (lfm.metal:1020-1068): the Q, K and V rows of one
//    input row in one launch, V stored straight into the KV cache at `pos`;
//  * conv3_gemv (lfm.metal:1070-1110): the B, C, X rows of each channel of
//    the short-conv input projection and the two-tap conv with its state;
//  * gemv_gu_act (lfm.metal:1447-1498): the dense FFN's gate and up rows and
//    SwiGLU on their bf16-rounded sums;
//  * the wide-input Q4 GEMV (lfm_gemv_q4_bf16_k11776, lfm.metal:169-183,
//    the dense FFN's down projection, K = 11776): the pre-scaled activations
//    live in shared memory instead of registers.
//
// Layout and traffic: one warp owns a task (a few rows whose sums one
// epilogue combines); lane l reads its group's 32 code bytes with 16-byte
// streaming loads, so a warp's loads cover each row contiguously. The
// algorithmic bytes are the weight rows (codes + scales + biases) plus the
// activation row and the outputs; nothing is re-read.
#include "gemv_common.cuh"

namespace {

constexpr int kWarps = 8;

// Row n of a Q4 matrix with K inputs.
struct QRow {
  const uint8_t* codes;
  const uint16_t* sc;
  const uint16_t* bi;
};

__device__ __forceinline__ QRow q4_row(const mc_qweights& w, int n, int K) {
  const int G = K / 64;
  return {reinterpret_cast<const uint8_t*>(w.codes) + (size_t)n * (K / 2),
          w.scales + (size_t)n * G, w.biases + (size_t)n * G};
}

// Sums of R rows (canonical order) against x's pre-scaled groups.
template <int GPL, int R>
__device__ __forceinline__ void task_dot(const QRow* rows, int G, int lane,
                                         const float2 (*xs)[32], const float* xg, float* out) {
  const uint8_t* c[R];
  const uint16_t* s[R];
  const uint16_t* b[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    c[r] = rows[r].codes;
    s[r] = rows[r].sc;
    b[r] = rows[r].bi;
  }
  rows_dot<4, GPL, R>(c, s, b, G, lane, xs, xg, out);
}

// ------------------------------------------------------------ Q / K / V

struct Proj3Args {
  mc_qweights q, k, v;
  const uint16_t* x;
  uint16_t* qo;
  uint16_t* ko;
  uint16_t* vcache;
  int nq, nk, nv, max_seq, pos;
};

__device__ __forceinline__ QRow proj3_row(const Proj3Args& A, int n) {
  if (n < A.nq) return q4_row(A.q, n, 2048);
  if (n < A.nq + A.nk) return q4_row(A.k, n - A.nq, 2048);
  return q4_row(A.v, n - A.nq - A.nk, 2048);
}

template <int R>
__global__ void __launch_bounds__(kWarps * 32) proj3_kernel(const Proj3Args A) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  float2 xs[1][32];
  float xg[1];
  xg[0] = load_group_x<4>(A.x, lane, xs[0]);
  const int N = A.nq + A.nk + A.nv;
  const int stride = gridDim.x * kWarps * R;
  for (int row0 = (blockIdx.x * kWarps + warp) * R; row0 < N; row0 += stride) {
    QRow rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = proj3_row(A, min(row0 + r, N - 1));
    float sum[R];
    task_dot<1, R>(rows, 32, lane, xs, xg, sum);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = row0 + r;
      if (lane != r || n >= N) continue;
      const uint16_t v = mc_f32_to_bf16(sum[r]);
      if (n < A.nq) {
        A.qo[n] = v;
      } else if (n < A.nq + A.nk) {
        A.ko[n - A.nq] = v;
      } else {
        const int i = n - A.nq - A.nk;
        A.vcache[((size_t)(i / 64) * A.max_seq + A.pos) * 64 + (i % 64)] = v;
      }
    }
  }
}

// ------------------------------------------------------------ short conv

struct Conv3Args {
  mc_qweights w;      // [3H][2048]: rows c, H + c, 2H + c are b, c, x of channel c
  const uint16_t* x;
  const uint16_t* taps;   // [H][3]
  const uint16_t* state;  // [2][H]
  uint16_t* out;          // [H]
  uint16_t* new_state;    // [2][H]
  int H;
};

__global__ void __launch_bounds__(kWarps * 32) conv3_kernel(const Conv3Args A) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  float2 xs[1][32];
  float xg[1];
  xg[0] = load_group_x<4>(A.x, lane, xs[0]);
  const int stride = gridDim.x * kWarps;
  for (int ch = blockIdx.x * kWarps + warp; ch < A.H; ch += stride) {
    QRow rows[3] = {q4_row(A.w, ch, 2048), q4_row(A.w, A.H + ch, 2048),
                    q4_row(A.w, 2 * A.H + ch, 2048)};
    float sum[3];
    task_dot<1, 3>(rows, 32, lane, xs, xg, sum);
    if (lane == 0) {
      const float b = mc_round_bf16(sum[0]), c = mc_round_bf16(sum[1]);
      const float xv = mc_round_bf16(sum[2]);
      const uint16_t s1 = A.state[A.H + ch];
      const float v0 = mc_bf16_to_f32(A.state[ch]), v1 = mc_bf16_to_f32(s1);
      const float v2 = mc_round_bf16(__fmul_rn(b, xv));
      const float w0 = mc_bf16_to_f32(A.taps[3 * ch]), w1 = mc_bf16_to_f32(A.taps[3 * ch + 1]);
      const float w2 = mc_bf16_to_f32(A.taps[3 * ch + 2]);
      const float z = __fadd_rn(__fadd_rn(__fmul_rn(w0, v0), __fmul_rn(w1, v1)), __fmul_rn(w2, v2));
      A.out[ch] = mc_f32_to_bf16(__fmul_rn(c, mc_round_bf16(z)));
      A.new_state[A.H + ch] = mc_f32_to_bf16(v2);
      A.new_state[ch] = s1;
    }
  }
}

// ------------------------------------------------------------ dense gate/up

struct GuArgs {
  mc_qweights gate, up;
  const uint16_t* x;  // [B][K]
  uint16_t* act;      // [B][N]
  int N, K;
};

// Two tasks (gate and up rows n, n + 1) per warp iteration: four rows in
// flight. grid.y = batch row.
template <int GPL>
__global__ void __launch_bounds__(kWarps * 32) gu_act_kernel(const GuArgs A) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int G = A.K / 64;
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  float2 xs[GPL][32];
  float xg[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    const int g = lane + 32 * j;
    xg[j] = g < G ? load_group_x<4>(A.x + (size_t)b * A.K, g, xs[j]) : 0.0f;
  }
  const int stride = gridDim.x * kWarps * 2;
  for (int n0 = (blockIdx.x * kWarps + warp) * 2; n0 < A.N; n0 += stride) {
    const int n1 = min(n0 + 1, A.N - 1);
    QRow rows[4] = {q4_row(A.gate, n0, A.K), q4_row(A.up, n0, A.K), q4_row(A.gate, n1, A.K),
                    q4_row(A.up, n1, A.K)};
    float sum[4];
    task_dot<GPL, 4>(rows, G, lane, xs, xg, sum);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (lane != t || n0 + t >= A.N) continue;
      const float sl = mc_round_bf16(mc_silu(mc_round_bf16(sum[2 * t])));
      A.act[(size_t)b * A.N + n0 + t] = mc_f32_to_bf16(__fmul_rn(sl, mc_round_bf16(sum[2 * t + 1])));
    }
  }
}

// ------------------------------------------------------------ wide-input GEMV

// Pre-scaled activation pairs in shared memory, lane-transposed so that the
// 32 lanes reading pair i of their groups 32j + l hit consecutive words:
// pair i of group g at [(g / 32) * 32 + i] * 32 + (g % 32); then the group
// sums xg[G]. One warp per row; lane l takes groups l, l + 32, ... in
// increasing order (the canonical order), all its code loads issued first.
template <int J>
__global__ void __launch_bounds__(kWarps * 32)
gemv_q4_wide_kernel(const uint32_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                    const uint16_t* __restrict__ biases, const uint16_t* __restrict__ x,
                    uint16_t* __restrict__ y, int N, int K) {
  extern __shared__ float2 xs_s[];
  const int G = K / 64;
  float* xg_s = reinterpret_cast<float*>(xs_s + (size_t)J * 32 * 32);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  for (int g = threadIdx.x; g < G; g += kWarps * 32) {
    float2 t[32];
    xg_s[g] = load_group_x<4>(x + (size_t)b * K, g, t);
#pragma unroll
    for (int i = 0; i < 32; ++i) xs_s[((g >> 5) * 32 + i) * 32 + (g & 31)] = t[i];
  }
  __syncthreads();
  const int stride = gridDim.x * kWarps;
  for (int n = blockIdx.x * kWarps + warp; n < N; n += stride) {
    const uint8_t* row = reinterpret_cast<const uint8_t*>(codes) + (size_t)n * (K / 2);
    uint4 qa[J], qb[J];
    float s[J], bb[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int g = lane + 32 * j;
      if (g < G) {
        qa[j] = mc_ldg_stream(row + 32 * g);
        qb[j] = mc_ldg_stream(row + 32 * g + 16);
        s[j] = mc_bf16_to_f32(__ldg(scales + (size_t)n * G + g));
        bb[j] = mc_bf16_to_f32(__ldg(biases + (size_t)n * G + g));
      }
    }
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int g = lane + 32 * j;
      if (g < G) {
        float2 xs[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) xs[i] = xs_s[(j * 32 + i) * 32 + lane];
        const float qx = q4_group_qx(qa[j], qb[j], xs);
        acc = __fadd_rn(acc, __fmaf_rn(s[j], qx, __fmul_rn(bb[j], xg_s[g])));
      }
    }
    const float sum = mc_warp_butterfly(acc);
    if (lane == 0) y[(size_t)b * N + n] = mc_f32_to_bf16(sum);
  }
}

template <int J>
int launch_wide(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y, int batch) {
  const int N = w->out_features, K = w->in_features;
  const size_t smem = (size_t)J * 32 * 32 * sizeof(float2) + (size_t)(K / 64) * sizeof(float);
  auto fn = gemv_q4_wide_kernel<J>;
  MC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int grid = (N + kWarps - 1) / kWarps;
  if (grid > ctx->num_sms * 8) grid = ctx->num_sms * 8;
  MC_CUDA(mc_launch_pdl(fn, dim3(grid, batch), dim3(kWarps * 32), smem, ctx->stream, w->codes,
                        w->scales, w->biases, x, y, N, K));
  return mc_after_launch("gemv_q4_wide_kernel");
}

int check_q4_decode(const mc_qweights* w, int k, const char* what) {
  int rc = mc_check_gemv_weights(w, what);
  if (rc) return rc;
  if (w->bits != 4) return mc_fail(MC_EINVAL, "%s: weights must be 4-bit", what);
  if (w->in_features != k)
    return mc_fail(MC_EINVAL, "%s: in_features %d, expected %d", what, w->in_features, k);
  if (!mc_aligned(w->scales, 2) || !mc_aligned(w->biases, 2))
    return mc_fail(MC_EINVAL, "%s: scales/biases misaligned", what);
  return MC_OK;
}

}  // namespace

// Wide-input Q4 GEMV (4096 < K <= 16384), called by mc_gemv_quant.
int mc_gemv_q4_wide(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                    int batch) {
  const int J = (w->in_features / 64 + 31) / 32;
  switch (J) {
    case 3: return launch_wide<3>(ctx, w, x, y, batch);
    case 4: return launch_wide<4>(ctx, w, x, y, batch);
    case 5: return launch_wide<5>(ctx, w, x, y, batch);
    case 6: return launch_wide<6>(ctx, w, x, y, batch);
    case 7: return launch_wide<7>(ctx, w, x, y, batch);
    case 8: return launch_wide<8>(ctx, w, x, y, batch);
    default:
      return mc_fail(MC_EUNSUPPORTED, "gemv_quant: in_features %d not built", w->in_features);
  }
}

extern "C" int mc_proj3_gemv_scatter(mc_ctx* ctx, const mc_qweights* q, const mc_qweights* k,
                                     const mc_qweights* v, const uint16_t* x, uint16_t* q_out,
                                     uint16_t* k_out, uint16_t* v_cache, int max_seq, int pos) {
  MC_REQUIRE(ctx, "proj3_gemv_scatter: null context");
  int rc;
  if ((rc = check_q4_decode(q, 2048, "proj3_gemv_scatter q"))) return rc;
  if ((rc = check_q4_decode(k, 2048, "proj3_gemv_scatter k"))) return rc;
  if ((rc = check_q4_decode(v, 2048, "proj3_gemv_scatter v"))) return rc;
  MC_REQUIRE(x && q_out && k_out && v_cache, "proj3_gemv_scatter: null pointer");
  MC_REQUIRE(mc_aligned(x, 16), "proj3_gemv_scatter: x must be 16-byte aligned");
  MC_REQUIRE(v->out_features % 64 == 0, "proj3_gemv_scatter: nv %d not a multiple of 64",
             v->out_features);
  MC_REQUIRE(max_seq >= 1 && pos >= 0 && pos < max_seq,
             "proj3_gemv_scatter: pos %d outside the cache of %d", pos, max_seq);
  Proj3Args A{*q, *k, *v, x, q_out, k_out, v_cache,
              q->out_features, k->out_features, v->out_features, max_seq, pos};
  const int N = A.nq + A.nk + A.nv;
  // one row per warp when the three matrices are small (every SM busy)
  const bool few = N < ctx->num_sms * kWarps * 2;
  if (few) {
    MC_CUDA(mc_launch_pdl(proj3_kernel<1>, dim3((N + kWarps - 1) / kWarps), dim3(kWarps * 32), 0,
                          ctx->stream, A));
  } else {
    int grid = (N + 2 * kWarps - 1) / (2 * kWarps);
    if (grid > ctx->num_sms * 8) grid = ctx->num_sms * 8;
    MC_CUDA(mc_launch_pdl(proj3_kernel<2>, dim3(grid), dim3(kWarps * 32), 0, ctx->stream, A));
  }
  return mc_after_launch("proj3_kernel");
}

extern "C" int mc_conv3_gemv(mc_ctx* ctx, const mc_qweights* w_proj, const uint16_t* x,
                             const uint16_t* taps, const uint16_t* state, uint16_t* out,
                             uint16_t* new_state, int channels) {
  MC_REQUIRE(ctx, "conv3_gemv: null context");
  int rc;
  if ((rc = check_q4_decode(w_proj, 2048, "conv3_gemv projection"))) return rc;
  MC_REQUIRE(channels >= 1 && w_proj->out_features == 3 * channels,
             "conv3_gemv: projection rows %d != 3 x %d channels", w_proj->out_features, channels);
  MC_REQUIRE(x && taps && state && out && new_state, "conv3_gemv: null pointer");
  MC_REQUIRE(mc_aligned(x, 16), "conv3_gemv: x must be 16-byte aligned");
  MC_REQUIRE(state != new_state, "conv3_gemv: new_state must not alias state");
  Conv3Args A{*w_proj, x, taps, state, out, new_state, channels};
  int grid = (channels + kWarps - 1) / kWarps;
  if (grid > ctx->num_sms * 8) grid = ctx->num_sms * 8;
  MC_CUDA(mc_launch_pdl(conv3_kernel, dim3(grid), dim3(kWarps * 32), 0, ctx->stream, A));
  return mc_after_launch("conv3_kernel");
}

extern "C" int mc_gemv_gu_act(mc_ctx* ctx, const mc_qweights* gate, const mc_qweights* up,
                              const uint16_t* x, uint16_t* act, int batch) {
  MC_REQUIRE(ctx, "gemv_gu_act: null context");
  int rc;
  if ((rc = mc_check_gemv_weights(gate, "gemv_gu_act gate"))) return rc;
  if ((rc = mc_check_gemv_weights(up, "gemv_gu_act up"))) return rc;
  MC_REQUIRE(gate->bits == 4 && up->bits == 4, "gemv_gu_act: dense gate/up must be 4-bit");
  MC_REQUIRE(up->out_features == gate->out_features && up->in_features == gate->in_features &&
                 up->group_size == gate->group_size,
             "gemv_gu_act: dense gate/up shapes");
  MC_REQUIRE(gate->in_features <= 4096, "gemv_gu_act: in_features %d > 4096",
             gate->in_features);
  MC_REQUIRE(x && act, "gemv_gu_act: null pointer");
  MC_REQUIRE(mc_aligned(x, 16), "gemv_gu_act: x must be 16-byte aligned");
  MC_REQUIRE(batch >= 1 && batch <= 65535, "gemv_gu_act: batch %d out of range", batch);
  GuArgs A{*gate, *up, x, act, gate->out_features, gate->in_features};
  const int N = A.N;
  int grid = (N + 2 * kWarps - 1) / (2 * kWarps);
  if (grid > ctx->num_sms * 8) grid = ctx->num_sms * 8;
  if (A.K <= 2048) {
    MC_CUDA(mc_launch_pdl(gu_act_kernel<1>, dim3(grid, batch), dim3(kWarps * 32), 0, ctx->stream,
                          A));
  } else {
    MC_CUDA(mc_launch_pdl(gu_act_kernel<2>, dim3(grid, batch), dim3(kWarps * 32), 0, ctx->stream,
                          A));
  }
  return mc_after_launch("gu_act_kernel");
}
