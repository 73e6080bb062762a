// Streaming decode GEMV for large row counts (the Q6 LM head + argmax, tall
// Q4 projections): gemv_quant / gemv_head_argmax (kernels/lfm.rs:112-149,
// 826-848) at batch 1 and K = 2048.
//
// One persistent CTA per SM owns a contiguous range of rows. A producer warp
// streams them through a ring of shared-memory stages with 1-D bulk (TMA)
// copies -- per stage 32 rows of codes, their scales and their biases, three
// contiguous copies -- and 8 compute warps take 4 rows each per stage, so
// every lane's pre-scaled activations (64 registers) serve four rows and the
// four rows' chains interleave. Measured on B200 (Q6 65536 x 2048): 16 warps
// x 1 row 26.1 us, 16 x 2 23.6, 8 x 4 22.0; a two-stage ring (106 KB for
// Q6, 74 KB for Q4) was faster than deeper ones (Q4 32768 x 2048: 11.4 us
// vs 12.6 with 192 KB). Per-row arithmetic is the canonical order of
// gemv_kernel (lane l owns group l, term = fma(s, qx, b * xg), 32-lane
// butterfly, here as a reduce-scatter over the four rows), so outputs are
// bit-identical to it and to the oracle.
//
// The producer starts streaming before the programmatic-dependent-launch
// wait (weights are never written by earlier kernels); the compute warps wait
// before they read x. Every mbarrier wait is bounded; a CTA whose copies did
// not all land waits for them (bounded again) before it exits.
#include <atomic>

#include "gemv_common.cuh"
#include "mc_async.cuh"

namespace {

constexpr int kK = 2048;
constexpr int kMaxStages = 8;
constexpr uint32_t kRingBudget = 110000;  // shared-memory ring: two stages at 8 x 4 rows
constexpr unsigned long long kTimeoutNs = 200000000ull;  // default limit per wait: 200 ms

// CW compute warps take RPW rows each per stage (rows w, w + CW, ...): a
// stage is CW * RPW rows of codes, then their scales, then their biases.
template <int BITS, int CW, int RPW, uint32_t BUDGET = kRingBudget>
struct RingShape {
  static constexpr int kRows = CW * RPW;
  static constexpr int kThreads = (CW + 1) * 32;                 // + the producer warp
  static constexpr uint32_t kCode = kK * BITS / 8;               // code bytes per row
  static constexpr uint32_t kStage = kRows * (kCode + 2 * 64);   // codes + scales + biases
  static constexpr int kStages =
      BUDGET / kStage < kMaxStages ? (int)(BUDGET / kStage) : kMaxStages;
  static constexpr uint32_t kSmem = kStages * kStage;
  static_assert(kStages >= 2, "ring needs two stages");
};

__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long deadline) {
  while (!mc_mbar_test_sleep(bar, parity, 20000u))
    if (mc_globaltimer() > deadline) return false;
  return true;
}

// MODE 0: y[n] = bf16(row n . x). MODE 1: keys[0] = max over rows of the
// argmax key of the bf16-rounded row values (the key must be zero on entry).
template <int BITS, int MODE, int CW, int RPW, uint32_t BUDGET>
__global__ void __launch_bounds__(RingShape<BITS, CW, RPW, BUDGET>::kThreads, 1)
gemv_ring_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                 const uint16_t* __restrict__ biases, const uint16_t* __restrict__ x,
                 uint16_t* __restrict__ y, unsigned long long* __restrict__ keys, int N,
                 unsigned int* __restrict__ status, unsigned long long timeout_ns) {
  using S = RingShape<BITS, CW, RPW, BUDGET>;
  constexpr int kRows = S::kRows;
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ float bv_s[CW];
  __shared__ uint32_t bi_s[CW];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int r0 = (int)(((long)cta * N) / G), r1 = (int)(((long)(cta + 1) * N) / G);
  const int nst = (r1 - r0 + kRows - 1) / kRows;
  if (t == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mc_mbar_init(full + s, 1);
      mc_mbar_init(empty + s, CW);
    }
    mc_fence_barrier_init();
  }
  __syncthreads();
  mc_pdl_launch_dependents();
  const unsigned long long deadline = mc_globaltimer() + timeout_ns;

  if (warp == CW) {
    // ---- producer: stage s goes to slot s % kStages once the compute warps
    // have released the slot's previous use
    bool ok = true;
    if (lane == 0) {
      const uint64_t pol = mc_policy_evict_first();
      for (int s = 0; s < nst; ++s) {
        const int slot = s % S::kStages;
        if (s >= S::kStages && !ring_wait(empty + slot, ((s / S::kStages) - 1) & 1, deadline)) {
          ok = false;
          break;
        }
        const int n0 = r0 + s * kRows, nr = min(kRows, r1 - n0);
        uint8_t* st = sm + (uint32_t)slot * S::kStage;
        mc_mbar_expect_tx(full + slot, (uint32_t)nr * (S::kCode + 128u));
        mc_bulk_g2s(st, codes + (size_t)n0 * S::kCode, (uint32_t)nr * S::kCode, full + slot, pol);
        mc_bulk_g2s(st + kRows * S::kCode, scales + (size_t)n0 * 32, (uint32_t)nr * 64u,
                    full + slot, pol);
        mc_bulk_g2s(st + kRows * (S::kCode + 64u), biases + (size_t)n0 * 32, (uint32_t)nr * 64u,
                    full + slot, pol);
      }
      // every issued copy lands before the CTA exits (immediate unless a
      // compute warp gave up)
      const int first = nst > S::kStages ? nst - S::kStages : 0;
      for (int s = first; s < nst; ++s)
        ok = ring_wait(full + s % S::kStages, (s / S::kStages) & 1, deadline + timeout_ns) && ok;
      if (!ok) atomicOr(status, 1u);
    }
    return;
  }

  // ---- compute warps: x of group `lane`, pre-scaled, once the previous
  // kernel's output is visible
  mc_pdl_wait();
  float2 xs[32];
  const float xg = load_group_x<BITS>(x, lane, xs);
  float best_v = -INFINITY;
  uint32_t best_i = 0;
  for (int s = 0; s < nst; ++s) {
    const int slot = s % S::kStages;
    // warp-uniform answer: the shuffles below need every lane
    if (!__all_sync(0xffffffffu, ring_wait(full + slot, (s / S::kStages) & 1, deadline))) {
      if (lane == 0) atomicOr(status, 2u);
      break;
    }
    const int n0 = r0 + s * kRows, nr = min(kRows, r1 - n0);
    const uint8_t* st = sm + (uint32_t)slot * S::kStage;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + kRows * S::kCode);
    const uint16_t* bi = reinterpret_cast<const uint16_t*>(st + kRows * (S::kCode + 64u));
    // all RPW rows are computed unconditionally, so their chains interleave;
    // a row past the end of a short last stage reads stale bytes of its own
    // stage slot and its result is dropped
    float sum[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp + j * CW;
      const float sv = mc_bf16_to_f32(sc[r * 32 + lane]);
      const float bv = mc_bf16_to_f32(bi[r * 32 + lane]);
      QGroup<BITS> q;
      const uint4* p = reinterpret_cast<const uint4*>(st + r * S::kCode + lane * (BITS * 8));
#pragma unroll
      for (int c = 0; c < BITS / 2; ++c) q.v[c] = p[c];
      sum[j] = __fadd_rn(0.0f, __fmaf_rn(sv, q.qx(xs), __fmul_rn(bv, xg)));
    }
    // the canonical 32-lane butterfly of each row, as a reduce-scatter: the
    // first log2(RPW) steps hand each half (quarter) of the warp one row and
    // exchange one value per lane instead of one per row; every lane still
    // forms the same tree nodes (IEEE addition commutes), so the row sums are
    // bit-identical to mc_warp_butterfly's
    int jr = 0;
    float v;
    if constexpr (RPW == 2) {
      const bool h = lane & 16;
      v = __fadd_rn(h ? sum[1] : sum[0], __shfl_xor_sync(0xffffffffu, h ? sum[0] : sum[1], 16));
      jr = h;
#pragma unroll
      for (int m = 8; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    } else if constexpr (RPW == 4) {
      const bool h = lane & 16, q = lane & 8;
      const float k0 = __fadd_rn(h ? sum[2] : sum[0],
                                 __shfl_xor_sync(0xffffffffu, h ? sum[0] : sum[2], 16));
      const float k1 = __fadd_rn(h ? sum[3] : sum[1],
                                 __shfl_xor_sync(0xffffffffu, h ? sum[1] : sum[3], 16));
      v = __fadd_rn(q ? k1 : k0, __shfl_xor_sync(0xffffffffu, q ? k0 : k1, 8));
      jr = (h ? 2 : 0) + (q ? 1 : 0);
#pragma unroll
      for (int m = 4; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    } else {
      static_assert(RPW == 1, "rows per warp: 1, 2 or 4");
      v = mc_warp_butterfly(sum[0]);
    }
    __syncwarp();
    if (lane == 0) mc_mbar_arrive(empty + slot);
    // lane jr * 32 / RPW holds row jr (every lane of its group has it)
    const int r = warp + jr * CW;
    if (r < nr) {
      const int n = n0 + r;
      if (MODE == 0) {
        if ((lane & (32 / RPW - 1)) == 0) y[n] = mc_f32_to_bf16(v);
      } else {
        const float vr = mc_round_bf16(v);
        if (mc_better(vr, (uint32_t)n, best_v, best_i)) {
          best_v = vr;
          best_i = (uint32_t)n;
        }
      }
    }
  }
  if (MODE == 1) {
    // the lane groups held different rows: fold their bests into lane 0
#pragma unroll
    for (int m = 16; m >= 32 / RPW; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best_v, m);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, best_i, m);
      if (mc_better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if (lane == 0) {
      bv_s[warp] = best_v;
      bi_s[warp] = best_i;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32));
    if (t == 0) {
      float v = bv_s[0];
      uint32_t i = bi_s[0];
      for (int w = 1; w < CW; ++w)
        if (mc_better(bv_s[w], bi_s[w], v, i)) {
          v = bv_s[w];
          i = bi_s[w];
        }
      atomicMax(keys, mc_argmax_key(v, i));
    }
  }
}

__device__ unsigned int g_ring_status;

template <int BITS, int MODE, int CW, int RPW, uint32_t BUDGET = kRingBudget>
int launch_ring(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                unsigned long long* keys) {
  using S = RingShape<BITS, CW, RPW, BUDGET>;
  auto fn = gemv_ring_kernel<BITS, MODE, CW, RPW, BUDGET>;
  // per device: the shared-memory limit raised once, the status word's address
  static std::atomic<bool> ready[64];
  static unsigned int* status_of[64];
  const int dev = ctx->device & 63;
  if ((int)S::kSmem + 4096 > ctx->max_smem_optin) return 1;
  if (!ready[dev].load()) {
    MC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmem));
    MC_CUDA(cudaGetSymbolAddress((void**)&status_of[dev], g_ring_status));
    ready[dev].store(true);
  }
  unsigned int* status = status_of[dev];
  MC_CUDA(mc_launch_pdl(fn, dim3(ctx->num_sms), dim3(S::kThreads), S::kSmem, ctx->stream,
                        reinterpret_cast<const uint8_t*>(w->codes), w->scales, w->biases, x, y,
                        keys, w->out_features, status, mc_wait_limit(ctx, kTimeoutNs)));
  return mc_after_launch("gemv_ring_kernel");
}

// The configuration per bit width: compute warps, rows per warp and stage.
constexpr int kCW4 = 8, kRPW4 = 4;
constexpr int kCW6 = 8, kRPW6 = 4;

}  // namespace

// Used by mc_gemv_quant / mc_gemv_head_argmax (gemv.cu) for batch 1, K = 2048
// and at least two stages of rows per SM. Returns 1 when the shape does not
// qualify (the caller then uses gemv_kernel), else MC_OK or an error code.
int mc_gemv_ring(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                 unsigned long long* keys, int batch, int mode) {
  if (batch != 1 || w->in_features != kK || w->group_size != 64) return 1;
  const int rows = w->bits == 6 ? kCW6 * kRPW6 : kCW4 * kRPW4;
  if (w->out_features < ctx->num_sms * 2 * rows) return 1;
  if (!mc_aligned(w->codes, 16) || !mc_aligned(w->scales, 16) || !mc_aligned(w->biases, 16))
    return 1;
  if (w->bits == 6)
    return mode ? launch_ring<6, 1, kCW6, kRPW6>(ctx, w, x, y, keys)
                : launch_ring<6, 0, kCW6, kRPW6>(ctx, w, x, y, keys);
  return mode ? launch_ring<4, 1, kCW4, kRPW4>(ctx, w, x, y, keys)
              : launch_ring<4, 0, kCW4, kRPW4>(ctx, w, x, y, keys);
}
