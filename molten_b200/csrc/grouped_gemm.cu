// Prefill grouped expert GEMM on the 5th-generation tensor cores
// (gemm_q4_grouped_mlx / _gu, quant.rs:146-266 -> lfm_qmm_t_body,
// quant_nax.metal:4091-4234).
//
//   C[i][n] = sum_k A[i][k] * bf16(s*q + b)[e*N + n][k]
//
// for the sorted rows i of each row chunk (m0, m_end, expert e); A bf16
// [rows][K] (the expert-sorted activations), W the stacked [E*N][K] MLX Q4
// matrix. The gate/up variant computes both GEMMs of a chunk against the same
// A rows and writes act = bf16(bf16(silu(bf16(g))) * bf16(u)) in the
// epilogue (silu_mul_bf16, elementwise.metal:7-15).
//
// The MMA runs "weights x tokens": the dequantised 128-feature weight block
// is the M = 128 operand and the chunk's token rows are the N operand, with
// N = the chunk height rounded up to 16 (at most 256), so one dequantised
// weight tile serves up to 256 tokens and small experts do not pay for
// padding rows. D (TMEM) is [128 features][N tokens] fp32.
//
// Persistent kernel, one CTA per SM, work items = (row chunk, 128-feature
// block) in chunk-major order so neighbouring CTAs share a chunk's token rows
// in L2. Warp roles (320 threads):
//   warp 0      TMA: 64-row x 64-K bf16 boxes of the chunk's token rows,
//               128-byte swizzle, into the stage ring
//   warp 1      TMEM allocation (512 columns); lane 0 issues tcgen05.mma
//               (M=128, N=chunk, K=16, bf16 x bf16 -> fp32) and commits
//   warps 2..9  dequantise the weight tiles straight into the UMMA K-major
//               128-byte-swizzled layout (w = bf16(fma(s, q, b)), MLX's
//               dequantize): gate/up: warps 2-5 gate, 6-9 up; down: warps
//               2-5 even K steps, 6-9 odd ones. Then the epilogue from TMEM.
// Two rings: token rows (bfull: TMA tx, bempty: tcgen05.commit) and weight
// tiles (afull: dequant arrivals, aempty: tcgen05.commit).
// Every wait is bounded by a %globaltimer deadline; on timeout the kernel
// records status bit 1, stops issuing and still drains what it issued before
// freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include "mc_internal.cuh"
#include "mc_async.cuh"

namespace {

constexpr int BF = 128;    // weight features per item (the MMA's M)
constexpr int BK = 64;     // K per stage
constexpr int MAXN = 256;  // token rows per chunk (the MMA's N, rounded up to 16)
constexpr int BOX_ROWS = 64;
constexpr int BOX_BYTES = BOX_ROWS * BK * 2;  // 8 KB token box
constexpr int kDeqThreads = 256;
constexpr int kThreads = 64 + kDeqThreads;
constexpr unsigned long long kTimeoutNs = 1000000000ull;  // 1 s per wait

template <bool GU>
struct Cfg {
  static constexpr int NMAT = GU ? 2 : 1;
  static constexpr int B_BYTES = MAXN * BK * 2;        // 32 KB of token rows per K step
  static constexpr int A_BYTES = BF * BK * 2;          // 16 KB per weight matrix per K step
  static constexpr int A_STAGE = NMAT * A_BYTES;
  // Token rows come by TMA from L2/HBM (microseconds away): a deep ring. The
  // weight tiles are produced on chip by the dequant warps: a short one.
  static constexpr int BSTAGES = GU ? 3 : 4;
  static constexpr int ASTAGES = GU ? 3 : 4;
  static constexpr int SMEM = BSTAGES * B_BYTES + ASTAGES * A_STAGE + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int NBUF = GU ? 1 : 2;  // accumulator buffers (gate+up fill TMEM)
  // dequant arrivals per stage: gate/up both groups, down one group
  static constexpr uint32_t DEQ_ARRIVALS = GU ? 256u : 128u;
};
static_assert(Cfg<true>::SMEM + 512 <= 232448 && Cfg<false>::SMEM + 512 <= 232448,
              "shared memory budget");

struct GemmParams {
  mc_qweights w0, w1;
  uint16_t* out;
  const uint4* tiles;
  const uint32_t* n_tiles;
  uint32_t* status;
  int N, K, rows, max_tiles, n_experts;
};

// One work item: token rows [m0, mend) of expert e against feature block nb.
struct Item {
  uint32_t m0, mend, e;
  int nb, n;  // n = MMA N (rows rounded up to 16)
  bool ok;
};

__device__ __forceinline__ Item item_info(const GemmParams& P, int item, int nblk) {
  const uint4 tile = P.tiles[item / nblk];
  Item it;
  it.nb = item % nblk;
  it.ok = tile.z < (uint32_t)P.n_experts && tile.x < tile.y && tile.y <= (uint32_t)P.rows &&
          tile.y - tile.x <= (uint32_t)MAXN;
  // a malformed tile still runs through the pipeline (every role sees the same
  // shape) on row 0 of expert 0, and its results are not stored
  it.m0 = it.ok ? tile.x : 0u;
  it.mend = it.ok ? tile.y : 1u;
  it.e = it.ok ? tile.z : 0u;
  it.n = (int)((it.mend - it.m0 + 15u) & ~15u);
  return it;
}

// ---- PTX wrappers -----------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(mc_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mc_smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO = 1024), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D f32, A/B bf16, both K-major, M = BF; N per item.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BF >> 4) << 24);
__device__ __forceinline__ uint32_t idesc_for(int n) { return kIdescBase | ((uint32_t)(n >> 3) << 17); }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          mc_smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Bounded mbarrier wait that also gives up when another role aborted. The
// clock is read only once the barrier was found incomplete.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_f) {
  if (mc_mbar_test_sleep(bar, parity, 20000u)) return true;
  const unsigned long long deadline = mc_globaltimer() + kTimeoutNs;
  while (!mc_mbar_test_sleep(bar, parity, 20000u)) {
    if (*abort_f) return false;
    if (mc_globaltimer() > deadline) return false;
  }
  return true;
}

// ---- epilogue arithmetic ------------------------------------------------------
// Single-value float->bf16 conversions and MUFU exp/rcp each issue at about
// 16 per clock per SM, so the epilogue rounds with integer ops (round to
// nearest even on the bit pattern; inputs are finite), takes one MUFU per
// element for the sigmoid, and converts the outputs two at a time.
__device__ __forceinline__ float bf16_round(float x) {
  uint32_t u = __float_as_uint(x);
  u += 0x7fffu + ((u >> 16) & 1u);
  return __uint_as_float(u & 0xffff0000u);
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// silu(g) = g * sigmoid(g), sigmoid(g) = 0.5 + 0.5 * tanh(g / 2): the prefill
// activations are compared within the bf16 tolerance (the tensor cores'
// summation order is unspecified anyway), so the decode path's bit-exact
// exponential is not needed here.
__device__ __forceinline__ float silu_fast(float g) {
  return __fmul_rn(g, __fmaf_rn(0.5f, tanh_approx(__fmul_rn(0.5f, g)), 0.5f));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&t);
}

// ---- dequantisation of one 64-wide K slice of one weight row ----------------
// 8 Q4 words (64 codes, k = 16m + j in the order of the word pairs) ->
// 64 bf16 values in natural k order, stored as 8 16-byte chunks at
// row_base + ((c ^ swz) * 16): the UMMA K-major 128B-swizzle layout.
// w = bf16(fma(s, q, b)) with s*q exact (MLX dequantize, quant_nax.metal:2947).
__device__ __forceinline__ void dequant_row64(uint4 a, uint4 b, float s, float bias,
                                              uint8_t* row_base, int swz) {
  const uint32_t W[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float v[64];
  const float2 neg = make_float2(-MC_MAGIC_F, -MC_MAGIC_F);
  const float2 bb = make_float2(bias, bias);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t wa = W[2 * m], wb = W[2 * m + 1];
    const uint64_t Wd = ((uint64_t)wb << 32) | wa;
    const uint64_t Sd = ((uint64_t)(wb >> 12) << 32) | (wa >> 12);
    const uint64_t MAG = 0x4B0000004B000000ull;
    const uint64_t masked[8] = {Wd & 0x0000000F0000000Full, Wd & 0x000000F0000000F0ull,
                                Wd & 0x00000F0000000F00ull, Wd & 0x0000F0000000F000ull,
                                Wd & 0x000F0000000F0000ull, Sd & 0x00000F0000000F00ull,
                                Sd & 0x0000F0000000F000ull, Sd & 0x000F0000000F0000ull};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = j < 5 ? 4 * j : 4 * (j - 3);
      const float se = __fmul_rn(s, mc_pow2_neg(e));  // exact for |s| >= 2^-110
      const uint64_t qb = masked[j] | MAG;
      float2 q = make_float2(__uint_as_float((uint32_t)qb), __uint_as_float((uint32_t)(qb >> 32)));
      q = __fadd2_rn(q, neg);                              // (q_k, q_{k+8}) * 2^e, exact
      const float2 w = __ffma2_rn(q, make_float2(se, se), bb);  // s*q + b, one rounding
      v[16 * m + j] = w.x;
      v[16 * m + 8 + j] = w.y;
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t p[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const __nv_bfloat162 t = __floats2bfloat162_rn(v[8 * c + 2 * h], v[8 * c + 2 * h + 1]);
      p[h] = *reinterpret_cast<const uint32_t*>(&t);
    }
    *reinterpret_cast<uint4*>(row_base + ((c ^ swz) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
  }
}

template <bool GU>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const GemmParams P) {
  using C = Cfg<GU>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bfull[C::BSTAGES], bempty[C::BSTAGES];
  __shared__ __align__(8) uint64_t afull[C::ASTAGES], aempty[C::ASTAGES];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile uint32_t abort_s;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

  if (t == 0) {
    for (int s = 0; s < C::BSTAGES; ++s) {
      mc_mbar_init(&bfull[s], 1);
      mc_mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < C::ASTAGES; ++s) {
      mc_mbar_init(&afull[s], C::DEQ_ARRIVALS);
      mc_mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mc_mbar_init(&acc_full[b], 1);
      mc_mbar_init(&acc_empty[b], kDeqThreads);
    }
    mc_mbar_init(&drain_bar, 1);
    mc_fence_barrier_init();
    abort_s = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     mc_smem_u32(&tmem_base_s)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  const int nblk = P.N / BF;
  const int ksteps = P.K / BK;
  int ntiles = (int)*P.n_tiles;
  if (ntiles > P.max_tiles) ntiles = P.max_tiles;
  const int total = ntiles * nblk;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x) {
        const Item w = item_info(P, item, nblk);
        int nbox = (w.n + BOX_ROWS - 1) / BOX_ROWS;
        // boxes that start past the last row would only read fill values
        const int rows_left = P.rows - (int)w.m0;
        if (nbox * BOX_ROWS > rows_left + BOX_ROWS - 1) nbox = (rows_left + BOX_ROWS - 1) / BOX_ROWS;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % C::BSTAGES;
          const uint32_t ph = (it / C::BSTAGES) & 1;
          if (!wait_bar(&bempty[s], ph ^ 1, &abort_s)) {
            abort_s = 1;
            break;
          }
          mc_mbar_expect_tx(&bfull[s], (uint32_t)(nbox * BOX_BYTES));
          for (int bx = 0; bx < nbox; ++bx)
            tma_load_2d(smem + s * C::B_BYTES + bx * BOX_BYTES, &tmA, kk * BK,
                        (int)w.m0 + bx * BOX_ROWS, &bfull[s]);
        }
      }
      if (abort_s) {
        // loads already issued finish within microseconds; give them a bounded
        // time to land before the CTA may leave
        for (int k = 0; k < 200; ++k) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, j = 0;
      for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x, ++j) {
        const Item w = item_info(P, item, nblk);
        const uint32_t idesc = idesc_for(w.n);
        const int buf = (int)(j % C::NBUF);
        const uint32_t use = j / C::NBUF;
        if (!wait_bar(&acc_empty[buf], (use & 1) ^ 1, &abort_s)) {
          abort_s = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * 256);
        bool ok = true;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int sb = it % C::BSTAGES, sa = it % C::ASTAGES;
          if (!wait_bar(&bfull[sb], (it / C::BSTAGES) & 1, &abort_s) ||
              !wait_bar(&afull[sa], (it / C::ASTAGES) & 1, &abort_s)) {
            abort_s = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sw128_desc(mc_smem_u32(smem + sb * C::B_BYTES));
          const uint32_t abase = mc_smem_u32(smem + C::BSTAGES * C::B_BYTES + sa * C::A_STAGE);
          const uint64_t adesc0 = sw128_desc(abase);
          const uint64_t adesc1 = sw128_desc(abase + C::A_BYTES);
#pragma unroll
          for (int k16 = 0; k16 < BK / 16; ++k16) {
            const uint32_t acc = (kk > 0 || k16 > 0) ? 1u : 0u;
            umma_bf16(d0, adesc0 + 2 * k16, bdesc + 2 * k16, idesc, acc);
            if (GU) umma_bf16(d0 + 256, adesc1 + 2 * k16, bdesc + 2 * k16, idesc, acc);
          }
          umma_commit(&bempty[sb]);  // both stages free once these MMAs have read them
          umma_commit(&aempty[sa]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------ dequant producers + epilogue
    const int dt = t - 64;            // 0..255
    const int grp = dt >> 7;          // gate/up: matrix; down: K-step parity
    const int d = dt & 127;           // weight row within the feature block
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const uint32_t* wcodes = (GU && grp) ? P.w1.codes : P.w0.codes;
    const uint16_t* wscales = (GU && grp) ? P.w1.scales : P.w0.scales;
    const uint16_t* wbiases = (GU && grp) ? P.w1.biases : P.w0.biases;
    // K steps of this thread: all (gate/up) or every other one (down)
    const int step = GU ? 1 : 2;
    // two K slices in flight per thread: slot 0 holds the slice being
    // dequantised while slot 1's loads are outstanding, then they swap; the
    // next item's first two slices are requested before this item's epilogue
    // (scale and bias stay raw bf16 until use: converting them at load time
    // would make the thread wait for the load right there)
    uint4 ca0 = make_uint4(0, 0, 0, 0), cb0 = ca0, ca1 = ca0, cb1 = ca0;
    uint16_t sc0 = 0, bi0 = 0, sc1 = 0, bi1 = 0;
    const uint8_t* crow = nullptr;
    const uint16_t *srow = nullptr, *brow = nullptr;
    auto load_slice = [&](int kk, uint4& ca, uint4& cb, uint16_t& sc, uint16_t& bi) {
      if (kk < ksteps) {
        ca = __ldg(reinterpret_cast<const uint4*>(crow + kk * 32));
        cb = __ldg(reinterpret_cast<const uint4*>(crow + kk * 32) + 1);
        sc = __ldg(srow + kk);
        bi = __ldg(brow + kk);
      }
    };
    // point at item `item`'s weight row and request its first two slices
    auto start_item = [&](int item, uint32_t it_base) -> Item {
      const Item w = item_info(P, item, nblk);
      const size_t wrow = (size_t)w.e * P.N + (size_t)w.nb * BF + d;
      crow = reinterpret_cast<const uint8_t*>(wcodes) + wrow * (P.K / 2);
      srow = wscales + wrow * (P.K / 64);
      brow = wbiases + wrow * (P.K / 64);
      const int k0 = GU ? 0 : (int)((grp - it_base) & 1u);
      load_slice(k0, ca0, cb0, sc0, bi0);
      load_slice(k0 + step, ca1, cb1, sc1, bi1);
      return w;
    };
    uint32_t it = 0, j = 0;
    Item w = start_item(blockIdx.x < total ? blockIdx.x : 0, 0);
    for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x, ++j) {
      if (!w.ok && dt == 0 && P.status) atomicOr(P.status, 2u);
      const int k0 = GU ? 0 : (int)((grp - it) & 1u);
      bool ok = true;
      auto do_slice = [&](int kk, uint4& ca, uint4& cb, uint16_t& sc, uint16_t& bi) -> bool {
        const uint4 xa = ca, xb = cb;
        const uint16_t xs = sc, xbias = bi;
        load_slice(kk + 2 * step, ca, cb, sc, bi);  // refill this slot two slices ahead
        const uint32_t itk = it + (uint32_t)kk;
        const int s = itk % C::ASTAGES;
        const uint32_t ph = (itk / C::ASTAGES) & 1;
        if (!wait_bar(&aempty[s], ph ^ 1, &abort_s)) return false;
        uint8_t* at = smem + C::BSTAGES * C::B_BYTES + s * C::A_STAGE + (GU ? grp * C::A_BYTES : 0);
        dequant_row64(xa, xb, mc_bf16_to_f32(xs), mc_bf16_to_f32(xbias), at + d * 128, d & 7);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mc_mbar_arrive(&afull[s]);
        return true;
      };
      for (int kk = k0; kk < ksteps; kk += 2 * step) {
        if (!do_slice(kk, ca0, cb0, sc0, bi0)) {
          ok = false;
          break;
        }
        if (kk + step < ksteps && !do_slice(kk + step, ca1, cb1, sc1, bi1)) {
          ok = false;
          break;
        }
      }
      if (!ok) abort_s = 1;
      it += (uint32_t)ksteps;
      if (!ok) break;
      const Item cur = w;
      if (item + (int)gridDim.x < total) w = start_item(item + gridDim.x, it);
      // ---- epilogue: TMEM [feature][token] -> bf16 out[token][feature]
      const int buf = (int)(j % C::NBUF);
      const uint32_t use = j / C::NBUF;
      if (!wait_bar(&acc_full[buf], use & 1, &abort_s)) {
        abort_s = 1;
        break;
      }
      tc_fence_after();
      const int f = 32 * q + lane;  // feature row of D this thread reads
      const int n16 = cur.n >> 4, split = (n16 + 1) >> 1;
      const int c_lo = grp ? split : 0, c_hi = grp ? n16 : split;
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * 256);
      uint16_t* ocol = P.out + (size_t)cur.nb * BF + f;
#pragma unroll 1
      for (int c = c_lo; c < c_hi; ++c) {
        uint32_t g[16], u[16];
        tmem_ld16(lane_base + 16 * c, g);
        if (GU) tmem_ld16(lane_base + 256 + 16 * c, u);
        tmem_wait_ld();
        const uint32_t r0 = cur.m0 + 16u * (uint32_t)c;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float o0, o1;
          if (GU) {
            const float g0 = bf16_round(__uint_as_float(g[i])), g1 = bf16_round(__uint_as_float(g[i + 1]));
            const float u0 = bf16_round(__uint_as_float(u[i])), u1 = bf16_round(__uint_as_float(u[i + 1]));
            o0 = __fmul_rn(bf16_round(silu_fast(g0)), u0);
            o1 = __fmul_rn(bf16_round(silu_fast(g1)), u1);
          } else {
            o0 = __uint_as_float(g[i]);
            o1 = __uint_as_float(g[i + 1]);
          }
          const uint32_t pk = pack_bf16x2(o0, o1);
          if (cur.ok && r0 + i < cur.mend) ocol[(size_t)(r0 + i) * P.N] = (uint16_t)pk;
          if (cur.ok && r0 + i + 1 < cur.mend) ocol[(size_t)(r0 + i + 1) * P.N] = (uint16_t)(pk >> 16);
        }
      }
      tc_fence_before();
      mc_mbar_arrive(&acc_empty[buf]);
    }
  }

  // ---- shutdown: record an abort, drain, free TMEM
  __syncthreads();
  if (abort_s && t == 0 && P.status) atomicOr(P.status, 1u);
  if (warp == 1) {
    if (abort_s && lane == 0) {
      // no MMA may still write TMEM when it is freed: this commit arrives once
      // every MMA issued before it has completed
      umma_commit(&drain_bar);
      const unsigned long long dl = mc_globaltimer() + kTimeoutNs;
      while (!mc_mbar_test_sleep(&drain_bar, 0, 20000u))
        if (mc_globaltimer() > dl) break;
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::TMEM_COLS)
                 : "memory");
  }
}

// ---- host side ---------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_a_map(CUtensorMap* map, const uint16_t* a, int rows, int K) {
  auto enc = get_encode();
  if (!enc) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, BOX_ROWS};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MC_OK;
}

template <bool GU>
int launch(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w0, const mc_qweights* w1,
           int n_experts, uint16_t* out, const uint32_t* tiles, const uint32_t* n_tiles,
           int max_tiles, uint32_t* status) {
  using C = Cfg<GU>;
  const int N = w0->out_features / n_experts, K = w0->in_features;
  CUtensorMap map;
  int rc = make_a_map(&map, a, rows, K);
  if (rc) return rc;
  GemmParams P{*w0, GU ? *w1 : *w0, out, reinterpret_cast<const uint4*>(tiles), n_tiles, status,
               N, K, rows, max_tiles, n_experts};
  MC_CUDA(cudaFuncSetAttribute(grouped_gemm_kernel<GU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::SMEM));
  grouped_gemm_kernel<GU><<<ctx->num_sms, kThreads, C::SMEM, ctx->stream>>>(map, P);
  return mc_after_launch("grouped_gemm_kernel");
}

int check_grouped(const uint16_t* a, int rows, const mc_qweights* w, int n_experts,
                  const uint16_t* out, const uint32_t* tiles, const uint32_t* n_tiles,
                  int max_tiles, const char* what) {
  int rc = mc_check_gemv_weights(w, what);
  if (rc) return rc;
  MC_REQUIRE(w->bits == 4, "%s: grouped GEMM needs 4-bit weights", what);
  MC_REQUIRE(n_experts >= 1 && w->out_features % n_experts == 0,
             "%s: stacked rows %d not a multiple of n_experts %d", what, w->out_features,
             n_experts);
  const int N = w->out_features / n_experts;
  MC_REQUIRE(N % BF == 0, "%s: expert width %d must be a multiple of %d", what, N, BF);
  MC_REQUIRE(w->in_features % BK == 0, "%s: K %d must be a multiple of %d", what, w->in_features,
             BK);
  MC_REQUIRE(rows >= 1, "%s: rows %d", what, rows);
  MC_REQUIRE(a && out && tiles && n_tiles && max_tiles >= 1, "%s: null pointer", what);
  MC_REQUIRE(mc_aligned(a, 16) && mc_aligned(out, 16) && mc_aligned(tiles, 16),
             "%s: a/out/tiles must be 16-byte aligned", what);
  return MC_OK;
}

}  // namespace

extern "C" int mc_gemm_q4_grouped(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w,
                                  int n_experts, uint16_t* c, const uint32_t* tiles,
                                  const uint32_t* n_tiles, int max_tiles, uint32_t* status) {
  MC_REQUIRE(ctx, "gemm_q4_grouped: null context");
  int rc = check_grouped(a, rows, w, n_experts, c, tiles, n_tiles, max_tiles, "gemm_q4_grouped");
  if (rc) return rc;
  return launch<false>(ctx, a, rows, w, nullptr, n_experts, c, tiles, n_tiles, max_tiles, status);
}

extern "C" int mc_gemm_q4_grouped_gu(mc_ctx* ctx, const uint16_t* a, int rows,
                                     const mc_qweights* gate, const mc_qweights* up, int n_experts,
                                     uint16_t* act, const uint32_t* tiles, const uint32_t* n_tiles,
                                     int max_tiles, uint32_t* status) {
  MC_REQUIRE(ctx, "gemm_q4_grouped_gu: null context");
  int rc = check_grouped(a, rows, gate, n_experts, act, tiles, n_tiles, max_tiles,
                         "gemm_q4_grouped_gu gate");
  if (rc) return rc;
  rc = check_grouped(a, rows, up, n_experts, act, tiles, n_tiles, max_tiles,
                     "gemm_q4_grouped_gu up");
  if (rc) return rc;
  MC_REQUIRE(gate->out_features == up->out_features && gate->in_features == up->in_features,
             "gemm_q4_grouped_gu: gate/up shapes differ");
  return launch<true>(ctx, a, rows, gate, up, n_experts, act, tiles, n_tiles, max_tiles, status);
}
