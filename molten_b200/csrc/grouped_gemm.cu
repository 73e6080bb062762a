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
// padding rows. D (TMEM) is [128 features][N tokens] fp32: gate/up 2 x 256
// columns (all of TMEM, one buffer), down 256 (two buffers, so the next
// item's MMAs overlap this item's epilogue).
//
// A TMA copy takes about the same time whatever its size, so each K step's
// token rows come as ONE box of 64, 128 or 256 rows (the smallest that covers
// the chunk), several stages in flight.
//
// Persistent kernel, one CTA per SM. Work items = (row chunk, 128-feature
// block), chunk-major, dealt to CTAs in snake order; with the tile list from
// mc_moe_sort_map (full chunks first, then partial ones by decreasing
// height) every CTA gets a similar share. Warp roles (352 threads):
//   warp 0      TMA of the token rows (128-byte swizzle) into the token ring
//   warp 1      TMEM allocation (512 columns); lane 0 issues tcgen05.mma
//               (M=128, N=chunk, K=16, bf16 x bf16 -> fp32) and commits
//   warps 2..9  dequantise the weight tiles straight into the UMMA K-major
//               128-byte-swizzled layout (w = bf16(s*q + b) in bf16x2
//               arithmetic, MLX's dequantize): gate/up: warps 2-5 the gate
//               tile, 6-9 the up tile; down: warps 2-5 the first 32 K of
//               every row, 6-9 the second. Then the epilogue from TMEM, half
//               the columns each, staged per warp in shared memory and
//               stored as 16-byte rows (or, for the expert-parallel step,
//               into each row's home buffer on its source rank)
//   warp 10     TMA of the Q4 code tiles (64-byte swizzle, two K steps per
//               stage) into the code ring, ahead of the dequant warps
// Three rings: token rows (bfull: TMA tx, bempty: tcgen05.commit), code
// tiles (cfull: TMA tx, cempty: one arrival per dequant warp) and weight
// tiles (afull: one arrival per dequant warp, aempty: tcgen05.commit). The
// TMA and MMA roles run on whole warps with one elected lane issuing, and
// every wait a warp takes gives all its lanes one answer.
// Every wait is bounded by a %globaltimer deadline; on timeout the kernel
// records status bit 1, stops issuing and still drains what it issued before
// freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include "mc_internal.cuh"
#include "mc_async.cuh"

namespace {

constexpr int BF = 128;    // weight features per work item (the MMA's M)
constexpr int BK = 64;     // K per stage
constexpr int MAXN = 256;  // token rows per chunk (the MMA's N, rounded up to 16)
constexpr int kDeqThreads = 256;
constexpr int kCodeWarp = (64 + kDeqThreads) / 32;  // the code-tile TMA warp
constexpr int kThreads = 64 + kDeqThreads + 32;
constexpr unsigned long long kTimeoutNs = 1000000000ull;  // default limit per wait: 1 s

template <bool GU>
struct Cfg {
  static constexpr int NMAT = GU ? 2 : 1;              // weight tiles per K step
  static constexpr int B_BYTES = MAXN * BK * 2;        // 32 KB of token rows per K step
  static constexpr int A_BYTES = BF * BK * 2;          // 16 KB per weight tile
  static constexpr int A_STAGE = NMAT * A_BYTES;
  // Ring depths measured best on B200 (cfg3 workload). While the dequant
  // threads still loaded their codes themselves, those loads in flight lived
  // in L1, which shares each SM's 256 KB with shared memory, and deeper rings
  // were slower (down at 4 + 4 stages: 254 us, at 3 + 3: 160 us). With the
  // codes brought by TMA the token rings can be deeper: gate/up 3 token +
  // 2 weight + 2 code stages 247 us (2 + 2 + 4: 262 us), down 4 + 3 + 2
  // 157 us.
  static constexpr int BSTAGES = GU ? 3 : 4;
  static constexpr int ASTAGES = GU ? 2 : 3;
  // per epilogue warp a [16 tokens][32 features] bf16 tile: the warp's
  // outputs leave as 16-byte row vectors instead of one 2-byte store each
  static constexpr int EPI_BYTES = (kDeqThreads / 32) * 16 * 64;
  // Q4 code tiles: per stage two K steps (64 bytes) of the block's 128 rows
  // per weight matrix, brought in by TMA ahead of the dequant warps
  static constexpr int C_STAGE = NMAT * BF * 64;
  static constexpr int CSTAGES = 2;
  static constexpr int SMEM =
      BSTAGES * B_BYTES + ASTAGES * A_STAGE + EPI_BYTES + CSTAGES * C_STAGE + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int ACC_COLS = NMAT * MAXN;         // accumulator columns per item
  static constexpr int NBUF = TMEM_COLS / ACC_COLS;    // gate/up: 1, down: 2
};
static_assert(Cfg<true>::SMEM + 512 <= 232448 && Cfg<false>::SMEM + 512 <= 232448,
              "shared memory budget");

// Where the expert-parallel step's down GEMM stores its rows (set when
// seg_row is not null): the rows of local expert j come from the W source
// ranks in order, source s's from row seg_row[j][s] to seg_row[j][s+1], and
// row r of that segment goes to row seg_home[j][s] + (r - seg_row[j][s]) of
// source s's home buffer home[s] (local or another GPU's, H features).
constexpr int kRetRanks = 8;
struct ReturnMap {
  const uint32_t* seg_row;   // [n_experts][W + 1]
  const uint32_t* seg_home;  // [n_experts][W]
  uint16_t* home[kRetRanks];
  int W;
  uint32_t home_cap;
};

// The expert-parallel step's arrival check (set when flags is not null):
// before its first token load the GEMM waits until every rank's slot of this
// rank's flag words has reached *epoch, the epoch the ranks' dispatch
// launches stored after their rows (into this GEMM's token buffer) were
// written -- the barrier after the dispatch, inside the GEMM, so the GEMM's
// set-up and first weight stages overlap the wait.
struct ArrivalWait {
  const uint32_t* flags;  // this rank's flag words [W]
  const uint32_t* epoch;  // this rank's epoch word
  int W;
};

struct GemmParams {
  mc_qweights w0, w1;
  uint16_t* out;
  const uint4* tiles;
  const uint32_t* n_tiles;
  uint32_t* status;
  int N, K, rows, max_tiles, n_experts;
  unsigned long long timeout_ns;  // limit of every bounded wait (mc_set_wait_limit)
  ReturnMap ret;
  ArrivalWait arrive;
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

// The i-th work item of this CTA: items are dealt in snake order (0..G-1,
// then G-1..0, ...) so that, with the tile list sorted by decreasing height,
// every CTA gets a similar total.
__device__ __forceinline__ int cta_item(int i) {
  const int G = (int)gridDim.x, b = (int)blockIdx.x;
  return i * G + ((i & 1) ? G - 1 - b : b);
}

// Token-row box for a chunk of n rows: one TMA copy of 64, 128 or 256 rows
// (a TMA copy costs about the same time whatever its size, so one big box per
// stage beats several small ones).
struct TokenMaps {
  CUtensorMap m64, m128, m256;
  CUtensorMap c0, c1;  // Q4 codes of w0 / w1 as bytes [E*N rows][K/2], 64-byte swizzle
};

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
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_f,
                                         unsigned long long timeout_ns) {
  if (mc_mbar_test_sleep(bar, parity, 20000u)) return true;
  const unsigned long long deadline = mc_globaltimer() + timeout_ns;
  while (!mc_mbar_test_sleep(bar, parity, 20000u)) {
    if (*abort_f) return false;
    if (mc_globaltimer() > deadline) return false;
  }
  return true;
}

// The same wait for a whole warp, with one answer for all lanes.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_f,
                                          unsigned long long timeout_ns) {
  return __all_sync(0xffffffffu, wait_bar(bar, parity, abort_f, timeout_ns));
}

// One lane of a converged warp (the lowest), chosen with elect.sync.
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(e));
  return e != 0;
}

// ---- epilogue arithmetic ------------------------------------------------------
// Single-value float->bf16 conversions and MUFU exp/rcp each issue at about
// 16 per clock per SM, so the epilogue rounds with integer ops (round to
// nearest even on the bit pattern; inputs are finite) and converts the
// outputs two at a time.
__device__ __forceinline__ float bf16_round(float x) {
  uint32_t u = __float_as_uint(x);
  u += 0x7fffu + ((u >> 16) & 1u);
  return __uint_as_float(u & 0xffff0000u);
}
// silu(g) = g / (1 + e^-g) with the hardware exponential and a fast divide
// (two MUFU ops; accurate in relative terms on both tails, unlike
// 0.5 + 0.5 tanh(g/2) for g << 0): the prefill activations are compared
// within the bf16 tolerance (the tensor cores' summation order is unspecified
// anyway), so the decode path's bit-exact exponential is not needed here.
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&t);
}

// ---- dequantisation of Q4 words into the UMMA layout -------------------------
// NW Q4 words (8 codes each, code j of word i at bits 4j is k = 8i + j) ->
// 8*NW bf16 values in natural k order, word i stored as the 16-byte chunk
// c0 + i at row_base + ((c ^ swz) * 16): the UMMA K-major 128B-swizzle
// layout. In bf16x2 arithmetic, per code pair (k, k+1): one prmt gathers the
// pair's byte from w and w >> 4, one lop3 keeps the two nibbles and ORs the
// exponent of 128 into both halves (bf16 128 + q, exact for q < 16), one
// sub.bf16x2 takes 128 off (exact) and one fma.bf16x2 gives
// w = bf16(s*q + b) rounded once from the exact value (MLX dequantize,
// quant_nax.metal:2948-2951, computes s*q + b in fp32 and then rounds to
// bf16; the two agree except where that double rounding lands on a bf16
// tie, which stays inside the prefill tolerance).
template <int NW>
__device__ __forceinline__ void dequant_words(const uint32_t* W, uint32_t s2, uint32_t b2,
                                              uint8_t* row_base, int swz, int c0) {
  const uint32_t M = 0x43004300u;  // (128, 128) in bf16
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    const uint32_t w = W[i], wo = w >> 4;
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t p, q;
      const uint32_t sel = h | (h << 4) | ((h + 4) << 8) | ((h + 4) << 12);
      asm("prmt.b32 %0, %1, %2, %3;" : "=r"(p) : "r"(w), "r"(wo), "r"(sel));
      asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(p) : "r"(p), "n"(0x000F000F), "r"(M));
      asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(p), "r"(M));
      asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(o[h]) : "r"(s2), "r"(q), "r"(b2));
    }
    *reinterpret_cast<uint4*>(row_base + (((c0 + i) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <bool GU>
__global__ void __launch_bounds__(kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ TokenMaps tm, const GemmParams P) {
  using C = Cfg<GU>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bfull[C::BSTAGES], bempty[C::BSTAGES];
  __shared__ __align__(8) uint64_t afull[C::ASTAGES], aempty[C::ASTAGES];
  __shared__ __align__(8) uint64_t cfull[C::CSTAGES], cempty[C::CSTAGES];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile uint32_t abort_s;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* a_ring = smem + C::BSTAGES * C::B_BYTES;
  uint8_t* epi_ring = a_ring + C::ASTAGES * C::A_STAGE;
  uint8_t* c_ring = epi_ring + C::EPI_BYTES;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

  if (t == 0) {
    for (int s = 0; s < C::BSTAGES; ++s) {
      mc_mbar_init(&bfull[s], 1);
      mc_mbar_init(&bempty[s], 1);
    }
    for (int s = 0; s < C::ASTAGES; ++s) {
      mc_mbar_init(&afull[s], kDeqThreads / 32);
      mc_mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < C::CSTAGES; ++s) {
      mc_mbar_init(&cfull[s], 1);
      mc_mbar_init(&cempty[s], kDeqThreads / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mc_mbar_init(&acc_full[b], 1);
      mc_mbar_init(&acc_empty[b], kDeqThreads / 32);
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
    // The issuing roles run their loops on the whole warp (stage indices and
    // descriptors are warp-uniform) and one elected lane issues: a lone lane
    // in a divergent branch issued tcgen05.mma at about half the rate the
    // tensor pipe takes them while the dequant warps kept its sub-partition busy.
    if (P.arrive.flags) {
      // every rank's rows are in the token buffer once its flag slot holds
      // this step's epoch (bounded; the async-proxy fence then orders the
      // TMA reads after what the acquire loads observed)
      bool arrived = true;
      if (lane == 0) {
        uint32_t ep;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ep) : "l"(P.arrive.epoch) : "memory");
        const unsigned long long dl = mc_globaltimer() + P.timeout_ns;
        for (int q = 0; q < P.arrive.W && arrived; ++q) {
          for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(P.arrive.flags + q) : "memory");
            if ((int)(v - ep) >= 0) break;
            if (mc_globaltimer() > dl) {
              arrived = false;
              break;
            }
            __nanosleep(200);
          }
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        if (!arrived) {
          if (P.status) atomicOr(P.status, 8u);
          abort_s = 1;
        }
      }
      __syncwarp();
    }
    uint32_t it = 0;
    for (int i = 0, item = cta_item(0); item < total; item = cta_item(++i)) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;
      const Item w = item_info(P, item, nblk);
      const CUtensorMap* map = w.n <= 64 ? &tm.m64 : (w.n <= 128 ? &tm.m128 : &tm.m256);
      const uint32_t bytes = (uint32_t)(w.n <= 64 ? 64 : (w.n <= 128 ? 128 : 256)) * BK * 2;
      bool ok = true;
      for (int kk = 0; kk < ksteps; ++kk, ++it) {
        const int s = it % C::BSTAGES;
        const uint32_t ph = (it / C::BSTAGES) & 1;
        if (!warp_wait(&bempty[s], ph ^ 1, &abort_s, P.timeout_ns)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          mc_mbar_expect_tx(&bfull[s], bytes);
          tma_load_2d(smem + s * C::B_BYTES, map, kk * BK, (int)w.m0, &bfull[s]);
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) abort_s = 1;
        break;
      }
    }
    __syncwarp();
    if (abort_s) {
      // loads already issued finish within microseconds; give them a bounded
      // time to land before the CTA may leave
      for (int k = 0; k < 200; ++k) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (lane 0 is the elected lane: the commits track its MMAs, and the
    // shutdown drain below commits from lane 0 too)
    uint32_t it = 0, j = 0;
    for (int i = 0, item = cta_item(0); item < total; item = cta_item(++i), ++j) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;
      const Item w = item_info(P, item, nblk);
      const uint32_t idesc = idesc_for(w.n);
      const int buf = (int)(j % C::NBUF);
      const uint32_t use = j / C::NBUF;
      if (!warp_wait(&acc_empty[buf], (use & 1) ^ 1, &abort_s, P.timeout_ns)) {
        if (lane == 0) abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d0 = tmem + (uint32_t)(buf * C::ACC_COLS);
      bool ok = true;
      for (int kk = 0; kk < ksteps; ++kk, ++it) {
        const int sb = it % C::BSTAGES, sa = it % C::ASTAGES;
        if (!warp_wait(&bfull[sb], (it / C::BSTAGES) & 1, &abort_s, P.timeout_ns) ||
            !warp_wait(&afull[sa], (it / C::ASTAGES) & 1, &abort_s, P.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(mc_smem_u32(smem + sb * C::B_BYTES));
        const uint32_t abase = mc_smem_u32(a_ring + sa * C::A_STAGE);
        if (elect_one()) {
#pragma unroll
          for (int ti = 0; ti < C::NMAT; ++ti) {
            const uint64_t adesc = sw128_desc(abase + ti * C::A_BYTES);
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16)
              umma_bf16(d0 + ti * MAXN, adesc + 2 * k16, bdesc + 2 * k16, idesc,
                        (kk > 0 || k16 > 0) ? 1u : 0u);
          }
          umma_commit(&bempty[sb]);  // both stages free once these MMAs have read them
          umma_commit(&aempty[sa]);
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) abort_s = 1;
        break;
      }
      if (elect_one()) umma_commit(&acc_full[buf]);
      __syncwarp();
    }
    __syncwarp();
  } else if (warp == kCodeWarp) {
    // ------------------------------------------------------- code-tile TMA
    // per item and K-step pair one 64-byte x 128-row box of each weight
    // matrix's codes; runs ahead of the dequant warps by the ring's depth,
    // across item boundaries too
    uint32_t cs = 0;
    const int npairs = ksteps / 2;
    for (int i = 0, item = cta_item(0); item < total; item = cta_item(++i)) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;
      const Item w = item_info(P, item, nblk);
      const int row0 = (int)(w.e * (uint32_t)P.N) + w.nb * BF;
      bool ok = true;
      for (int pr = 0; pr < npairs; ++pr, ++cs) {
        const int s = (int)(cs % C::CSTAGES);
        const uint32_t ph = (cs / C::CSTAGES) & 1;
        if (!warp_wait(&cempty[s], ph ^ 1, &abort_s, P.timeout_ns)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          mc_mbar_expect_tx(&cfull[s], C::C_STAGE);
          tma_load_2d(c_ring + s * C::C_STAGE, &tm.c0, pr * 64, row0, &cfull[s]);
          if (GU) tma_load_2d(c_ring + s * C::C_STAGE + BF * 64, &tm.c1, pr * 64, row0, &cfull[s]);
        }
        __syncwarp();
      }
      if (!ok) {
        if (lane == 0) abort_s = 1;
        break;
      }
    }
    __syncwarp();
    if (abort_s) {
      for (int k = 0; k < 200; ++k) __nanosleep(1000);
    }
  } else {
    // ------------------------------------------ dequant producers + epilogue
    // gate/up: group g = matrix, each thread one 64-code row slice per K
    // step; down: group g = K half, each thread 32 codes of a row per K step.
    constexpr int NU = GU ? 2 : 1;  // uint4 code loads per thread per K step
    const int dt = t - 64;            // 0..255
    const int grp = dt >> 7;
    const int d = dt & 127;           // weight row within the feature block
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const uint16_t* wscales = (GU && grp) ? P.w1.scales : P.w0.scales;
    const uint16_t* wbiases = (GU && grp) ? P.w1.biases : P.w0.biases;
    // Codes come from the TMA ring (cfull / cempty, one stage per K-step
    // pair; row d's 64 bytes have their 16-byte chunks at c ^ ((d >> 1) & 3),
    // the 64-byte swizzle, so eight consecutive rows' chunk c hit eight
    // different bank groups). The scale and bias of a K-step pair are one
    // 32-bit word each, kSB pairs ahead (raw until use: converting at load
    // time would wait for the load there); the next item's first words are
    // requested before this item's epilogue.
    constexpr int kSB = 2;
    uint32_t swr[kSB], bwr[kSB];
    const uint32_t *srow = nullptr, *brow = nullptr;
#pragma unroll
    for (int p = 0; p < kSB; ++p) swr[p] = bwr[p] = 0u;
    auto load_sb = [&](int slot, int pair) {
      if (2 * pair < ksteps) {
        swr[slot] = __ldg(srow + pair);
        bwr[slot] = __ldg(brow + pair);
      }
    };
    auto start_item = [&](int item) -> Item {
      const Item w = item_info(P, item, nblk);
      const size_t wrow = (size_t)w.e * P.N + (size_t)w.nb * BF + d;
      srow = reinterpret_cast<const uint32_t*>(wscales + wrow * (P.K / 64));
      brow = reinterpret_cast<const uint32_t*>(wbiases + wrow * (P.K / 64));
#pragma unroll
      for (int p = 0; p < kSB; ++p) load_sb(p, p);
      return w;
    };
    // dequantise the slice held in c (K step kk) into stage itk
    auto do_slice = [&](const uint4* c, uint32_t itk, uint32_t sc, uint32_t bi) -> bool {
      const int s = itk % C::ASTAGES;
      const uint32_t ph = (itk / C::ASTAGES) & 1;
      if (!warp_wait(&aempty[s], ph ^ 1, &abort_s, P.timeout_ns)) return false;
      uint8_t* row = a_ring + s * C::A_STAGE + (GU ? grp * C::A_BYTES : 0) + d * 128;
      uint32_t W[4 * NU];
#pragma unroll
      for (int u = 0; u < NU; ++u) {
        W[4 * u] = c[u].x;
        W[4 * u + 1] = c[u].y;
        W[4 * u + 2] = c[u].z;
        W[4 * u + 3] = c[u].w;
      }
      dequant_words<4 * NU>(W, sc, bi, row, d & 7, GU ? 0 : 4 * grp);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mc_mbar_arrive(&afull[s]);
      return true;
    };
    const int csw = (d >> 1) & 3;
    const uint32_t c_off = (GU ? (uint32_t)grp * BF * 64u : 0u) + (uint32_t)d * 64u;
    uint32_t it = 0, j = 0, cs = 0;
    Item w = start_item(cta_item(0) < total ? cta_item(0) : 0);
    for (int i = 0, item = cta_item(0); item < total; item = cta_item(++i), ++j) {
      if (__any_sync(0xffffffffu, abort_s != 0)) break;
      if (!w.ok && dt == 0 && P.status) atomicOr(P.status, 2u);
      bool ok = true;
      for (int kk = 0; kk < ksteps && ok; kk += 2, ++cs) {
        const int cst = (int)(cs % C::CSTAGES);
        if (!warp_wait(&cfull[cst], (cs / C::CSTAGES) & 1, &abort_s, P.timeout_ns)) {
          ok = false;
          break;
        }
        const uint8_t* cb = c_ring + cst * C::C_STAGE + c_off;
        const int slot = (kk / 2) % kSB;
        const uint32_t sw = swr[slot], bw = bwr[slot];
        load_sb(slot, kk / 2 + kSB);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 x[NU];
#pragma unroll
          for (int u = 0; u < NU; ++u) {
            const int c = 2 * h + (GU ? u : grp);
            x[u] = *reinterpret_cast<const uint4*>(cb + ((c ^ csw) << 4));
          }
          // the K step's bf16 scale and bias, each in both halves
          const uint32_t sel = h ? 0x3232u : 0x1010u;
          if (!do_slice(x, it + kk + h, __byte_perm(sw, 0, sel), __byte_perm(bw, 0, sel))) {
            ok = false;
            break;
          }
        }
        // both K steps of the stage are read: the code stage is free
        __syncwarp();
        if (ok && lane == 0) mc_mbar_arrive(&cempty[cst]);
      }
      if (!ok) {
        abort_s = 1;
        break;
      }
      it += (uint32_t)ksteps;
      const Item cur = w;
      if (cta_item(i + 1) < total) w = start_item(cta_item(i + 1));
      // ---- epilogue: TMEM [feature][token] -> bf16 out[token][feature]
      const int buf = (int)(j % C::NBUF);
      const uint32_t use = j / C::NBUF;
      if (!warp_wait(&acc_full[buf], use & 1, &abort_s, P.timeout_ns)) {
        abort_s = 1;
        break;
      }
      tc_fence_after();
      const int n16 = cur.n >> 4, split = (n16 + 1) >> 1;
      const int c_lo = grp ? split : 0, c_hi = grp ? n16 : split;
      const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * C::ACC_COLS);
      const bool ret = !GU && P.ret.seg_row != nullptr;
      uint32_t seg[kRetRanks + 1], segh[kRetRanks];
      if (ret) {  // this expert's source segments (uniform over the warp)
#pragma unroll
        for (int k = 0; k <= kRetRanks; ++k)
          seg[k] = k <= P.ret.W ? __ldg(P.ret.seg_row + (size_t)cur.e * (P.ret.W + 1) + k) : 0u;
#pragma unroll
        for (int k = 0; k < kRetRanks; ++k)
          segh[k] = k < P.ret.W ? __ldg(P.ret.seg_home + (size_t)cur.e * P.ret.W + k) : 0u;
      }
      // the source segment holding the current rows: rows [s_lo, s_hi) go to
      // home rows from s_base (null when the segment would pass the home
      // buffer's end); looked up again only when a group leaves it
      uint32_t s_lo = 1u, s_hi = 0u;
      uint16_t* s_base = nullptr;
      auto locate = [&](uint32_t r) {
        s_lo = 1u;
        s_hi = 0u;
        s_base = nullptr;
#pragma unroll
        for (int k = 0; k < kRetRanks; ++k)
          if (k < P.ret.W && r >= seg[k] && r < seg[k + 1]) {
            s_lo = seg[k];
            s_hi = seg[k + 1];
            s_base = segh[k] + (s_hi - s_lo) <= P.ret.home_cap
                         ? P.ret.home[k] + (size_t)segh[k] * P.N
                         : nullptr;
          }
      };
      auto home_row = [&](uint32_t r) -> uint16_t* {
        uint16_t* d = nullptr;
#pragma unroll
        for (int k = 0; k < kRetRanks; ++k)
          if (k < P.ret.W && r >= seg[k] && r < seg[k + 1]) {
            const uint32_t hr = segh[k] + (r - seg[k]);
            d = hr < P.ret.home_cap ? P.ret.home[k] + (size_t)hr * P.N : nullptr;
          }
        return d;
      };
      // two 16-column groups per TMEM wait: their loads and the two groups'
      // independent arithmetic overlap (one group per wait left the epilogue
      // latency-bound)
#pragma unroll 1
      for (int c2 = c_lo; c2 < c_hi; c2 += 2) {
        const bool two = c2 + 1 < c_hi;  // warp-uniform
        uint32_t gg[2][16], uu[2][16];
        tmem_ld16(lane_base + 16 * c2, gg[0]);
        if (GU) tmem_ld16(lane_base + MAXN + 16 * c2, uu[0]);
        if (two) {
          tmem_ld16(lane_base + 16 * (c2 + 1), gg[1]);
          if (GU) tmem_ld16(lane_base + MAXN + 16 * (c2 + 1), uu[1]);
        }
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && !two) break;
          const int c = c2 + h;
          const uint32_t* g = gg[h];
          const uint32_t* u = uu[h];
          const uint32_t r0 = cur.m0 + 16u * (uint32_t)c;
          // a 16-row group inside one source segment gets one home base
          uint16_t* gbase = nullptr;
          if (ret) {
            const uint32_t rl = min(r0 + 15u, cur.mend - 1u);
            if (!(r0 >= s_lo && rl < s_hi)) locate(r0);
            if (r0 >= s_lo && rl < s_hi && s_base) gbase = s_base + (size_t)(r0 - s_lo) * P.N;
          }
          // this group's 16 tokens x the warp's 32 features through the warp's
          // shared tile, then one 16-byte vector per (token, 8 features)
          uint8_t* tb = epi_ring + (dt >> 5) * 1024;
#pragma unroll
          for (int i2 = 0; i2 < 16; i2 += 2) {
            float o0, o1;
            if (GU) {
              const float g0 = bf16_round(__uint_as_float(g[i2]));
              const float g1 = bf16_round(__uint_as_float(g[i2 + 1]));
              const float u0 = bf16_round(__uint_as_float(u[i2]));
              const float u1 = bf16_round(__uint_as_float(u[i2 + 1]));
              o0 = __fmul_rn(bf16_round(silu_fast(g0)), u0);
              o1 = __fmul_rn(bf16_round(silu_fast(g1)), u1);
            } else {
              o0 = __uint_as_float(g[i2]);
              o1 = __uint_as_float(g[i2 + 1]);
            }
            const uint32_t pk = pack_bf16x2(o0, o1);
            *reinterpret_cast<uint16_t*>(tb + i2 * 64 + lane * 2) = (uint16_t)pk;
            *reinterpret_cast<uint16_t*>(tb + (i2 + 1) * 64 + lane * 2) = (uint16_t)(pk >> 16);
          }
          __syncwarp();
          const size_t col = (size_t)cur.nb * BF + 32 * q + 8 * (lane & 3);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int rr = (lane >> 2) + 8 * hh;
            const uint4 v = *reinterpret_cast<const uint4*>(tb + rr * 64 + (lane & 3) * 16);
            const uint32_t row = r0 + (uint32_t)rr;
            if (cur.ok && row < cur.mend) {
              uint16_t* rp = ret ? (gbase ? gbase + (size_t)rr * P.N : home_row(row))
                                 : P.out + (size_t)row * P.N;
              if (rp) *reinterpret_cast<uint4*>(rp + col) = v;
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mc_mbar_arrive(&acc_empty[buf]);
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
      const unsigned long long dl = mc_globaltimer() + P.timeout_ns;
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

int make_a_map(CUtensorMap* map, const uint16_t* a, int rows, int K, int box_rows) {
  auto enc = get_encode();
  if (!enc) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MC_OK;
}

// The Q4 codes of a stacked [rows][K] matrix as bytes [rows][K/2]; box =
// two K steps (64 bytes) x 128 rows, 64-byte swizzle.
int make_code_map(CUtensorMap* map, const void* codes, int rows, int K) {
  auto enc = get_encode();
  if (!enc) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)K / 2, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K / 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)BF};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(codes), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mc_fail(MC_ECUDA, "cuTensorMapEncodeTiled (codes) failed (%d)", (int)r);
  return MC_OK;
}

template <bool GU>
int launch(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w0, const mc_qweights* w1,
           int n_experts, uint16_t* out, const uint32_t* tiles, const uint32_t* n_tiles,
           int max_tiles, uint32_t* status, const ReturnMap* ret = nullptr,
           const ArrivalWait* arrive = nullptr) {
  using C = Cfg<GU>;
  const int N = w0->out_features / n_experts, K = w0->in_features;
  TokenMaps tm;
  int rc;
  if ((rc = make_a_map(&tm.m64, a, rows, K, 64)) || (rc = make_a_map(&tm.m128, a, rows, K, 128)) ||
      (rc = make_a_map(&tm.m256, a, rows, K, 256)) ||
      (rc = make_code_map(&tm.c0, w0->codes, w0->out_features, K)) ||
      (rc = make_code_map(&tm.c1, GU ? w1->codes : w0->codes, w0->out_features, K)))
    return rc;
  GemmParams P{*w0, GU ? *w1 : *w0, out, reinterpret_cast<const uint4*>(tiles), n_tiles, status,
               N, K, rows, max_tiles, n_experts, mc_wait_limit(ctx, kTimeoutNs), {}};
  if (ret) P.ret = *ret;
  if (arrive) P.arrive = *arrive;
  MC_CUDA(cudaFuncSetAttribute(grouped_gemm_kernel<GU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::SMEM));
  grouped_gemm_kernel<GU><<<ctx->num_sms, kThreads, C::SMEM, ctx->stream>>>(tm, P);
  return mc_after_launch("grouped_gemm_kernel");
}

// Row chunks of a dense GEMM (one expert): tiles[i] = {256 i, min(256 i + 256,
// m), 0, 0}, *n_tiles = their count.
__global__ void dense_tiles_kernel(uint4* __restrict__ tiles, uint32_t* __restrict__ n_tiles,
                                   int m) {
  const int T = (m + MAXN - 1) / MAXN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x)
    tiles[i] = make_uint4((uint32_t)(i * MAXN), (uint32_t)min((i + 1) * MAXN, m), 0u, 0u);
  if (blockIdx.x == 0 && threadIdx.x == 0) *n_tiles = (uint32_t)T;
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
  // K steps come in pairs whose scales (and biases) are read as one 32-bit word
  MC_REQUIRE(w->in_features % (2 * BK) == 0, "%s: K %d must be a multiple of %d", what,
             w->in_features, 2 * BK);
  MC_REQUIRE(mc_aligned(w->scales, 4) && mc_aligned(w->biases, 4),
             "%s: scales/biases must be 4-byte aligned", what);
  MC_REQUIRE(mc_aligned(w->codes, 16), "%s: codes must be 16-byte aligned", what);
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

// The down GEMM of the expert-parallel step: mc_gemm_q4_grouped with each
// output row stored into its source rank's home buffer (ep_prefill.cu).
int mc_gemm_q4_grouped_return(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w,
                              int n_experts, const uint32_t* seg_row, const uint32_t* seg_home,
                              void* const* home, int world, size_t home_cap,
                              const uint32_t* tiles, const uint32_t* n_tiles, int max_tiles,
                              uint32_t* status) {
  MC_REQUIRE(ctx && seg_row && seg_home && home, "gemm_q4_grouped_return: null pointer");
  MC_REQUIRE(world >= 1 && world <= kRetRanks, "gemm_q4_grouped_return: world %d", world);
  int rc = check_grouped(a, rows, w, n_experts, a, tiles, n_tiles, max_tiles,
                         "gemm_q4_grouped_return");
  if (rc) return rc;
  ReturnMap rm{};
  rm.seg_row = seg_row;
  rm.seg_home = seg_home;
  for (int k = 0; k < world; ++k) {
    MC_REQUIRE(home[k] && mc_aligned(home[k], 16), "gemm_q4_grouped_return: home buffer %d", k);
    rm.home[k] = static_cast<uint16_t*>(home[k]);
  }
  rm.W = world;
  rm.home_cap = (uint32_t)(home_cap < 0xffffffffu ? home_cap : 0xffffffffu);
  return launch<false>(ctx, a, rows, w, nullptr, n_experts, nullptr, tiles, n_tiles, max_tiles,
                       status, &rm);
}

extern "C" size_t mc_gemm_q4_workspace_words(int m) {
  return m < 1 ? 0 : (size_t)4 * ((m + MAXN - 1) / MAXN) + 4;
}

extern "C" int mc_gemm_q4(mc_ctx* ctx, const uint16_t* a, int m, const mc_qweights* w,
                          uint16_t* c, uint32_t* workspace, size_t ws_words, uint32_t* status) {
  MC_REQUIRE(ctx, "gemm_q4: null context");
  MC_REQUIRE(m >= 1, "gemm_q4: m %d", m);
  MC_REQUIRE(workspace && ws_words >= mc_gemm_q4_workspace_words(m),
             "gemm_q4: workspace of %zu words, %zu needed", ws_words, mc_gemm_q4_workspace_words(m));
  const int T = (m + MAXN - 1) / MAXN;
  uint32_t* tiles = workspace;
  uint32_t* n_tiles = workspace + 4 * (size_t)T;
  int rc = check_grouped(a, m, w, 1, c, tiles, n_tiles, T, "gemm_q4");
  if (rc) return rc;
  dense_tiles_kernel<<<(T + 255) / 256, 256, 0, ctx->stream>>>(reinterpret_cast<uint4*>(tiles),
                                                              n_tiles, m);
  if ((rc = mc_after_launch("dense_tiles_kernel"))) return rc;
  return launch<false>(ctx, a, m, w, nullptr, 1, c, tiles, n_tiles, T, status);
}

int mc_gemm_q4_grouped_gu_after(mc_ctx* ctx, const uint16_t* a, int rows,
                                const mc_qweights* gate, const mc_qweights* up, int n_experts,
                                uint16_t* act, const uint32_t* tiles, const uint32_t* n_tiles,
                                int max_tiles, uint32_t* status, const uint32_t* flags,
                                const uint32_t* epoch, int world) {
  MC_REQUIRE(ctx && flags && epoch, "gemm_q4_grouped_gu_after: null pointer");
  MC_REQUIRE(world >= 1 && world <= kRetRanks, "gemm_q4_grouped_gu_after: world %d", world);
  int rc = check_grouped(a, rows, gate, n_experts, act, tiles, n_tiles, max_tiles,
                         "gemm_q4_grouped_gu_after gate");
  if (rc) return rc;
  rc = check_grouped(a, rows, up, n_experts, act, tiles, n_tiles, max_tiles,
                     "gemm_q4_grouped_gu_after up");
  if (rc) return rc;
  MC_REQUIRE(gate->out_features == up->out_features && gate->in_features == up->in_features,
             "gemm_q4_grouped_gu_after: gate/up shapes differ");
  const ArrivalWait aw{flags, epoch, world};
  return launch<true>(ctx, a, rows, gate, up, n_experts, act, tiles, n_tiles, max_tiles, status,
                      nullptr, &aw);
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
