// Prefill grouped expert GEMM on the 5th-generation tensor cores
// (gemm_q4_grouped_mlx / _gu, quant.rs:146-266 -> lfm_qmm_t_body,
// quant_nax.metal:4091-4234).
//
//   C[i][n] = sum_k A[i][k] * bf16(s*q + b)[e*N + n][k]
//
// for the sorted rows i of each row tile (m0, m_end, expert e); A bf16
// [rows][K] (the expert-sorted activations), W the stacked [E*N][K] MLX Q4
// matrix. The gate/up variant computes both GEMMs of a tile against the same
// A tile and writes act = bf16(bf16(silu(bf16(g))) * bf16(u)) in the
// epilogue (silu_mul_bf16, elementwise.metal:7-15).
//
// Persistent kernel, one CTA per SM, work items = (row tile, 128-column
// block) in tile-major order so neighbouring CTAs share the A tile in L2.
// Warp roles (192 threads):
//   warp 0      TMA: 128x64 bf16 A tiles, 128-byte swizzle, into the stage ring
//   warp 1      TMEM allocation; lane 0 issues tcgen05.mma (M=128, N=128,
//               K=16, bf16 x bf16 -> fp32) and tcgen05.commit
//   warps 2..5  dequantise the B tile(s) straight into the UMMA K-major
//               128-byte-swizzled layout (w = bf16(fma(s, q, b)), MLX's
//               dequantize), then run the epilogue from TMEM (tcgen05.ld)
// Stage s: full[s] (TMA tx + 128 dequant arrivals), empty[s] (tcgen05.commit).
// Every wait is bounded by a %globaltimer deadline; on timeout the kernel
// records status bit 1, stops issuing and still drains what it issued before
// freeing TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include "mc_internal.cuh"
#include "mc_async.cuh"

namespace {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int kThreads = 192;
constexpr unsigned long long kTimeoutNs = 1000000000ull;  // 1 s per wait

template <bool GU>
struct Cfg {
  static constexpr int STAGES = GU ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;  // 16 KB per weight matrix
  static constexpr int NMAT = GU ? 2 : 1;
  static constexpr int STAGE_BYTES = A_BYTES + NMAT * B_BYTES;
  static constexpr int TMEM_COLS = GU ? 256 : 128;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
};

struct GemmParams {
  mc_qweights w0, w1;
  uint16_t* out;
  const uint4* tiles;
  const uint32_t* n_tiles;
  uint32_t* status;
  int N, K, rows, max_tiles, n_experts;
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

// Instruction descriptor: D f32, A/B bf16, both K-major, N = BN, M = BM.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
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

// Bounded mbarrier wait that also gives up when another role aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_f,
                                         unsigned long long deadline) {
  while (!mc_mbar_test_sleep(bar, parity, 20000u)) {
    if (*abort_f) return false;
    if (mc_globaltimer() > deadline) return false;
  }
  return true;
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
  __shared__ __align__(8) uint64_t full[C::STAGES], empty[C::STAGES];
  __shared__ __align__(8) uint64_t acc_full, acc_empty;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile uint32_t abort_s;
  __shared__ uint32_t acc_commits_s;  // commits the MMA thread made to acc_full

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const unsigned long long t_start = mc_globaltimer();

  if (t == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mc_mbar_init(&full[s], 1 + 128);
      mc_mbar_init(&empty[s], 1);
    }
    mc_mbar_init(&acc_full, 1);
    mc_mbar_init(&acc_empty, 128);
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

  const int nblk = P.N / BN;
  const int ksteps = P.K / BK;
  int ntiles = (int)*P.n_tiles;
  if (ntiles > P.max_tiles) ntiles = P.max_tiles;
  const int total = ntiles * nblk;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x) {
        const uint4 tile = P.tiles[item / nblk];
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!wait_bar(&empty[s], ph ^ 1, &abort_s, mc_globaltimer() + kTimeoutNs)) {
            abort_s = 1;
            break;
          }
          mc_mbar_expect_tx(&full[s], C::A_BYTES);
          tma_load_2d(smem + s * C::STAGE_BYTES, &tmA, kk * BK, (int)tile.x, &full[s]);
        }
      }
    }
    if (lane == 0 && abort_s) {
      // loads already issued finish within microseconds; give them a bounded
      // time to land before the CTA may leave
      for (int k = 0; k < 200; ++k) __nanosleep(1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, j = 0;
      acc_commits_s = 0;
      for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x, ++j) {
        if (!wait_bar(&acc_empty, (j & 1) ^ 1, &abort_s, mc_globaltimer() + kTimeoutNs)) {
          abort_s = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kk = 0; kk < ksteps; ++kk, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!wait_bar(&full[s], ph, &abort_s, mc_globaltimer() + kTimeoutNs)) {
            abort_s = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = mc_smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc0 = sw128_desc(a_addr + C::A_BYTES);
          const uint64_t bdesc1 = sw128_desc(a_addr + C::A_BYTES + C::B_BYTES);
#pragma unroll
          for (int k16 = 0; k16 < BK / 16; ++k16) {
            const uint32_t acc = (kk > 0 || k16 > 0) ? 1u : 0u;
            umma_bf16(tmem, adesc + 2 * k16, bdesc0 + 2 * k16, acc);
            if (GU) umma_bf16(tmem + BN, adesc + 2 * k16, bdesc1 + 2 * k16, acc);
          }
          umma_commit(&empty[s]);  // stage free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&acc_full);
        acc_commits_s = j + 1;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------ dequant producers + epilogue
    const int d = t - 64;  // B-tile row (0..127)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r_out = 32 * q + lane;  // accumulator row this thread reads
    uint32_t it = 0, j = 0;
    for (int item = blockIdx.x; item < total && !abort_s; item += gridDim.x, ++j) {
      const uint4 tile = P.tiles[item / nblk];
      const int nb = item % nblk;
      const uint32_t e = tile.z;
      const bool tile_ok = e < (uint32_t)P.n_experts && tile.x < tile.y &&
                           tile.y <= (uint32_t)P.rows && tile.y - tile.x <= (uint32_t)BM;
      if (!tile_ok && t == 64 && P.status) atomicOr(P.status, 2u);
      const size_t wrow = (size_t)(tile_ok ? e : 0) * P.N + (size_t)nb * BN + d;
      const uint8_t* c0 = reinterpret_cast<const uint8_t*>(P.w0.codes) + wrow * (P.K / 2);
      const uint16_t* s0 = P.w0.scales + wrow * (P.K / 64);
      const uint16_t* b0 = P.w0.biases + wrow * (P.K / 64);
      const uint8_t* c1 = GU ? reinterpret_cast<const uint8_t*>(P.w1.codes) + wrow * (P.K / 2) : c0;
      const uint16_t* s1 = GU ? P.w1.scales + wrow * (P.K / 64) : s0;
      const uint16_t* b1 = GU ? P.w1.biases + wrow * (P.K / 64) : b0;
      bool ok = true;
      uint4 na0 = __ldg(reinterpret_cast<const uint4*>(c0));
      uint4 nb0 = __ldg(reinterpret_cast<const uint4*>(c0) + 1);
      uint4 na1 = na0, nb1 = nb0;
      if (GU) {
        na1 = __ldg(reinterpret_cast<const uint4*>(c1));
        nb1 = __ldg(reinterpret_cast<const uint4*>(c1) + 1);
      }
      for (int kk = 0; kk < ksteps; ++kk, ++it) {
        const uint4 a0 = na0, bq0 = nb0, a1 = na1, bq1 = nb1;
        const float sc0 = mc_bf16_to_f32(__ldg(s0 + kk)), bi0 = mc_bf16_to_f32(__ldg(b0 + kk));
        float sc1 = 0.0f, bi1 = 0.0f;
        if (GU) {
          sc1 = mc_bf16_to_f32(__ldg(s1 + kk));
          bi1 = mc_bf16_to_f32(__ldg(b1 + kk));
        }
        if (kk + 1 < ksteps) {  // prefetch the next K slice's codes
          na0 = __ldg(reinterpret_cast<const uint4*>(c0 + (kk + 1) * 32));
          nb0 = __ldg(reinterpret_cast<const uint4*>(c0 + (kk + 1) * 32) + 1);
          if (GU) {
            na1 = __ldg(reinterpret_cast<const uint4*>(c1 + (kk + 1) * 32));
            nb1 = __ldg(reinterpret_cast<const uint4*>(c1 + (kk + 1) * 32) + 1);
          }
        }
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1;
        if (!wait_bar(&empty[s], ph ^ 1, &abort_s, mc_globaltimer() + kTimeoutNs)) {
          abort_s = 1;
          ok = false;
          break;
        }
        uint8_t* bt = smem + s * C::STAGE_BYTES + C::A_BYTES;
        dequant_row64(a0, bq0, sc0, bi0, bt + d * 128, d & 7);
        if (GU) dequant_row64(a1, bq1, sc1, bi1, bt + C::B_BYTES + d * 128, d & 7);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mc_mbar_arrive(&full[s]);
      }
      if (!ok) break;
      // ---- epilogue: TMEM -> registers -> bf16 rows
      if (!wait_bar(&acc_full, j & 1, &abort_s, mc_globaltimer() + kTimeoutNs)) {
        abort_s = 1;
        break;
      }
      tc_fence_after();
      const uint32_t m0 = tile.x, mend = tile.y;
      const bool live = tile_ok && m0 + r_out < mend;
      uint16_t* orow = P.out + (size_t)(m0 + r_out) * P.N + (size_t)nb * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t g[16], u[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c, g);
        if (GU) tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + BN + c, u);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          float o[2];
#pragma unroll
          for (int z = 0; z < 2; ++z) {
            const float gv = mc_round_bf16(__uint_as_float(g[2 * h + z]));
            if (GU) {
              const float uv = mc_round_bf16(__uint_as_float(u[2 * h + z]));
              o[z] = __fmul_rn(mc_round_bf16(mc_silu(gv)), uv);
            } else {
              o[z] = gv;
            }
          }
          pk[h] = (uint32_t)mc_f32_to_bf16(o[0]) | ((uint32_t)mc_f32_to_bf16(o[1]) << 16);
        }
        if (live) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      tc_fence_before();
      mc_mbar_arrive(&acc_empty);
    }
  }

  // ---- shutdown: record an abort, drain, free TMEM
  __syncthreads();
  if (abort_s && t == 0 && P.status) atomicOr(P.status, 1u);
  if (warp == 1) {
    if (abort_s && lane == 0) {
      // make sure no MMA is still writing TMEM before it is freed: one more
      // commit completes acc_full's next phase once all issued MMAs are done
      const uint32_t n = acc_commits_s;
      umma_commit(&acc_full);
      const unsigned long long dl = mc_globaltimer() + kTimeoutNs;
      while (!mc_mbar_test_sleep(&acc_full, n & 1, 20000u))
        if (mc_globaltimer() > dl) break;
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::TMEM_COLS)
                 : "memory");
  }
  (void)t_start;
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
  const cuuint32_t box[2] = {BK, BM};
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
  MC_REQUIRE(N % BN == 0, "%s: expert width %d must be a multiple of %d", what, N, BN);
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
