// Internal plumbing shared by the kernel files: the context, the thread-local
// error message, argument checks and small device helpers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>
#include "../../include/molten_cuda.h"
#include "mc_numerics.cuh"

struct mc_ctx {
  int device;
  cudaStream_t stream;
  int owns_stream;
  int num_sms;
  int max_smem_optin;
  int l2_bytes;
  unsigned long long* trace;  // optional per-CTA phase timestamps (mc_set_trace)
  int trace_len;
  const void* pf_ptr[2];      // L2 prefetch for the next decode-layer launch
  size_t pf_bytes[2];         // (mc_set_l2_prefetch; cleared by that launch)
  unsigned long long wait_limit_ns;  // bounded-wait limit (mc_set_wait_limit; 0 = default)
  int test_flags;             // MC_TEST_* (mc_set_test_flags; 0 in production)
  struct mc_ep_state* ep;     // expert-parallel state (mc_ep_init), or NULL
};

// Wait limit a kernel with default `dflt` uses on this context.
static inline unsigned long long mc_wait_limit(const mc_ctx* ctx, unsigned long long dflt) {
  return ctx->wait_limit_ns ? ctx->wait_limit_ns : dflt;
}

// The fused decode layer behind mc_moe_decode_layer, _noalloc and _proj
// (moe_decode_fused.cu). With `proj`, b is computed in the launch as
// bf16(proj . h) (b must be null) and copied to p_out when that is given.
int mc_decode_layer_impl(mc_ctx* ctx, const uint16_t* h, const uint16_t* b,
                         const uint16_t* norm_w, uint16_t* h_out, uint16_t* normed,
                         const void* router_w, int router_dtype, const float* expert_bias,
                         int route_mode, float* logits, uint32_t* ids, uint16_t* weights,
                         const mc_qweights* gate, const mc_qweights* up, const mc_qweights* down,
                         int n_experts, uint16_t* out, uint32_t* sync, size_t ws_words, float eps,
                         float route_eps, bool noalloc, uint32_t* status_out,
                         const mc_qweights* proj, uint16_t* p_out);
// Grouped GEMM (not gate/up) storing each output row into its source
// rank's home buffer: rows of expert j from source s are seg_row[j][s] ..
// seg_row[j][s+1] and go to rows from seg_home[j][s] of home[s]
// (grouped_gemm.cu).
// mc_ep_dispatch whose last CTA also writes the receive side's row chunks
// (as mc_ep_tiles) and the return map of the local slots: rows of local slot
// j from source s are seg_row[j][s] .. seg_row[j][s+1] and go to rows from
// seg_home[j][s] of s's home buffer (ep.cu).
int mc_ep_dispatch_plan(mc_ctx* ctx, const uint16_t* x, int m, int hidden,
                        const uint32_t* ids_sorted, const uint32_t* counts_all, int rank,
                        int world, int n_experts, void* const* recv_bufs, size_t recv_cap_rows,
                        uint32_t* status, int bm, uint32_t* tiles, uint32_t* n_tiles,
                        uint32_t* rows, int max_tiles, uint32_t* seg_row, uint32_t* seg_home,
                        uint32_t* const* flag_ptrs, uint32_t* epoch, uint32_t* done, int skip);
// mc_gemm_q4_grouped_gu whose token loads first wait (bounded) until every
// slot of `flags` [world] has reached *epoch (grouped_gemm.cu).
int mc_gemm_q4_grouped_gu_after(mc_ctx* ctx, const uint16_t* a, int rows,
                                const mc_qweights* gate, const mc_qweights* up, int n_experts,
                                uint16_t* act, const uint32_t* tiles, const uint32_t* n_tiles,
                                int max_tiles, uint32_t* status, const uint32_t* flags,
                                const uint32_t* epoch, int world);
int mc_gemm_q4_grouped_return(mc_ctx* ctx, const uint16_t* a, int rows, const mc_qweights* w,
                              int n_experts, const uint32_t* seg_row, const uint32_t* seg_home,
                              void* const* home, int world, size_t home_cap,
                              const uint32_t* tiles, const uint32_t* n_tiles, int max_tiles,
                              uint32_t* status);
// Expert-parallel state (ep_prefill.cu): waits for the stream while watching
// the communicator (mc_sync with a communicator); releases it on mc_destroy.
int mc_ep_wait(mc_ctx* ctx);
void mc_ep_release(mc_ctx* ctx);
// The built-in decode scratch of ctx's device and its size in u32 words; the
// first call per device zeroes it (moe_decode_noalloc.cu).
int mc_noalloc_decode_scratch(mc_ctx* ctx, uint32_t** ptr, size_t* words);

__device__ __forceinline__ unsigned long long mc_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Records a formatted message for mc_last_error() and returns `code`.
int mc_fail(int code, const char* fmt, ...);

#define MC_REQUIRE(cond, ...)                                  \
  do {                                                         \
    if (!(cond)) return mc_fail(MC_EINVAL, __VA_ARGS__);       \
  } while (0)

// A failed runtime call is reported once: the per-thread "last error" it set
// is cleared (a refused launch is not sticky), so a later launch check does
// not report it again.
#define MC_CUDA(call)                                                            \
  do {                                                                           \
    cudaError_t _e = (call);                                                     \
    if (_e != cudaSuccess) {                                                     \
      (void)cudaGetLastError();                                                  \
      return mc_fail(MC_ECUDA, "%s failed: %s", #call, cudaGetErrorString(_e));  \
    }                                                                            \
  } while (0)

// check_quant for the GEMV kernels (mc_api.cu): inputs up to 4096, or up to
// max_k for the kernels that take wider rows.
int mc_check_gemv_weights(const mc_qweights* w, const char* what);
int mc_check_gemv_weights_k(const mc_qweights* w, const char* what, int max_k);
// Q4 GEMV for 4096 < K <= 16384 (gemv_fused.cu).
int mc_gemv_q4_wide(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                    int batch);

// Checks the launch that was just issued.
int mc_after_launch(const char* what);
// Ring-streamed GEMV (gemv_ring.cu) for batch 1, K = 2048, tall matrices;
// returns 1 when the shape does not qualify. mode 0: y, mode 1: argmax keys.
int mc_gemv_ring(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                 unsigned long long* keys, int batch, int mode);
// Batched GEMV (gemv_batched.cu) for K <= 2048 at batch >= 2 on tall
// matrices, batch >= 8 on any: each code decoded once for up to 8 tokens;
// same return convention.
int mc_gemv_batched(mc_ctx* ctx, const mc_qweights* w, const uint16_t* x, uint16_t* y,
                    unsigned long long* keys, int batch, int mode);

static inline bool mc_aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

// ------------------------------------------------------------ device helpers

// Streaming 16-byte load that skips L1 (weights are read exactly once).
__device__ __forceinline__ uint4 mc_ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// One row of h16 16-byte words copied by a warp: eight loads per lane in
// flight before their stores (a load-store pair per step left the NVLink row
// copies latency-bound). `in` is read through the read-only path: it must
// not be written during the kernel.
__device__ __forceinline__ void mc_copy_row16(uint4* __restrict__ out,
                                              const uint4* __restrict__ in, int h16, int lane) {
  for (int c0 = 0; c0 < h16; c0 += 256) {
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c < h16) v[i] = __ldg(in + c);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c < h16) out[c] = v[i];
    }
  }
}

__device__ __forceinline__ float mc_warp_butterfly(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// 2^-e as a float constant (e in 0..23).
__device__ __forceinline__ float mc_pow2_neg(int e) { return __uint_as_float((uint32_t)(127 - e) << 23); }

// Programmatic dependent launch. The decode-chain kernels are launched with
// cudaLaunchAttributeProgrammaticStreamSerialization (mc_launch_pdl), so the
// next kernel of the stream is launched while this one still runs. Each of
// them calls mc_pdl_launch_dependents() at its start and mc_pdl_wait() before
// it reads anything an earlier kernel wrote or writes anything an earlier
// kernel may still read; the wait returns once the predecessors have
// completed and their memory is visible (at once when there is none).
__device__ __forceinline__ void mc_pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void mc_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t mc_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

#define MC_MAGIC 0x4B000000u
#define MC_MAGIC_F 8388608.0f
