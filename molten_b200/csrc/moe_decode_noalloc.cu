// mc_moe_decode_layer_noalloc: the one-launch MoE decode layer with its
// scratch in a fixed array compiled into this library, for callers that
// cannot hand the library device memory of their own: a host engine whose
// allocator is frozen once its weights and KV pages are laid out, a plugin
// that is not allowed to call an allocator on the serving path, or a caller
// holding no buffer it could lend for the epoch/counter words. Nothing is
// allocated by this entry point, and nothing in it calls cudaMalloc, cudaFree
// or any library that allocates.
//
// The scratch is the same layout mc_moe_decode_layer documents for its
// caller-owned workspace: word 0 epoch, word 1 exit counter, word 2 status
// (cleared before each launch here, copied to the caller's `status` after
// it), word 3 act counter, word 4 router counter, words 8..135 tagged router
// logits, then the
// bf16 act rows. It serves expert widths up to kNoallocMaxInter; wider layers
// are rejected with MC_EINVAL before anything is launched.
//
// All of it must be zero before the first launch on a device. The first call
// on each device does that set-up: it makes the device current, looks up the
// array's address with cudaGetSymbolAddress, zeroes it on the context's
// stream and waits for that. So the first call blocks and must come before
// any stream capture. Afterwards every launch leaves the control words as the
// next one needs them (the last CTA clears the counters and advances the
// epoch).
//
// There is ONE scratch per device, shared by every context and stream of the
// process on that device: two calls whose kernels can overlap on the device
// (different streams without an event between them, or different threads
// without ordering) race on it and give wrong results. Order them.

#include <mutex>

#include "mc_internal.cuh"

namespace {

constexpr int kNoallocMaxInter = 2048;            // widest expert row served
constexpr int kNoallocCtlWords = 136;             // control + tagged logits
constexpr size_t kNoallocWords = kNoallocCtlWords + 4 * (size_t)kNoallocMaxInter;  // 33,312 B
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint32_t g_decode_scratch[kNoallocWords];

std::mutex g_setup_mu;
uint32_t* g_scratch_ptr[kMaxDevices] = {};

// Address of this device's scratch; the first call per device zeroes it.
int scratch_for(mc_ctx* ctx, uint32_t** out) {
  MC_REQUIRE(ctx->device >= 0 && ctx->device < kMaxDevices,
             "moe_decode_layer_noalloc: device %d out of range", ctx->device);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[ctx->device]) {
    *out = g_scratch_ptr[ctx->device];
    return MC_OK;
  }
  int prev = -1;
  MC_CUDA(cudaGetDevice(&prev));
  if (prev != ctx->device) MC_CUDA(cudaSetDevice(ctx->device));
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, sizeof(uint32_t) * kNoallocWords, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (prev != ctx->device) {
    cudaError_t e2 = cudaSetDevice(prev);
    if (e == cudaSuccess) e = e2;
  }
  if (e != cudaSuccess)
    return mc_fail(MC_ECUDA,
                   "moe_decode_layer_noalloc: scratch set-up on device %d failed: %s "
                   "(the first call on a device must not be inside a stream capture)",
                   ctx->device, cudaGetErrorString(e));
  g_scratch_ptr[ctx->device] = static_cast<uint32_t*>(p);
  *out = g_scratch_ptr[ctx->device];
  return MC_OK;
}

}  // namespace

extern "C" int mc_moe_decode_layer_noalloc(
    mc_ctx* ctx, const uint16_t* h, const uint16_t* b, const uint16_t* norm_w, uint16_t* h_out,
    uint16_t* normed, const void* router_w, int router_dtype, const float* expert_bias,
    int route_mode, float* logits, uint32_t* ids, uint16_t* weights, const mc_qweights* gate,
    const mc_qweights* up, const mc_qweights* down, int n_experts, uint16_t* out,
    uint32_t* status, float eps, float route_eps) {
  MC_REQUIRE(ctx, "moe_decode_layer_noalloc: null context");
  MC_REQUIRE(gate && n_experts > 0, "moe_decode_layer_noalloc: null gate or no experts");
  const long inter = gate->out_features / n_experts;
  MC_REQUIRE(inter <= kNoallocMaxInter,
             "moe_decode_layer_noalloc: expert width %ld exceeds the built-in scratch "
             "(max %d; use mc_moe_decode_layer with a workspace)",
             inter, kNoallocMaxInter);
  uint32_t* scratch = nullptr;
  int rc = scratch_for(ctx, &scratch);
  if (rc) return rc;
  // the status word reports this call only (the workspace variant keeps it sticky)
  MC_CUDA(cudaMemsetAsync(scratch + 2, 0, sizeof(uint32_t), ctx->stream));
  rc = mc_moe_decode_layer(ctx, h, b, norm_w, h_out, normed, router_w, router_dtype, expert_bias,
                           route_mode, logits, ids, weights, gate, up, down, n_experts, out,
                           scratch, kNoallocWords, eps, route_eps);
  if (rc) return rc;
  if (status)
    MC_CUDA(cudaMemcpyAsync(status, scratch + 2, sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                            ctx->stream));
  return MC_OK;
}
