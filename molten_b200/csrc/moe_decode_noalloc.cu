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
// (moved to the caller's `status` and cleared by the launch's last CTA, so it
// reports that call only), words 3 and 4 reserved (zero; word 4 counts
// projection rows only in mc_moe_decode_layer_proj, which this entry point
// does not run), words 8..135 tagged router logits, then the bf16 act rows. It serves expert
// widths up to kNoallocMaxInter; wider layers are rejected with MC_EINVAL
// before anything is launched.
//
// Every argument is checked before anything is enqueued. All of the scratch
// must be zero before the first launch on a device: the first call on each
// device (after its checks pass) makes the device current, zeroes the array
// on the context's stream and waits for that. So the first call blocks and
// must come before any stream capture. Afterwards every launch leaves the
// control words as the next one needs them (the last CTA clears the counters
// and the status word and advances the epoch), and each call is one kernel
// launch, chained to its neighbours like the workspace entry point.
//
// The array's device address is looked up with cudaGetSymbolAddress on every
// call (with the context's device current), never cached: a host-side name of
// a __device__ array is not a device address.
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
bool g_zeroed[kMaxDevices] = {};

// Runs `fn` with ctx's device current, restoring the caller's device.
template <typename F>
cudaError_t on_device(int device, F fn) {
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return e;
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) return e;
  e = fn();
  if (prev != device) {
    const cudaError_t e2 = cudaSetDevice(prev);
    if (e == cudaSuccess) e = e2;
  }
  return e;
}

}  // namespace

int mc_noalloc_decode_scratch(mc_ctx* ctx, uint32_t** out, size_t* words) {
  MC_REQUIRE(ctx->device >= 0 && ctx->device < kMaxDevices,
             "moe_decode_layer_noalloc: device %d out of range", ctx->device);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  void* p = nullptr;
  const bool first = !g_zeroed[ctx->device];
  cudaError_t e = on_device(ctx->device, [&]() {
    cudaError_t r = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (r == cudaSuccess && first)
      r = cudaMemsetAsync(p, 0, sizeof(uint32_t) * kNoallocWords, ctx->stream);
    if (r == cudaSuccess && first) r = cudaStreamSynchronize(ctx->stream);
    return r;
  });
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return mc_fail(MC_ECUDA,
                   "moe_decode_layer_noalloc: scratch %s on device %d failed: %s "
                   "(the first call on a device must not be inside a stream capture)",
                   first ? "set-up" : "lookup", ctx->device, cudaGetErrorString(e));
  }
  g_zeroed[ctx->device] = true;
  *out = static_cast<uint32_t*>(p);
  *words = kNoallocWords;
  return MC_OK;
}

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
  // the remaining checks, then the scratch set-up, then the one launch
  return mc_decode_layer_impl(ctx, h, b, norm_w, h_out, normed, router_w, router_dtype,
                              expert_bias, route_mode, logits, ids, weights, gate, up, down,
                              n_experts, out, nullptr, 0, eps, route_eps, true, status,
                              nullptr, nullptr);
}
