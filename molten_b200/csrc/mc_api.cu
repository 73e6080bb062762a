// Context, errors and weight validation for the C ABI (include/molten_cuda.h).
#include "mc_internal.cuh"
#include <stdlib.h>
#include <string.h>

static thread_local char g_err[512] = "";

int mc_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int mc_after_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return mc_fail(MC_ECUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return MC_OK;
}

// check_quant (quant.rs:42-66) for the decode GEMVs: group 64, 4- or 6-bit,
// in_features a multiple of 64, codes 16-byte aligned (rows are read as
// 16-byte vectors), rows in range.
int mc_check_gemv_weights(const mc_qweights* w, const char* what) {
  return mc_check_gemv_weights_k(w, what, 4096);
}

int mc_check_gemv_weights_k(const mc_qweights* w, const char* what, int max_k) {
  if (!w) return mc_fail(MC_EINVAL, "%s: null weights", what);
  if (w->bits != 4 && w->bits != 6)
    return mc_fail(MC_EUNSUPPORTED, "%s: unsupported bit width %d", what, w->bits);
  if (w->group_size != 64)
    return mc_fail(MC_EUNSUPPORTED, "%s: group size %d (only 64 is built)", what, w->group_size);
  if (w->in_features <= 0 || w->in_features % 64 != 0 || w->in_features > max_k)
    return mc_fail(MC_EINVAL, "%s: in_features %d must be a positive multiple of 64 <= %d",
                   what, w->in_features, max_k);
  if (w->out_features <= 0)
    return mc_fail(MC_EINVAL, "%s: out_features %d", what, w->out_features);
  if (!w->codes || !w->scales || !w->biases)
    return mc_fail(MC_EINVAL, "%s: null codes/scales/biases", what);
  if (!mc_aligned(w->codes, 16))
    return mc_fail(MC_EINVAL, "%s: codes not 16-byte aligned; the kernels read codes as 16-byte vectors",
                   what);
  if (!mc_aligned(w->scales, 2) || !mc_aligned(w->biases, 2))
    return mc_fail(MC_EINVAL, "%s: scales/biases not 2-byte aligned", what);
  return MC_OK;
}

extern "C" int mc_check_quant(const mc_qweights* w) {
  if (!w) return mc_fail(MC_EINVAL, "check_quant: null weights");
  if (w->bits != 4 && w->bits != 6 && w->bits != 8)
    return mc_fail(MC_EINVAL, "unsupported bit width %d", w->bits);
  if (w->group_size <= 0 || w->in_features <= 0 || w->out_features <= 0)
    return mc_fail(MC_EINVAL, "check_quant: non-positive shape");
  // A 16-byte code block must not cross a quantization group (quant.rs:46-53).
  const int per_block = 128 / w->bits;
  if (w->in_features % w->group_size != 0 || (w->bits != 6 && w->group_size % per_block != 0))
    return mc_fail(MC_EINVAL, "in_features %d / group size %d not block-packable at %d bits",
                   w->in_features, w->group_size, w->bits);
  if (w->bits == 6 && w->group_size % 64 != 0)
    return mc_fail(MC_EINVAL, "6-bit group size %d must be a multiple of 64", w->group_size);
  if (!mc_aligned(w->codes, 16))
    return mc_fail(MC_EINVAL, "codes address not 16-aligned; the kernels read codes as 16-byte vectors");
  return MC_OK;
}

extern "C" const char* mc_last_error(void) { return g_err; }

extern "C" const char* mc_version(void) { return "molten_cuda 0.1 sm_100a"; }

extern "C" int mc_create(int device, void* stream, mc_ctx** out) {
  if (!out) return mc_fail(MC_EINVAL, "mc_create: null out");
  *out = nullptr;
  int n = 0;
  MC_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return mc_fail(MC_EINVAL, "mc_create: device %d of %d", device, n);
  MC_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  MC_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return mc_fail(MC_EUNSUPPORTED, "mc_create: device %d is sm_%d%d; this library is built for sm_100a",
                   device, prop.major, prop.minor);
  mc_ctx* c = (mc_ctx*)calloc(1, sizeof(mc_ctx));
  if (!c) return mc_fail(MC_EINVAL, "mc_create: out of host memory");
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  c->l2_bytes = prop.l2CacheSize;
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  c->max_smem_optin = optin;
  // NULL is CUDA's default stream, as everywhere in the runtime API.
  c->stream = (cudaStream_t)stream;
  c->owns_stream = 0;
  *out = c;
  return MC_OK;
}

extern "C" int mc_set_stream(mc_ctx* ctx, void* stream) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_set_stream: null context");
  ctx->stream = (cudaStream_t)stream;
  return MC_OK;
}

extern "C" int mc_set_trace(mc_ctx* ctx, unsigned long long* buf, int n) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_set_trace: null context");
  if (buf && n < 0) return mc_fail(MC_EINVAL, "mc_set_trace: n %d", n);
  ctx->trace = buf;
  ctx->trace_len = buf ? n : 0;
  return MC_OK;
}

extern "C" int mc_set_wait_limit(mc_ctx* ctx, unsigned long long ns) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_set_wait_limit: null context");
  ctx->wait_limit_ns = ns;
  return MC_OK;
}

extern "C" int mc_set_test_flags(mc_ctx* ctx, int flags) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_set_test_flags: null context");
  if (flags & ~(MC_TEST_SKIP_LOGIT_PUBLISH | MC_TEST_SKIP_BARRIER_ARRIVE))
    return mc_fail(MC_EINVAL, "mc_set_test_flags: unknown flags 0x%x", flags);
  ctx->test_flags = flags;
  return MC_OK;
}

extern "C" int mc_set_l2_prefetch(mc_ctx* ctx, const void* p0, size_t n0, const void* p1,
                                  size_t n1) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_set_l2_prefetch: null context");
  ctx->pf_ptr[0] = n0 ? p0 : nullptr;
  ctx->pf_bytes[0] = p0 ? n0 : 0;
  ctx->pf_ptr[1] = n1 ? p1 : nullptr;
  ctx->pf_bytes[1] = p1 ? n1 : 0;
  return MC_OK;
}

namespace {

// dst[i] = src[i] for n 16-byte words; either side may be pinned host memory
// mapped into the device's address space. Chained with programmatic
// dependent launch like the decode kernels: the copy waits for the kernel
// before it, and the next kernel's pre-wait part overlaps it. Loads are
// cache-volatile, so host writes made between graph replays are seen.
__global__ void __launch_bounds__(256) copy16_kernel(uint4* __restrict__ dst,
                                                     const uint4* __restrict__ src, size_t n) {
  mc_pdl_launch_dependents();
  mc_pdl_wait();
  for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (size_t)gridDim.x * 256)
    dst[i] = __ldcv(src + i);
}

// Memory this context's device can read and write at p: its own device
// memory, or page-locked host memory mapped at the same address (UVA).
bool device_addressable(const mc_ctx* ctx, const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeDevice) return a.device == ctx->device;
  if (a.type == cudaMemoryTypeHost) return a.devicePointer == p;
  return false;
}

}  // namespace

extern "C" int mc_copy_async(mc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  MC_REQUIRE(ctx, "copy_async: null context");
  if (bytes == 0) return MC_OK;
  MC_REQUIRE(dst && src, "copy_async: null pointer");
  const uintptr_t d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
  MC_REQUIRE(bytes <= UINTPTR_MAX - (d > s ? d : s), "copy_async: range wraps the address space");
  MC_REQUIRE(d + bytes <= s || s + bytes <= d, "copy_async: overlapping ranges");
  if (bytes % 16 == 0 && mc_aligned(dst, 16) && mc_aligned(src, 16) &&
      device_addressable(ctx, dst) && device_addressable(ctx, src)) {
    const size_t n = bytes / 16;
    size_t blocks = (n + 255) / 256;
    if (blocks > (size_t)ctx->num_sms * 4) blocks = (size_t)ctx->num_sms * 4;
    MC_CUDA(mc_launch_pdl(copy16_kernel, dim3((unsigned)blocks), dim3(256), 0, ctx->stream,
                          static_cast<uint4*>(dst), static_cast<const uint4*>(src), n));
    return mc_after_launch("copy16_kernel");
  }
  MC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, ctx->stream));
  return MC_OK;
}

extern "C" int mc_sync(mc_ctx* ctx) {
  if (!ctx) return mc_fail(MC_EINVAL, "mc_sync: null context");
  if (ctx->ep) return mc_ep_wait(ctx);
  MC_CUDA(cudaStreamSynchronize(ctx->stream));
  MC_CUDA(cudaGetLastError());
  return MC_OK;
}

extern "C" int mc_destroy(mc_ctx* ctx) {
  if (!ctx) return MC_OK;
  mc_ep_release(ctx);
  if (ctx->owns_stream) cudaStreamDestroy(ctx->stream);
  free(ctx);
  return MC_OK;
}
