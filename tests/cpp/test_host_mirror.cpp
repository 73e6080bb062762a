// Checks of the C++ host mirror (include/molten_b200.hpp) that need no GPU:
// each `ensure!`-style check throws molten::Error with the reference's
// message before anything reaches the C ABI, and a well-formed call does reach
// it (here with a null context, which the ABI rejects with its own message).
#include <cstdio>
#include <cstring>
#include <string>

#include "molten_b200.hpp"

using molten::DType;
using molten::Error;
using molten::QuantWeights;
using molten::Tensor;

static int failures = 0;

template <typename F>
static void expect_error(const char* what, int code, const char* needle, F&& f) {
  try {
    f();
    std::printf("FAIL %s: no error\n", what);
    ++failures;
  } catch (const Error& e) {
    if (e.code() != code || std::strstr(e.what(), needle) == nullptr) {
      std::printf("FAIL %s: code %d message '%s'\n", what, e.code(), e.what());
      ++failures;
    }
  }
}

int main() {
  // never dereferenced: every call below stops at a check
  void* p = reinterpret_cast<void*>(0x1000);
  molten::Context ctx = molten::Context::wrap(nullptr);

  QuantWeights w{Tensor(p, {2048, 256}, DType::U32), Tensor(p, {2048, 32}, DType::BF16),
                 Tensor(p, {2048, 32}, DType::BF16), 64, 4};
  const Tensor x(p, {2, 2048}, DType::BF16), y(p, {2, 2048}, DType::BF16);

  expect_error("gemv shape", MC_EINVAL, "gemv shape mismatch",
               [&] { molten::kernels::gemv_quant(ctx, w, Tensor(p, {2, 2000}, DType::BF16), y); });
  expect_error("gemv dtype", MC_EINVAL, "gemv BF16 only",
               [&] { molten::kernels::gemv_quant(ctx, w, Tensor(p, {2, 2048}, DType::F32), y); });
  QuantWeights bad = w;
  bad.codes.dtype = DType::F32;
  expect_error("check_quant codes", MC_EINVAL, "codes must be U32",
               [&] { molten::kernels::gemv_quant(ctx, bad, x, y); });
  bad = w;
  bad.scales = Tensor(p, {2048, 16}, DType::BF16);
  expect_error("check_quant scales", MC_EINVAL, "scales/biases shape mismatch",
               [&] { molten::kernels::gemv_quant(ctx, bad, x, y); });
  // well-formed: the ABI itself answers
  expect_error("gemv reaches the ABI", MC_EINVAL, "null context",
               [&] { molten::kernels::gemv_quant(ctx, w, x, y); });
  if (w.in_features() != 2048 || w.out_features() != 2048) {
    std::printf("FAIL QuantWeights dims %d %d\n", w.in_features(), w.out_features());
    ++failures;
  }

  const Tensor router(p, {64, 2048}, DType::F32);
  const Tensor ids(p, {2, 4}, DType::U32), wts(p, {2, 4}, DType::BF16), ctr(p, {2}, DType::U32);
  expect_error("router logits", MC_EINVAL, "router logits shape", [&] {
    molten::kernels::router_addnorm_route(ctx, x, &y, Tensor(p, {2048}, DType::BF16), y, y, router,
                                          Tensor(p, {2, 63}, DType::F32), nullptr, ids, wts, ctr);
  });
  expect_error("router counter", MC_EINVAL, "route counter shape", [&] {
    molten::kernels::router_addnorm_route(ctx, x, &y, Tensor(p, {2048}, DType::BF16), y, y, router,
                                          Tensor(p, {2, 64}, DType::F32), nullptr, ids, wts,
                                          Tensor(p, {1}, DType::U32));
  });

  const Tensor a(p, {300, 2048}, DType::BF16), ws(p, {8}, DType::U32);
  expect_error("gemm output", MC_EINVAL, "gemm output shape", [&] {
    molten::kernels::gemm_q4(ctx, a, w, Tensor(p, {300, 2047}, DType::BF16), ws);
  });
  expect_error("gemm reaches the ABI", MC_EINVAL, "null context", [&] {
    molten::kernels::gemm_q4(ctx, a, w, Tensor(p, {300, 2048}, DType::BF16), ws);
  });
  expect_error("head keys", MC_EINVAL, "head keys shape", [&] {
    molten::kernels::gemv_head_argmax(ctx, w, x, Tensor(p, {2}, DType::U32));
  });
  expect_error("copy reaches the ABI", MC_EINVAL, "null context",
               [&] { molten::kernels::copy_async(ctx, p, p, 16); });

  // a real context: an error without a GPU, a working handle with one
  try {
    molten::Context real(0);
    real.commit_wait();
    std::printf("context on device 0: ok\n");
  } catch (const Error& e) {
    if (e.code() != MC_ECUDA && e.code() != MC_EINVAL) {
      std::printf("FAIL context without a GPU: code %d '%s'\n", e.code(), e.what());
      ++failures;
    }
  }

  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
