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

  // the rest of the op surface: one failing check each
  namespace K = molten::kernels;
  QuantWeights gate = w, up = w;  // [64 * 32][2048]: expert width 32
  gate.codes.shape = {2048, 256};
  expect_error("token tail", MC_EINVAL, "token tail shapes", [&] {
    K::token_tail(ctx, Tensor(p, {2}, DType::U64), Tensor(p, {3}, DType::U32), nullptr, nullptr,
                  nullptr, nullptr);
  });
  expect_error("token tail embed", MC_EINVAL, "needs norm_w", [&] {
    const Tensor emb(p, {100, 2048}, DType::BF16);
    K::token_tail(ctx, Tensor(p, {2}, DType::U64), Tensor(p, {2}, DType::U32), &emb, nullptr,
                  nullptr, nullptr);
  });
  expect_error("argmax out", MC_EINVAL, "argmax out shape", [&] {
    K::argmax_bf16(ctx, Tensor(p, {3, 65536}, DType::BF16), Tensor(p, {2}, DType::U32));
  });
  expect_error("gather act ids", MC_EINVAL, "gather act ids shape", [&] {
    K::gemv_gather_act(ctx, gate, up, x, Tensor(p, {2, 3}, DType::U32),
                       Tensor(p, {2, 4, 32}, DType::BF16));
  });
  expect_error("gather act out", MC_EINVAL, "gather act output shape", [&] {
    K::gemv_gather_act(ctx, gate, up, x, ids, Tensor(p, {2, 4, 31}, DType::BF16));
  });
  expect_error("down out", MC_EINVAL, "down output shape", [&] {
    QuantWeights d{Tensor(p, {64 * 2048, 16}, DType::U32), Tensor(p, {64 * 2048, 2}, DType::BF16),
                   Tensor(p, {64 * 2048, 2}, DType::BF16), 64, 4};
    K::gemv_gather_down_combine4(ctx, d, Tensor(p, {2, 4, 128}, DType::BF16), ids, wts,
                                 Tensor(p, {2, 2047}, DType::BF16));
  });
  expect_error("decode workspace", MC_EINVAL, "decode workspace too small", [&] {
    const Tensor nw(p, {2048}, DType::BF16);
    K::moe_decode_layer(ctx, Tensor(p, {1, 2048}, DType::BF16), nullptr, nw,
                        Tensor(p, {1, 2048}, DType::BF16), Tensor(p, {1, 2048}, DType::BF16),
                        router, Tensor(p, {1, 64}, DType::F32), nullptr,
                        Tensor(p, {1, 4}, DType::U32), Tensor(p, {1, 4}, DType::BF16), gate, up, w,
                        Tensor(p, {1, 2048}, DType::BF16), Tensor(p, {4}, DType::U32), 64);
  });
  expect_error("grouped out", MC_EINVAL, "grouped GEMM output shape", [&] {
    K::gemm_q4_grouped_mlx(ctx, a, w, Tensor(p, {300, 31}, DType::BF16),
                           Tensor(p, {16, 4}, DType::U32), Tensor(p, {1}, DType::U32), 64);
  });
  expect_error("grouped gu out", MC_EINVAL, "grouped gate/up output shape", [&] {
    K::gemm_q4_grouped_mlx_gu(ctx, a, gate, up, Tensor(p, {300, 33}, DType::BF16),
                              Tensor(p, {16, 4}, DType::U32), Tensor(p, {1}, DType::U32), 64);
  });
  expect_error("gather rows", MC_EINVAL, "gather shapes", [&] {
    K::gather_rows_bf16(ctx, Tensor(p, {100, 2048}, DType::BF16), Tensor(p, {5}, DType::U32),
                        Tensor(p, {5, 2047}, DType::BF16));
  });
  expect_error("silu_mul dtype", MC_EINVAL, "silu_mul BF16 only", [&] {
    K::silu_mul_bf16(ctx, Tensor(p, {8}, DType::F32), Tensor(p, {8}, DType::BF16),
                     Tensor(p, {8}, DType::BF16));
  });
  expect_error("combine slots", MC_EINVAL, "combine slot shapes", [&] {
    K::moe_combine_rows(ctx, Tensor(p, {16, 2048}, DType::BF16), Tensor(p, {3, 4}, DType::U32),
                        Tensor(p, {4, 4}, DType::BF16), Tensor(p, {4, 2048}, DType::BF16));
  });
  expect_error("prefill logits", MC_EINVAL, "prefill logits shape", [&] {
    K::moe_prefill(ctx, Tensor(p, {16, 2048}, DType::BF16), Tensor(p, {16, 63}, DType::F32), gate,
                   up, w, Tensor(p, {1024}, DType::U32), Tensor(p, {16, 2048}, DType::BF16), 64);
  });
  expect_error("prefill reaches the ABI", MC_EINVAL, "null context", [&] {
    K::moe_prefill(ctx, Tensor(p, {16, 2048}, DType::BF16), Tensor(p, {16, 64}, DType::F32), gate,
                   up, w, Tensor(p, {1024}, DType::U32), Tensor(p, {16, 2048}, DType::BF16), 64);
  });

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

  // decode neighbours and the sampling draw: each check fires, then the ABI
  {
    QuantWeights q{Tensor(p, {2048, 256}, DType::U32), Tensor(p, {2048, 32}, DType::BF16),
                   Tensor(p, {2048, 32}, DType::BF16), 64, 4};
    QuantWeights kv{Tensor(p, {512, 256}, DType::U32), Tensor(p, {512, 32}, DType::BF16),
                    Tensor(p, {512, 32}, DType::BF16), 64, 4};
    const Tensor x1(p, {2048}, DType::BF16), qo(p, {2048}, DType::BF16), ko(p, {512}, DType::BF16);
    expect_error("proj3 cache shape", MC_EINVAL, "proj3 KV cache shape", [&] {
      molten::kernels::proj3_gemv_scatter(ctx, q, kv, kv, x1, qo, ko,
                                          Tensor(p, {8, 16, 64}, DType::BF16), 16);
    });
    expect_error("proj3 reaches the ABI", MC_EINVAL, "null context", [&] {
      molten::kernels::proj3_gemv_scatter(ctx, q, kv, kv, x1, qo, ko,
                                          Tensor(p, {8, 16, 64}, DType::BF16), 3);
    });
    QuantWeights c3{Tensor(p, {3 * 64, 256}, DType::U32), Tensor(p, {3 * 64, 32}, DType::BF16),
                    Tensor(p, {3 * 64, 32}, DType::BF16), 64, 4};
    expect_error("conv3 state shape", MC_EINVAL, "conv3 state shape", [&] {
      molten::kernels::conv3_gemv(ctx, c3, x1, Tensor(p, {64, 3}, DType::BF16),
                                  Tensor(p, {3, 64}, DType::BF16), Tensor(p, {64}, DType::BF16),
                                  Tensor(p, {2, 64}, DType::BF16));
    });
    expect_error("gu_act rows", MC_EINVAL, "dense gate/up rows", [&] {
      molten::kernels::gemv_gu_act(ctx, q, q, x1, Tensor(p, {100}, DType::BF16));
    });
    mc_sampling sp{1.0f, 0, 1.0f, 1.5f, 7};
    expect_error("sampling needs the seen set", MC_EINVAL, "needs the seen set", [&] {
      molten::kernels::sample_draw(ctx, Tensor(p, {65536}, DType::BF16), nullptr, sp, 0,
                                   Tensor(p, {1}, DType::U64), Tensor(p, {64}, DType::U32));
    });
  }
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
