// The C++ host mirror on a B200: a Q4 GEMV and a Q6 head + argmax through
// molten::kernels against expected outputs the test harness computed with the
// CPU oracle (raw little-endian files in argv[1]). Bit-exact comparison.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "molten_b200.hpp"

using molten::DType;
using molten::QuantWeights;
using molten::Tensor;

static std::vector<char> slurp(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

static void* upload(const std::vector<char>& h) {
  void* d = nullptr;
  if (cudaMalloc(&d, h.size()) != cudaSuccess) throw std::runtime_error("cudaMalloc");
  if (cudaMemcpy(d, h.data(), h.size(), cudaMemcpyHostToDevice) != cudaSuccess)
    throw std::runtime_error("cudaMemcpy");
  return d;
}

static QuantWeights load_q(const std::string& dir, const std::string& name, int n, int k, int bits) {
  QuantWeights w;
  w.codes = Tensor(upload(slurp(dir + "/" + name + "_codes.bin")), {n, k * bits / 32}, DType::U32);
  w.scales = Tensor(upload(slurp(dir + "/" + name + "_scales.bin")), {n, k / 64}, DType::BF16);
  w.biases = Tensor(upload(slurp(dir + "/" + name + "_biases.bin")), {n, k / 64}, DType::BF16);
  w.group_size = 64;
  w.bits = bits;
  return w;
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const std::string dir = argv[1];
  int failures = 0;
  try {
    molten::Context ctx(0);
    {  // Q4 GEMV 2048 x 2048 at batch 3
      const int n = 2048, k = 2048, b = 3;
      QuantWeights w = load_q(dir, "q4", n, k, 4);
      Tensor x(upload(slurp(dir + "/q4_x.bin")), {b, k}, DType::BF16);
      void* yd = nullptr;
      cudaMalloc(&yd, (size_t)b * n * 2);
      Tensor y(yd, {b, n}, DType::BF16);
      molten::kernels::gemv_quant(ctx, w, x, y);
      ctx.commit_wait();
      std::vector<char> got((size_t)b * n * 2), want = slurp(dir + "/q4_want.bin");
      cudaMemcpy(got.data(), yd, got.size(), cudaMemcpyDeviceToHost);
      if (want.size() != got.size() || std::memcmp(got.data(), want.data(), got.size()) != 0) {
        std::printf("FAIL q4 gemv differs from the oracle\n");
        ++failures;
      }
    }
    {  // Q6 head 65536 x 2048 + argmax at batch 2
      const int n = 65536, k = 2048, b = 2;
      QuantWeights w = load_q(dir, "q6", n, k, 6);
      Tensor x(upload(slurp(dir + "/q6_x.bin")), {b, k}, DType::BF16);
      void* kd = nullptr;
      cudaMalloc(&kd, (size_t)b * 8);
      cudaMemset(kd, 0, (size_t)b * 8);
      Tensor keys(kd, {b}, DType::U64);
      molten::kernels::gemv_head_argmax(ctx, w, x, keys);
      ctx.commit_wait();
      std::vector<char> got((size_t)b * 8), want = slurp(dir + "/q6_keys.bin");
      cudaMemcpy(got.data(), kd, got.size(), cudaMemcpyDeviceToHost);
      if (want.size() != got.size() || std::memcmp(got.data(), want.data(), got.size()) != 0) {
        std::printf("FAIL q6 head keys differ from the oracle\n");
        ++failures;
      }
    }
  } catch (const std::exception& e) {
    std::printf("FAIL exception: %s\n", e.what());
    ++failures;
  }
  std::printf("%s (%d failures)\n", failures ? "FAILED" : "ok", failures);
  return failures ? 1 : 0;
}
