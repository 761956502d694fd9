// The drop-in, as the reference sees it: the device MatMulQ registered into the
// reference's own mtrt::KernelRegistry (include/mtrtq_registry.hpp) and reached
// through lookup("MatMulQ", kF32) -> fn(OpContext), the way its executor and its
// tests call kernels (src/runtime/executor.cpp:105-142).
//
//   registry_drop_in GOLDENS_DIR
//
// 1. The reference's TEST(Golden, MatMulQ) (tests/golden_kernel_test.cpp:155-175),
//    compiled unmodified against the local gtest stand-in, runs with its registry
//    call redirected here: the reference's builtin kernels are registered, then
//    ("MatMulQ", kF32) is rebound to the device kernel. The test packs its fixture
//    with its own packer lines, calls the kernel through the registry and checks
//    the result with its own 0.05 bar. GOLDENS_DIR holds op_matmul_{a,b,out}.npy.
// 2. Seeded shapes: the same OpContext goes to the reference's CPU kernel and to
//    the device kernel (MTRTQ_MODE_FP32); the outputs must agree within
//    |d| <= 1e-4 * (|ref| + rms(ref)) element-wise and 1e-4 * max|ref| overall.
// Prints one line per check and exits 0 only if all pass.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include <gtest/gtest.h>

#include "mtrt/node.h"
#include "mtrt/op_context.h"
#include "mtrt/registry.h"
#include "mtrt/tensor.h"
#include "mtrtq_registry.hpp"

namespace {
std::string g_goldens_dir;
}

const char* pin_goldens_dir() { return g_goldens_dir.c_str(); }

namespace mtrt {
// Called by the reference's test in place of register_builtin_kernels.
void pin_register_builtin_kernels(KernelRegistry& reg) {
  register_builtin_kernels(reg);
  mtrtq::register_device_matmulq(reg, MTRTQ_MODE_FP32);
}
}  // namespace mtrt

namespace {

// C = MatMulQ(A, W, s) through `reg`.
void run_matmulq(const mtrt::KernelRegistry& reg, const mtrt::Tensor& A, const mtrt::Tensor& W,
                 const mtrt::Tensor& s, mtrt::Tensor& C) {
  mtrt::KernelFn fn = reg.lookup("MatMulQ", mtrt::DType::kF32);
  std::vector<const mtrt::Tensor*> ins{&A, &W, &s};
  std::vector<mtrt::Tensor*> outs{&C};
  mtrt::Node node;
  node.op_type = "MatMulQ";
  fn(mtrt::OpContext{ins, outs, node});
}

bool seeded_case(int64_t M, int64_t K, int64_t N, unsigned seed) {
  std::mt19937 gen(seed);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  mtrt::Tensor A = mtrt::Tensor::owning(mtrt::DType::kF32, {M, K});
  mtrt::Tensor W = mtrt::Tensor::owning(mtrt::DType::kI8, {K, N});
  mtrt::Tensor s = mtrt::Tensor::owning(mtrt::DType::kF32, {N});
  std::vector<float> Wf(static_cast<size_t>(K * N));
  for (auto& v : Wf) v = 0.02f * nd(gen);
  for (int64_t i = 0; i < M * K; ++i) A.data<float>()[i] = nd(gen);
  // The reference packer (tests/golden_kernel_test.cpp:163-170).
  for (int64_t j = 0; j < N; ++j) {
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) amax = std::max(amax, std::abs(Wf[k * N + j]));
    const float sc = amax / 127.0f;
    s.data<float>()[j] = sc;
    for (int64_t k = 0; k < K; ++k)
      W.data<int8_t>()[k * N + j] = static_cast<int8_t>(std::lround(Wf[k * N + j] / sc));
  }
  mtrt::KernelRegistry cpu, dev;
  mtrt::register_builtin_kernels(cpu);
  mtrt::register_builtin_kernels(dev);
  mtrtq::register_device_matmulq(dev, MTRTQ_MODE_FP32);
  mtrt::Tensor Cr = mtrt::Tensor::owning(mtrt::DType::kF32, {M, N});
  mtrt::Tensor Cd = mtrt::Tensor::owning(mtrt::DType::kF32, {M, N});
  run_matmulq(cpu, A, W, s, Cr);
  run_matmulq(dev, A, W, s, Cd);
  run_matmulq(dev, A, W, s, Cd);  // again: the packed weight and workspace are reused
  const float* r = Cr.data<float>();
  const float* d = Cd.data<float>();
  double rms = 0.0, mx = 0.0, worst_norm = 0.0, worst_elem = 0.0;
  for (int64_t i = 0; i < M * N; ++i) {
    rms += double(r[i]) * r[i];
    mx = std::max(mx, std::abs(double(r[i])));
  }
  rms = std::sqrt(rms / double(M * N));
  for (int64_t i = 0; i < M * N; ++i) {
    const double e = std::abs(double(d[i]) - r[i]);
    worst_norm = std::max(worst_norm, e / mx);
    worst_elem = std::max(worst_elem, e / (std::abs(double(r[i])) + rms));
  }
  const bool ok = std::isfinite(worst_norm) && worst_norm <= 1e-4 && worst_elem <= 1e-4;
  std::printf("seeded %lldx%lldx%lld: normwise %.3e element-wise %.3e %s\n", (long long)M, (long long)K,
              (long long)N, worst_norm, worst_elem, ok ? "ok" : "FAIL");
  return ok;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s GOLDENS_DIR\n", argv[0]);
    return 2;
  }
  g_goldens_dir = argv[1];
  bool all = true;
  const int failed = ::testing::shim::run("Golden.MatMulQ");
  std::printf("Golden.MatMulQ through the reference registry (device kernel): %d failed checks %s\n",
              failed, failed == 0 ? "ok" : "FAIL");
  all &= failed == 0;
  const int64_t shapes[][3] = {{2, 3, 5}, {5, 100, 129}, {1, 768, 2304}, {8, 768, 50257}, {64, 768, 3072}};
  unsigned seed = 1;
  for (const auto& sh : shapes) all &= seeded_case(sh[0], sh[1], sh[2], seed++);
  return all ? 0 : 1;
}
