// Runs the reference's own int8 packer: the body of TEST(Golden, MatMulQ) in the
// reference's tests/golden_kernel_test.cpp:155-175 (packer loop at :163-170),
// compiled unmodified against oracle/gtest_shim. TEST INFRASTRUCTURE ONLY.
//
//   ref_packer_pin GOLDENS_DIR OUT_PREFIX
//
// GOLDENS_DIR holds op_matmul_a.npy, op_matmul_b.npy and op_matmul_out.npy (the
// reference's fixtures, or seeded inputs written in the same format). The test
// body packs B per column, then calls the registry's MatMulQ; that lookup is
// routed here (build_ref.sh renames register_builtin_kernels in the test's
// translation unit), so the packed weights and scales the test built are written
// to OUT_PREFIX.q (int8 [K,N]) and OUT_PREFIX.s (f32 [N]) before the reference
// kernel runs on them. When the output tensor the test allocated ([2,5]) fits the
// product, the reference kernel's output goes to OUT_PREFIX.c as well; for other
// shapes the kernel is not run (the test's fixed output would be too small).
// Prints "checks_failed=<n>" (the test's own assertions) and exits 0 when the
// test ran.
#include <cstdio>
#include <string>
#include <vector>

#include <gtest/gtest.h>

#include "mtrt/node.h"
#include "mtrt/op_context.h"
#include "mtrt/registry.h"
#include "mtrt/tensor.h"

namespace {

std::string g_goldens_dir;
std::string g_out_prefix;
mtrt::KernelFn g_matmulq = nullptr;
bool g_dumped = false;

bool write_file(const std::string& path, const void* data, size_t bytes) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return false;
  const bool ok = std::fwrite(data, 1, bytes, f) == bytes;
  return std::fclose(f) == 0 && ok;
}

// MatMulQ as registered for the test: record the packed inputs, then run the
// reference kernel when the test's output tensor is large enough.
void capture_matmulq(const mtrt::OpContext& ctx) {
  const mtrt::Tensor& A = *ctx.inputs[0];
  const mtrt::Tensor& W = *ctx.inputs[1];
  const mtrt::Tensor& s = *ctx.inputs[2];
  mtrt::Tensor& C = *ctx.outputs[0];
  const int64_t M = A.shape()[0], K = W.shape()[0], N = W.shape()[1];
  g_dumped = write_file(g_out_prefix + ".q", W.data<int8_t>(), static_cast<size_t>(K * N)) &&
             write_file(g_out_prefix + ".s", s.data<float>(), static_cast<size_t>(N) * sizeof(float));
  if (C.numel() == M * N) {
    g_matmulq(ctx);
    write_file(g_out_prefix + ".c", C.data<float>(), static_cast<size_t>(M * N) * sizeof(float));
  }
}

}  // namespace

// The goldens directory, read by the test's load_golden() (MTRT_GOLDENS_DIR).
const char* pin_goldens_dir() { return g_goldens_dir.c_str(); }

namespace mtrt {
// Called by the test in place of register_builtin_kernels.
void pin_register_builtin_kernels(KernelRegistry& reg) {
  register_builtin_kernels(reg);
  g_matmulq = reg.lookup("MatMulQ", DType::kF32);
  reg.register_kernel("MatMulQ", DType::kF32, &capture_matmulq);
}
}  // namespace mtrt

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s GOLDENS_DIR OUT_PREFIX\n", argv[0]);
    return 2;
  }
  g_goldens_dir = argv[1];
  g_out_prefix = argv[2];
  const int failed = ::testing::shim::run("Golden.MatMulQ");
  if (failed < 0) {
    std::fprintf(stderr, "Golden.MatMulQ is not registered\n");
    return 3;
  }
  if (!g_dumped) {
    std::fprintf(stderr, "the test did not reach MatMulQ\n");
    return 4;
  }
  std::printf("checks_failed=%d\n", failed);
  return 0;
}
