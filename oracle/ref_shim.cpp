// C entry points over the reference's own MatMulQ code path.
//
// TEST INFRASTRUCTURE ONLY. oracle/build_ref.sh compiles this file together
// with the reference's unmodified sources (tensor, registry, CPU kernels, CPU
// GEMM ladder and thread pool) into oracle/_ref/libmtrt_ref.so. It is used to
// pin the C restatement (oracle/matmulq_oracle.c) and as the timed CPU
// baseline; the product library never links it.
//
// Each call goes through the reference's public kernel interface exactly as
// its executor and its Golden.MatMulQ test do (src/runtime/executor.cpp:105-142,
// tests/golden_kernel_test.cpp:18-29): KernelRegistry::lookup(op, kF32) then
// fn(OpContext{inputs, outputs, node}).
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "backends/cpu/gemm.h"
#include "mtrt/node.h"
#include "mtrt/op_context.h"
#include "mtrt/registry.h"
#include "mtrt/tensor.h"

namespace {

const mtrt::KernelRegistry& registry() {
  static const mtrt::KernelRegistry reg = [] {
    mtrt::KernelRegistry r;
    mtrt::register_builtin_kernels(r);
    return r;
  }();
  return reg;
}

// Wraps caller memory in a reference Tensor without copying: view() of an
// owning 1-element tensor is not possible for foreign memory, so the
// reference's own owning() + memcpy is used (the kernel reads the copy).
mtrt::Tensor make_tensor(mtrt::DType dt, std::vector<int64_t> shape, const void* src) {
  mtrt::Tensor t = mtrt::Tensor::owning(dt, shape);
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  if (src) {
    void* dst = dt == mtrt::DType::kI8 ? static_cast<void*>(t.data<int8_t>())
                                       : static_cast<void*>(t.data<float>());
    std::memcpy(dst, src, static_cast<size_t>(n) * mtrt::dtype_size(dt));
  }
  return t;
}

}  // namespace

extern "C" {

// C[M,N] = MatMulQ(A[M,K] f32, W[K,N] i8, scale[N] f32) via the registry.
// Returns 0 on success, 1 if the kernel is not registered.
int ref_matmulq(const float* A, const int8_t* W, const float* scale, float* C, int64_t M,
                int64_t K, int64_t N) {
  mtrt::KernelFn fn = registry().lookup("MatMulQ", mtrt::DType::kF32);
  if (!fn) return 1;
  mtrt::Tensor tA = make_tensor(mtrt::DType::kF32, {M, K}, A);
  mtrt::Tensor tW = make_tensor(mtrt::DType::kI8, {K, N}, W);
  mtrt::Tensor tS = make_tensor(mtrt::DType::kF32, {N}, scale);
  mtrt::Tensor tC = mtrt::Tensor::owning(mtrt::DType::kF32, {M, N});
  std::vector<const mtrt::Tensor*> ins{&tA, &tW, &tS};
  std::vector<mtrt::Tensor*> outs{&tC};
  mtrt::Node node;
  node.op_type = "MatMulQ";
  fn(mtrt::OpContext{ins, outs, node});
  std::memcpy(C, tC.data<float>(), static_cast<size_t>(M * N) * sizeof(float));
  return 0;
}

// A MatMulQ call prepared once -- its reference Tensors built and the kernel looked
// up, as the reference executor does at construction (src/runtime/executor.cpp:
// 51-123) -- so that timing ref_matmulq_run measures the kernel call alone, as the
// executor's run loop makes it (:139-142).
struct RefMatmulq {
  mtrt::KernelFn fn;
  mtrt::Tensor A, W, S, C;
  mtrt::Node node;
};

void* ref_matmulq_prepare(const float* A, const int8_t* W, const float* scale, int64_t M, int64_t K,
                          int64_t N) {
  mtrt::KernelFn fn = registry().lookup("MatMulQ", mtrt::DType::kF32);
  if (!fn) return nullptr;
  RefMatmulq* h = new RefMatmulq{fn, make_tensor(mtrt::DType::kF32, {M, K}, A),
                                 make_tensor(mtrt::DType::kI8, {K, N}, W),
                                 make_tensor(mtrt::DType::kF32, {N}, scale),
                                 mtrt::Tensor::owning(mtrt::DType::kF32, {M, N}), mtrt::Node{}};
  h->node.op_type = "MatMulQ";
  return h;
}

void ref_matmulq_run(void* handle) {
  RefMatmulq* h = static_cast<RefMatmulq*>(handle);
  std::vector<const mtrt::Tensor*> ins{&h->A, &h->W, &h->S};
  std::vector<mtrt::Tensor*> outs{&h->C};
  h->fn(mtrt::OpContext{ins, outs, h->node});
}

void ref_matmulq_output(void* handle, float* C) {
  RefMatmulq* h = static_cast<RefMatmulq*>(handle);
  std::memcpy(C, h->C.data<float>(), static_cast<size_t>(h->C.numel()) * sizeof(float));
}

void ref_matmulq_free(void* handle) { delete static_cast<RefMatmulq*>(handle); }

// Y[M,N] = Y + b[N] through the registry's "Add" kernel (bias broadcast form).
int ref_add_bias(float* Y, const float* b, int64_t M, int64_t N) {
  mtrt::KernelFn fn = registry().lookup("Add", mtrt::DType::kF32);
  if (!fn) return 1;
  mtrt::Tensor tY = make_tensor(mtrt::DType::kF32, {M, N}, Y);
  mtrt::Tensor tB = make_tensor(mtrt::DType::kF32, {N}, b);
  mtrt::Tensor tO = mtrt::Tensor::owning(mtrt::DType::kF32, {M, N});
  std::vector<const mtrt::Tensor*> ins{&tY, &tB};
  std::vector<mtrt::Tensor*> outs{&tO};
  mtrt::Node node;
  node.op_type = "Add";
  fn(mtrt::OpContext{ins, outs, node});
  std::memcpy(Y, tO.data<float>(), static_cast<size_t>(M * N) * sizeof(float));
  return 0;
}

// The reference's fp32 "NEON / multithreaded" dispatcher (backends/cpu/gemm.cpp:288-302)
// on caller memory: C[M,N] = A[M,K] @ B[K,N]. On x86-64 its NEON step is the scalar
// packed fallback (gemm.cpp:251-254); it threads over rows when M >= 32.
void ref_gemm_auto(const float* A, const float* B, float* C, int M, int N, int K) {
  mtrt::cpu::gemm_auto(A, B, C, M, N, K);
}

// Threads the reference's ThreadPool uses (backends/cpu/thread_pool.cpp:8-9).
int ref_hardware_threads(void) {
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : static_cast<int>(n);
}

}  // extern "C"
