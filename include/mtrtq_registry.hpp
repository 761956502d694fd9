// The device MatMulQ as a kernel of the reference's own registry.
//
// Header-only; include it where the reference's headers are on the include path
// (include/mtrt), and link libmtrtq.so and the CUDA runtime.
//
// register_device_matmulq(reg) binds ("MatMulQ", DType::kF32) in a reference
// mtrt::KernelRegistry (include/mtrt/registry.h:17-40) to matmulq_device_kernel,
// a plain KernelFn (include/mtrt/op_context.h:13-20) with the reference kernel's
// inputs and preconditions (src/ops/kernels_matmul.cpp:42-74: A f32 [M,K],
// W i8 [K,N], scale f32 [N], C f32 [M,N], all contiguous). A caller that looks
// the op up and calls fn(OpContext) -- the executor's run loop
// (src/runtime/executor.cpp:105-142) or a test -- gets the product from the GPU:
//
//   * the tensors are the reference's host Tensors, so the kernel copies A in and C
//     out around the device product on one stream (mtrtq_matmul_host) and returns
//     when C is written, as the CPU kernel it replaces does;
//   * each weight is packed to the device layout once, on its first call, and kept
//     by the address of its int8 data: the reference binds weights at executor
//     construction and never writes them afterwards, which this relies on;
//   * the staging workspace of each (M, K, N) is allocated on its first call;
//     a caller that must not allocate inside run() calls once at setup (or uses
//     mtrtq_matmul with a planned arena, include/mtrtq_cuda.hpp).
//
// Errors abort with the library's message, as the reference's CUDA backend does
// on a failed CUDA call (backends/cuda/kernels.cu:13-21).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>

#include "mtrt/op_context.h"
#include "mtrt/registry.h"
#include "mtrt/tensor.h"
#include "mtrtq.h"
#include "mtrtq_cuda.hpp"

namespace mtrtq {

class DeviceMatmulqState {
 public:
  static DeviceMatmulqState& instance() {
    static DeviceMatmulqState s;
    return s;
  }

  int mode = MTRTQ_MODE_FP32;

  const PackedWeight& weight(const int8_t* q, const float* scale, int64_t K, int64_t N) {
    std::lock_guard<std::mutex> lk(mu_);
    auto key = std::make_tuple(static_cast<const void*>(q), K, N);
    auto it = weights_.find(key);
    if (it == weights_.end())
      it = weights_.emplace(key, std::make_unique<PackedWeight>(q, scale, K, N)).first;
    return *it->second;
  }

  void* workspace(int64_t M, int64_t K, int64_t N, size_t* bytes) {
    std::lock_guard<std::mutex> lk(mu_);
    auto key = std::make_tuple(M, K, N, mode);
    auto it = ws_.find(key);
    if (it == ws_.end()) {
      const int64_t need = mtrtq_host_workspace_bytes(M, K, N, mode);
      if (need < 0) check_or_abort(MTRTQ_ERR_INVALID_ARG, "mtrtq_host_workspace_bytes");
      void* p = nullptr;
      cuda_or_abort(cudaMalloc(&p, static_cast<size_t>(need)), "cudaMalloc(workspace)");
      cuda_or_abort(cudaMemset(p, 0, static_cast<size_t>(need)), "cudaMemset(workspace)");
      it = ws_.emplace(key, Buffer{p, static_cast<size_t>(need)}).first;
    }
    *bytes = it->second.bytes;
    return it->second.ptr;
  }

  ~DeviceMatmulqState() {
    for (auto& kv : ws_) cudaFree(kv.second.ptr);
  }

 private:
  struct Buffer {
    void* ptr;
    size_t bytes;
  };
  std::mutex mu_;
  std::map<std::tuple<const void*, int64_t, int64_t>, std::unique_ptr<PackedWeight>> weights_;
  std::map<std::tuple<int64_t, int64_t, int64_t, int>, Buffer> ws_;
};

// KernelFn for ("MatMulQ", kF32): C = A x dequant(W, scale) on the GPU.
inline void matmulq_device_kernel(const mtrt::OpContext& ctx) {
  if (ctx.inputs.size() != 3 || ctx.outputs.size() != 1)
    check_or_abort(MTRTQ_ERR_INVALID_ARG, "MatMulQ expects A, W_int8, scale and one output");
  const mtrt::Tensor& A = *ctx.inputs[0];
  const mtrt::Tensor& W = *ctx.inputs[1];
  const mtrt::Tensor& S = *ctx.inputs[2];
  mtrt::Tensor& C = *ctx.outputs[0];
  if (A.dtype() != mtrt::DType::kF32 || W.dtype() != mtrt::DType::kI8 || S.dtype() != mtrt::DType::kF32 ||
      C.dtype() != mtrt::DType::kF32 || A.rank() != 2 || W.rank() != 2 || C.rank() != 2 ||
      !A.is_contiguous() || !W.is_contiguous() || !C.is_contiguous())
    check_or_abort(MTRTQ_ERR_INVALID_ARG, "MatMulQ: A f32 [M,K], W i8 [K,N], C f32 [M,N], contiguous");
  const int64_t M = A.shape()[0], K = A.shape()[1], N = W.shape()[1];
  if (W.shape()[0] != K || C.shape()[0] != M || C.shape()[1] != N || S.numel() != N)
    check_or_abort(MTRTQ_ERR_INVALID_ARG, "MatMulQ shapes disagree");
  DeviceMatmulqState& st = DeviceMatmulqState::instance();
  const PackedWeight& pw = st.weight(W.data<int8_t>(), S.data<float>(), K, N);
  size_t ws_bytes = 0;
  void* ws = st.workspace(M, K, N, &ws_bytes);
  check_or_abort(mtrtq_matmul_host(A.data<float>(), pw.packed(), pw.scale(), nullptr, C.data<float>(), M, K,
                                   N, st.mode, ws, ws_bytes, /*blocking=*/1, /*stream=*/nullptr),
                 "MatMulQ (device)");
}

// Binds ("MatMulQ", kF32) to the device kernel; mode MTRTQ_MODE_FP32 (the
// reference's arithmetic, within 1e-4) or MTRTQ_MODE_BF16.
inline void register_device_matmulq(mtrt::KernelRegistry& reg, int mode = MTRTQ_MODE_FP32) {
  DeviceMatmulqState::instance().mode = mode;
  reg.register_kernel("MatMulQ", mtrt::DType::kF32, &matmulq_device_kernel);
}

}  // namespace mtrtq
