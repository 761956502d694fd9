// C++ host adapter over the mtrtq C ABI for the reference's CUDA backend.
//
// Header-only; needs include/mtrtq.h, cuda_runtime.h and libmtrtq.so at link time.
//
//  * mtrt::cuda::matmul_q8(...) -- a raw-device-pointer launcher with the shape and
//    calling convention of the reference's other CUDA launchers
//    (backends/cuda/kernels.h:11-76: device pointers, row-major, default stream,
//    abort with a message on error as CE_CK / CUDA_CHECK do,
//    backends/cuda/cuda_executor.cpp:19-27, backends/cuda/kernels.cu:13-21).
//    It is what a `MatMulQ` branch of CudaExecutor::run calls
//    (backends/cuda/cuda_executor.cpp:99-155, which throws on MatMulQ today).
//  * mtrtq::PackedWeight -- the construction-time upload of one int8 [K,N] weight
//    and its scales (cf. the weight upload at backends/cuda/cuda_executor.cpp:61-72),
//    pre-packed to the device layout once.
//  * mtrtq::WorkspacePool -- per-device scratch reserved at setup, so launches
//    never allocate (the reference's run() contract, include/mtrt/executor.h:31-33).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "mtrtq.h"

namespace mtrtq {

// Abort with the library's message, the reference CUDA backend's error behaviour.
inline void check_or_abort(int status, const char* what) {
  if (status != MTRTQ_OK) {
    std::fprintf(stderr, "mtrtq error %d (%s) in %s: %s\n", status, mtrtq_status_string(status),
                 what, mtrtq_last_error());
    std::abort();
  }
}

inline void cuda_or_abort(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "CUDA error %s in %s\n", cudaGetErrorString(e), what);
    std::abort();
  }
}

// One int8 weight on the device in the library's packed layout, with its scales.
class PackedWeight {
 public:
  PackedWeight() = default;
  // q_host: int8 [K,N] row-major (the reference's MatMulQ W), scale_host: f32 [N].
  PackedWeight(const int8_t* q_host, const float* scale_host, int64_t K, int64_t N,
               cudaStream_t stream = nullptr)
      : K_(K), N_(N) {
    const int64_t nbytes = mtrtq_packed_bytes(K, N);
    if (nbytes < 0) check_or_abort(MTRTQ_ERR_INVALID_ARG, "mtrtq_packed_bytes");
    bytes_ = static_cast<size_t>(nbytes);
    std::vector<uint8_t> host(bytes_);
    check_or_abort(mtrtq_prepack_host(q_host, K, N, host.data(), bytes_), "mtrtq_prepack_host");
    cuda_or_abort(cudaMalloc(&packed_, bytes_), "cudaMalloc(packed)");
    cuda_or_abort(cudaMalloc(reinterpret_cast<void**>(&scale_), sizeof(float) * N), "cudaMalloc(scale)");
    cuda_or_abort(cudaMemcpyAsync(packed_, host.data(), bytes_, cudaMemcpyHostToDevice, stream),
                  "upload packed");
    cuda_or_abort(cudaMemcpyAsync(scale_, scale_host, sizeof(float) * N, cudaMemcpyHostToDevice, stream),
                  "upload scale");
    cuda_or_abort(cudaStreamSynchronize(stream), "upload sync");
  }
  ~PackedWeight() { release(); }
  PackedWeight(const PackedWeight&) = delete;
  PackedWeight& operator=(const PackedWeight&) = delete;
  PackedWeight(PackedWeight&& o) noexcept { *this = static_cast<PackedWeight&&>(o); }
  PackedWeight& operator=(PackedWeight&& o) noexcept {
    if (this != &o) {
      release();
      packed_ = o.packed_; scale_ = o.scale_; K_ = o.K_; N_ = o.N_; bytes_ = o.bytes_;
      o.packed_ = nullptr; o.scale_ = nullptr;
    }
    return *this;
  }

  const void* packed() const { return packed_; }
  const float* scale() const { return scale_; }
  int64_t K() const { return K_; }
  int64_t N() const { return N_; }

 private:
  void release() {
    if (packed_) cudaFree(packed_);
    if (scale_) cudaFree(scale_);
    packed_ = nullptr;
    scale_ = nullptr;
  }
  void* packed_ = nullptr;
  float* scale_ = nullptr;
  int64_t K_ = 0, N_ = 0;
  size_t bytes_ = 0;
};

// Zero-filled per-device scratch, grown only by reserve() (setup time).
class WorkspacePool {
 public:
  static WorkspacePool& instance() {
    static WorkspacePool pool;
    return pool;
  }
  // Make sure the current device's workspace holds `bytes`.
  void reserve(size_t bytes) {
    std::lock_guard<std::mutex> lk(mu_);
    int dev = 0;
    cuda_or_abort(cudaGetDevice(&dev), "cudaGetDevice");
    if (static_cast<size_t>(dev) >= slots_.size()) slots_.resize(dev + 1);
    Slot& s = slots_[dev];
    if (s.bytes >= bytes) return;
    if (s.ptr) cuda_or_abort(cudaFree(s.ptr), "cudaFree(workspace)");
    cuda_or_abort(cudaMalloc(&s.ptr, bytes), "cudaMalloc(workspace)");
    cuda_or_abort(cudaMemset(s.ptr, 0, bytes), "cudaMemset(workspace)");
    s.bytes = bytes;
  }
  void* get(size_t* bytes) {
    std::lock_guard<std::mutex> lk(mu_);
    int dev = 0;
    cuda_or_abort(cudaGetDevice(&dev), "cudaGetDevice");
    if (static_cast<size_t>(dev) >= slots_.size()) {
      *bytes = 0;
      return nullptr;
    }
    *bytes = slots_[dev].bytes;
    return slots_[dev].ptr;
  }

 private:
  struct Slot {
    void* ptr = nullptr;
    size_t bytes = 0;
  };
  std::mutex mu_;
  std::vector<Slot> slots_;
};

// Reserve the scratch one MatMulQ shape needs (call at setup, e.g. executor construction).
inline void reserve_matmul_q8(int M, int N, int K, int mode = MTRTQ_MODE_BF16) {
  const int64_t ws = mtrtq_workspace_bytes(M, K, N, MTRTQ_DTYPE_F32, mode);
  if (ws < 0) check_or_abort(MTRTQ_ERR_INVALID_ARG, "mtrtq_workspace_bytes");
  WorkspacePool::instance().reserve(static_cast<size_t>(ws));
}

}  // namespace mtrtq

namespace mtrt::cuda {

// C[M,N] = A[M,K] x dequant(W) (+ bias[N]); all DEVICE pointers, row-major, f32
// activations and output, default stream (the convention of backends/cuda/kernels.h).
// W is the pre-packed weight; mode MTRTQ_MODE_BF16 (default) or MTRTQ_MODE_FP32.
// The scratch must have been reserved (mtrtq::reserve_matmul_q8) at setup.
inline void matmul_q8(const float* A, const mtrtq::PackedWeight& W, const float* bias, float* C,
                      int M, int N, int K, int mode = MTRTQ_MODE_BF16,
                      cudaStream_t stream = nullptr) {
  size_t ws_bytes = 0;
  void* ws = mtrtq::WorkspacePool::instance().get(&ws_bytes);
  mtrtq::check_or_abort(mtrtq_matmul(A, MTRTQ_DTYPE_F32, K, W.packed(), W.scale(), bias, C, N, M,
                                     K, N, mode, ws, ws_bytes, stream),
                        "mtrt::cuda::matmul_q8");
}

}  // namespace mtrt::cuda
