// Weight pre-pack and activation staging kernels.
//
// Packed weight layout ("channel tiles of 16-k slabs"): for channel tile t
// (channels 128t..128t+127) and slab s (k = 16s..16s+15) the 2048 bytes at
// ((t * KS + s) * 128 + r) * 16 hold channel 128t + r's 16 weights in k order,
// KS = K_pad / 16. Padding (n >= N or k >= K) is zero. One warp reading one slab
// of 32 channels touches 512 contiguous bytes, and one 64-k pipeline stage of a
// tile is 8 KiB contiguous, so both the GEMV (plain 16-byte loads) and the GEMM
// (one bulk TMA copy per stage) stream the weights with full coalescing.
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

__global__ void prepack_kernel(const int8_t* __restrict__ q, int64_t K, int64_t N, int64_t KS,
                               int64_t total_chunks, uint4* __restrict__ out) {
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total_chunks;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx % kTileN;
    const int64_t s = (idx / kTileN) % KS;
    const int64_t t = idx / (kTileN * KS);
    const int64_t n = t * kTileN + r;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (n < N) {
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        const int64_t k = s * kSlabK + b;
        const uint32_t v = (k < K) ? (uint32_t)(uint8_t)q[k * N + n] : 0u;
        w[b >> 2] |= v << (8 * (b & 3));
      }
    }
    out[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

cudaError_t launch_prepack(const int8_t* q, int64_t K, int64_t N, void* packed, cudaStream_t st) {
  const int64_t n_pad = round_up64(N, kTileN);
  const int64_t k_pad = round_up64(K, kBlockK);
  const int64_t KS = k_pad / kSlabK;
  const int64_t total = (n_pad / kTileN) * KS * kTileN;
  const int threads = 256;
  int64_t blocks = ceil_div64(total, threads);
  if (blocks > 148 * 64) blocks = 148 * 64;
  prepack_kernel<<<(unsigned)blocks, threads, 0, st>>>(q, K, N, KS, total,
                                                       static_cast<uint4*>(packed));
  return cudaGetLastError();
}

// Xb[m, k] = bf16_rn(X[m, k]) for k < K, 0 for K <= k < ldxb.
template <bool IN_BF16>
__global__ void x_to_bf16_kernel(const void* __restrict__ X, int64_t ldx, int64_t M, int64_t K,
                                 __nv_bfloat16* __restrict__ Xb, int64_t ldxb) {
  const int64_t total = M * ldxb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / ldxb, k = i - m * ldxb;
    __nv_bfloat16 v = __float2bfloat16_rn(0.0f);
    if (k < K) {
      if (IN_BF16)
        v = static_cast<const __nv_bfloat16*>(X)[m * ldx + k];
      else
        v = __float2bfloat16_rn(static_cast<const float*>(X)[m * ldx + k]);
    }
    Xb[i] = v;
  }
}

cudaError_t launch_x_to_bf16(const void* X, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                             void* Xb, int64_t ldxb, cudaStream_t st) {
  const int64_t total = M * ldxb;
  const int threads = 256;
  int64_t blocks = ceil_div64(total, threads);
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  if (x_dtype == 1)
    x_to_bf16_kernel<true><<<(unsigned)blocks, threads, 0, st>>>(
        X, ldx, M, K, static_cast<__nv_bfloat16*>(Xb), ldxb);
  else
    x_to_bf16_kernel<false><<<(unsigned)blocks, threads, 0, st>>>(
        X, ldx, M, K, static_cast<__nv_bfloat16*>(Xb), ldxb);
  return cudaGetLastError();
}

}  // namespace mtrtq
