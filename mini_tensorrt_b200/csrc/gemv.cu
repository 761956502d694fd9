// Decode GEMV for the INT8 weight-only MatMul: M <= 8 token rows per launch chunk.
//
// Replaces, for the decode sites, the reference's scalar MatMulQ triple loop
// (src/ops/kernels_matmul.cpp:66-73) and the fp32 gemm_auto GEMV of the KV-cache
// decoder (tools/run_gpt2.cpp:125-132, :189).
//
// Work decomposition: one CTA = 128 threads = one channel tile (128 output
// channels) x one k-split. Thread r owns channel 128t + r; each 16-k slab of the
// packed weights is one 16-byte streaming load per thread (a warp reads 512
// contiguous bytes), converted to exact floats with the exponent-bias trick and
// multiplied with the CTA's staged activations using packed fp32x2 FMAs.
// No cross-lane reduction is needed: a thread accumulates its own channel.
//
// Split-K: when the channel tiles alone cannot fill the GPU, the k range is cut
// into `splits` pieces; each CTA writes an fp32 partial to the workspace and the
// last CTA of a tile to arrive (atomic ticket) sums the partials in split order,
// so results are deterministic run to run. The ticket counter is reset to zero
// by that CTA, leaving the workspace ready for the next call.
//
// Epilogue: y = sum * scale[n] (+ bias[n]) with separate multiply and add, the
// reference's MatMulQ-then-Add order.
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

struct GemvParams {
  const void* X;
  int64_t ldx;
  const uint4* W;
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  Epilogue epi;
  int M, K, N;
  int n_pad;
  int KS;               // slabs of 16 in K_pad
  int slabs_per_split;
  int chunk_slabs;      // slabs of activations staged in shared memory at a time (% 8 == 0)
  int splits;
  int n_tiles;
  float* partials;      // [splits][M][n_pad]
  unsigned* counters;   // [m_chunks][n_tiles]
};

template <int MT>
__device__ __forceinline__ void dot_slab(const uint4& w, const float* __restrict__ xs_slab,
                                         int klen, float2 (&acc)[MT]) {
  float2 wf[8];
  i8x4_to_f32x4(w.x, wf[0], wf[1]);
  i8x4_to_f32x4(w.y, wf[2], wf[3]);
  i8x4_to_f32x4(w.z, wf[4], wf[5]);
  i8x4_to_f32x4(w.w, wf[6], wf[7]);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float4* xv = reinterpret_cast<const float4*>(xs_slab + m * klen);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 x = xv[j];
      acc[m] = fma2(wf[2 * j], make_float2(x.x, x.y), acc[m]);
      acc[m] = fma2(wf[2 * j + 1], make_float2(x.z, x.w), acc[m]);
    }
  }
}

template <int MT, bool X_BF16, bool ROUND, int U>
__global__ void __launch_bounds__(128) gemv_q8_kernel(const GemvParams p) {
  extern __shared__ __align__(16) float xs[];  // [MT][klen]
  __shared__ unsigned s_ticket;
  const int nt = blockIdx.x;
  const int split = blockIdx.y;
  const int mc = blockIdx.z;
  const int tid = threadIdx.x;

  const int s0 = split * p.slabs_per_split;
  const int s1 = min(s0 + p.slabs_per_split, p.KS);
  const int nsl = s1 - s0;
  const int CH = p.chunk_slabs;   // multiple of U
  const int klen = CH * kSlabK;   // staged activations per row
  const int m0 = mc * 8;
  const int mrem = min(MT, p.M - m0);

  // Issue the first weight loads before staging activations so they overlap.
  const uint4* wp = p.W + ((int64_t)nt * p.KS + s0) * kTileN + tid;
  uint4 buf[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (u < nsl) buf[u] = ldg_stream_v4(wp + (int64_t)u * kTileN);

  float2 acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.0f, 0.0f);

  int in_chunk = CH;  // slabs consumed from the staged chunk
  for (int s = 0; s < nsl; s += U) {
    if (in_chunk == CH) {
      // Stage activations for slabs [s0+s, s0+s+CH) as fp32 [MT][klen] (zero
      // beyond K and M); the weight loads already in flight keep streaming.
      if (s > 0) __syncthreads();
      const int64_t k0 = (int64_t)(s0 + s) * kSlabK;
      const int kn = min(CH, nsl - s) * kSlabK;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        for (int kk = tid; kk < kn; kk += 128) {
          const int64_t k = k0 + kk;
          float v = 0.0f;
          if (m < mrem && k < p.K) {
            if (X_BF16) {
              v = __bfloat162float(
                  static_cast<const __nv_bfloat16*>(p.X)[(int64_t)(m0 + m) * p.ldx + k]);
            } else {
              v = static_cast<const float*>(p.X)[(int64_t)(m0 + m) * p.ldx + k];
              if (ROUND) v = round_bf16(v);
            }
          }
          xs[m * klen + kk] = v;
        }
      }
      __syncthreads();
      in_chunk = 0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (s + u < nsl) {
        const uint4 w = buf[u];
        if (s + u + U < nsl) buf[u] = ldg_stream_v4(wp + (int64_t)(s + u + U) * kTileN);
        dot_slab<MT>(w, xs + (in_chunk + u) * kSlabK, klen, acc);
      }
    }
    in_chunk += U;
  }

  const int n = nt * kTileN + tid;
  float r[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) r[m] = acc[m].x + acc[m].y;

  if (p.splits == 1) {
    if (n < p.N) {
      const float sc = p.scale[n];
      const float b = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < mrem) {
          float y = __fmul_rn(r[m], sc);
          if (p.bias) y = __fadd_rn(y, b);
          p.Y[(int64_t)(m0 + m) * p.ldy + n] = epi_apply(p.epi, y, m0 + m, n);
        }
      }
    }
    return;
  }

  // Split-K: publish this split's partial, then the last CTA of the tile reduces.
  float* part = p.partials + ((int64_t)split * p.M + m0) * p.n_pad + n;
#pragma unroll
  for (int m = 0; m < MT; ++m)
    if (m < mrem) __stcg(part + (int64_t)m * p.n_pad, r[m]);
  __syncthreads();
  unsigned* counter = p.counters + (int64_t)mc * p.n_tiles + nt;
  if (tid == 0) s_ticket = ticket_acq_rel(counter);
  __syncthreads();
  if (s_ticket != (unsigned)(p.splits - 1)) return;
  if (n < p.N) {
    const float sc = p.scale[n];
    const float b = p.bias ? p.bias[n] : 0.0f;
    // All rows' loads of one split are independent and issued together; the
    // sum still runs split 0, 1, 2, ... for every output.
    const float* src = p.partials + (int64_t)m0 * p.n_pad + n;
    const int64_t split_stride = (int64_t)p.M * p.n_pad;
    float sum[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sum[m] = 0.0f;
#pragma unroll 4
    for (int sp = 0; sp < p.splits; ++sp) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < mrem) sum[m] += __ldcg(src + sp * split_stride + (int64_t)m * p.n_pad);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < mrem) {
        float y = __fmul_rn(sum[m], sc);
        if (p.bias) y = __fadd_rn(y, b);
        p.Y[(int64_t)(m0 + m) * p.ldy + n] = epi_apply(p.epi, y, m0 + m, n);
      }
    }
  }
  if (tid == 0) *counter = 0u;
}

template <int MT, bool X_BF16, bool ROUND>
static cudaError_t launch_mt(const GemvParams& gp, dim3 grid, size_t smem, cudaStream_t st) {
  constexpr int U = kGemvUnroll;
  gemv_q8_kernel<MT, X_BF16, ROUND, U><<<grid, 128, smem, st>>>(gp);
  return cudaGetLastError();
}

template <bool X_BF16, bool ROUND>
static cudaError_t launch_by_mt(int mt, const GemvParams& gp, dim3 grid, cudaStream_t st) {
  const size_t smem = (size_t)mt * gp.chunk_slabs * kSlabK * sizeof(float);
  switch (mt) {
    case 1: return launch_mt<1, X_BF16, ROUND>(gp, grid, smem, st);
    case 2: return launch_mt<2, X_BF16, ROUND>(gp, grid, smem, st);
    case 3: return launch_mt<3, X_BF16, ROUND>(gp, grid, smem, st);
    case 4: return launch_mt<4, X_BF16, ROUND>(gp, grid, smem, st);
    case 5: return launch_mt<5, X_BF16, ROUND>(gp, grid, smem, st);
    case 6: return launch_mt<6, X_BF16, ROUND>(gp, grid, smem, st);
    case 7: return launch_mt<7, X_BF16, ROUND>(gp, grid, smem, st);
    default: return launch_mt<8, X_BF16, ROUND>(gp, grid, smem, st);
  }
}

cudaError_t launch_gemv(const Plan& p, const void* X, int x_dtype, int64_t ldx, const void* packed,
                        const float* scale, const float* bias, float* Y, int64_t ldy,
                        void* workspace, const Epilogue& epi, cudaStream_t st) {
  GemvParams gp;
  gp.epi = epi;
  gp.X = X;
  gp.ldx = ldx;
  gp.W = static_cast<const uint4*>(packed);
  gp.scale = scale;
  gp.bias = bias;
  gp.Y = Y;
  gp.ldy = ldy;
  gp.M = (int)p.M;
  gp.K = (int)p.K;
  gp.N = (int)p.N;
  gp.n_pad = (int)p.n_pad;
  gp.KS = p.kunits;
  gp.slabs_per_split = p.kunits_per_split;
  gp.chunk_slabs = p.chunk_units;
  gp.splits = p.splits;
  gp.n_tiles = p.n_tiles;
  char* ws = static_cast<char*>(workspace);
  gp.counters = ws ? reinterpret_cast<unsigned*>(ws + p.off_counters) : nullptr;
  gp.partials = ws ? reinterpret_cast<float*>(ws + p.off_partials) : nullptr;
  const dim3 grid((unsigned)p.n_tiles, (unsigned)p.splits, (unsigned)p.m_tiles);
  // Rows per launch chunk: all chunks but the last hold 8 rows; a single chunk
  // holds M rows, so small M compiles to exactly M accumulators.
  const int mt = p.m_tiles == 1 ? (int)p.M : 8;
  if (x_dtype == 1) return launch_by_mt<true, false>(mt, gp, grid, st);
  if (p.round_x) return launch_by_mt<false, true>(mt, gp, grid, st);
  return launch_by_mt<false, false>(mt, gp, grid, st);
}

}  // namespace mtrtq
