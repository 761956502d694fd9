// Stream-K decode GEMV on CUDA cores for the INT8 weight-only MatMul, M <= 8.
//
// Replaces, for the decode sites, the reference's scalar MatMulQ loop
// (src/ops/kernels_matmul.cpp:66-73) and the KV-cache decoder's fp32 GEMV
// (tools/run_gpt2.cpp:125-132, :189).
//
// The work is a stream over the packed int8 weights. A "unit" is one 64-k block of
// one 128-channel tile: 8 KiB, contiguous in the packed layout ([tile][slab]).
// The grid is persistent -- four 128-thread CTAs per SM -- and CTA c takes the
// units [c*U/G, (c+1)*U/G): one contiguous byte range, the same length for every
// CTA, so there is no tail wave.
//
// Thread r of a CTA owns channel row r of the tile it is in. Per unit it issues
// four 16-byte loads (one per 16-k slab; a warp reads 512 contiguous bytes per
// load) and keeps the next unit's four in flight, converts the int8 weights to
// exact floats (exponent-bias trick) and accumulates with packed fp32x2 FMAs
// against activations staged in shared memory. Only the k-blocks the CTA's range
// visits are staged (a cyclic interval of k-blocks, at most all of them), rounded
// to bf16 in MTRTQ_MODE_BF16.
//
// A tile cut by CTA boundaries gets one fp32 partial per CTA that touches it; the
// last of them to finish (atomic ticket per cut tile) sums them in CTA order --
// deterministic -- and applies scale and bias. Tiles inside one CTA are written
// directly: y = sum * scale (+ bias), multiply then add, the reference's
// MatMulQ-then-Add order.
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

// Units (8 KiB each, 64 bytes per thread) in flight per thread.
constexpr int kGemvSkDepth = 2;

struct GemvSkParams {
  const void* X;
  int64_t ldx;
  const uint4* W;        // packed weights: unit u, slab j, row r at uint4 index u*512 + j*128 + r
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  int M, K, N;
  int KB;                // 64-k blocks per tile
  int n_tiles;
  long long units;       // n_tiles * KB
  int grid;              // CTAs
  float* partials;       // [grid][2][M][128]
  unsigned* counters;    // [grid]: a cut tile's ticket, indexed by the CTA owning its first unit
};

__device__ __forceinline__ int gsk_owner(long long u, long long U, int G) {
  return (int)(((u + 1) * (long long)G - 1) / U);
}

template <int MT>
__device__ __forceinline__ void gsk_dot_unit(const uint4 (&w)[4], const float* __restrict__ xs_blk,
                                             float2 (&acc)[MT]) {
  // xs_blk: [MT][64] fp32 for this unit's k-block.
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 wf[8];
    i8x4_to_f32x4(w[j].x, wf[0], wf[1]);
    i8x4_to_f32x4(w[j].y, wf[2], wf[3]);
    i8x4_to_f32x4(w[j].z, wf[4], wf[5]);
    i8x4_to_f32x4(w[j].w, wf[6], wf[7]);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4* xv = reinterpret_cast<const float4*>(xs_blk + m * 64 + j * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 x = xv[q];
        acc[m] = fma2(wf[2 * q], make_float2(x.x, x.y), acc[m]);
        acc[m] = fma2(wf[2 * q + 1], make_float2(x.z, x.w), acc[m]);
      }
    }
  }
}

// Four consecutive activations of row m from k (zeros past K), as fp32. Vector
// loads when the row stride allows them and all four lie inside the row.
template <bool X_BF16>
__device__ __forceinline__ float4 gsk_load_x4(const GemvSkParams& p, int m, int k, bool vec) {
  const int64_t off = (int64_t)m * p.ldx + k;
  if (X_BF16) {
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.X) + off;
    if (vec && k + 3 < p.K) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(x));
      return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                         __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    }
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = k + i < p.K ? __bfloat162float(x[i]) : 0.0f;
    return make_float4(v[0], v[1], v[2], v[3]);
  }
  const float* x = static_cast<const float*>(p.X) + off;
  if (vec && k + 3 < p.K) return __ldg(reinterpret_cast<const float4*>(x));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = k + i < p.K ? __ldg(x + i) : 0.0f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Stages the k-blocks a CTA visits: slot s holds k-block (kb0 + s) % KB as
// [MT][64] fp32 (rows >= M and k >= K are zero; fp32 input rounded to bf16 when
// ROUND). Each thread issues up to eight 4-element loads before it stores any, so
// the staging costs about one memory latency per eight groups, not one per element.
template <int MT, bool X_BF16, bool ROUND>
__device__ __forceinline__ void gsk_stage_x(const GemvSkParams& p, float* xs, int kb0, int nslots,
                                            int tid) {
  constexpr int kBatch = 8;
  const int groups = nslots * MT * 16;  // 4-element groups
  // X is 16-byte aligned (checked by the caller); rows keep 8- (bf16) or 16-byte
  // (fp32) alignment when the stride is a multiple of 4 elements.
  const bool vec = (p.ldx & 3) == 0;
  for (int g0 = tid; g0 < groups; g0 += 128 * kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int g = g0 + b * 128;
      v[b] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (g < groups) {
        const int s = g / (MT * 16), rem = g - s * (MT * 16), m = rem >> 4, k4 = (rem & 15) * 4;
        int kbs = kb0 + s;
        if (kbs >= p.KB) kbs -= p.KB;
        if (m < p.M) v[b] = gsk_load_x4<X_BF16>(p, m, kbs * 64 + k4, vec);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int g = g0 + b * 128;
      if (g < groups) {
        float4 w = v[b];
        if (ROUND) {
          w.x = round_bf16(w.x);
          w.y = round_bf16(w.y);
          w.z = round_bf16(w.z);
          w.w = round_bf16(w.w);
        }
        reinterpret_cast<float4*>(xs)[g] = w;
      }
    }
  }
}

// End of a segment (the CTA's units of tile t from seg_start to u_end): write the
// tile, or leave a partial and let the tile's last CTA sum them. Clears acc.
template <int MT>
__device__ __forceinline__ void gsk_segment_end(const GemvSkParams& p, float2 (&acc)[MT], int c, int t,
                                                int t_first, long long seg_start, long long u_end,
                                                int tid, unsigned* s_ticket) {
  const long long U = p.units;
  const int G = p.grid;
  const bool full_tile = seg_start == (long long)t * p.KB && u_end == (long long)(t + 1) * p.KB;
  const int n = t * kTileN + tid;
  const bool n_ok = n < p.N;
  float r[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    r[m] = acc[m].x + acc[m].y;
    acc[m] = make_float2(0.0f, 0.0f);
  }
  if (full_tile) {
    if (n_ok) {
      const float sc = p.scale[n];
      const float bi = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < p.M) {
          float y = __fmul_rn(r[m], sc);
          if (p.bias) y = __fadd_rn(y, bi);
          p.Y[(int64_t)m * p.ldy + n] = y;
        }
      }
    }
    return;
  }
  // Slot 0 holds the partial of the tile the CTA starts in, slot 1 that of the
  // tile it ends in (when they differ).
  const int slot = (t == t_first) ? 0 : 1;
  float* part = p.partials + ((int64_t)(c * 2 + slot) * p.M) * kTileN + tid;
#pragma unroll
  for (int m = 0; m < MT; ++m)
    if (m < p.M) part[(int64_t)m * kTileN] = r[m];
  __threadfence();
  __syncthreads();
  const int c_first = gsk_owner((long long)t * p.KB, U, G);
  const int c_last = gsk_owner((long long)(t + 1) * p.KB - 1, U, G);
  // Only the last tile that starts inside a CTA's range can leave it, so c_first
  // identifies the cut tile.
  unsigned* counter = p.counters + c_first;
  if (tid == 0) *s_ticket = atomicAdd(counter, 1u);
  __syncthreads();
  if (*s_ticket != (unsigned)(c_last - c_first)) return;
  __threadfence();
  if (n_ok) {
    float sum[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sum[m] = 0.0f;
    for (int cc = c_first; cc <= c_last; ++cc) {
      const int sl = ((int)((long long)cc * U / G / p.KB) == t) ? 0 : 1;
      const float* src = p.partials + ((int64_t)(cc * 2 + sl) * p.M) * kTileN + tid;
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < p.M) sum[m] += __ldcg(src + (int64_t)m * kTileN);
    }
    const float sc = p.scale[n];
    const float bi = p.bias ? p.bias[n] : 0.0f;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < p.M) {
        float y = __fmul_rn(sum[m], sc);
        if (p.bias) y = __fadd_rn(y, bi);
        p.Y[(int64_t)m * p.ldy + n] = y;
      }
    }
  }
  if (tid == 0) *counter = 0u;
}

// D: units whose weights each thread keeps in flight (16 * 4 * D bytes).
template <int MT, bool X_BF16, bool ROUND, int D>
__global__ void __launch_bounds__(128, 4) gemv_sk_kernel(const GemvSkParams p) {
  extern __shared__ __align__(16) float xs[];  // [nslots][MT][64]
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x;
  const int c = blockIdx.x;
  const long long U = p.units;
  const int G = p.grid;
  const long long u0 = (long long)c * U / G;
  const long long u1 = (long long)(c + 1) * U / G;
  const int n_units = (int)(u1 - u0);
  const int kb0 = (int)(u0 % p.KB);
  const int nslots = min(p.KB, n_units);

  // The first D units' weights go in flight before the activations are staged.
  // Buffer d serves units d, d + D, ...; the unit loop is unrolled by D so that
  // every buffer index is static and the buffers stay in registers.
  const uint4* wp = p.W + u0 * 512 + tid;
  uint4 buf[D][4];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    if (d < n_units) {
#pragma unroll
      for (int j = 0; j < 4; ++j) buf[d][j] = ldg_stream_v4(wp + d * 512 + j * 128);
    }
  }

  gsk_stage_x<MT, X_BF16, ROUND>(p, xs, kb0, nslots, tid);
  __syncthreads();

  float2 acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.0f, 0.0f);
  int kb = kb0;       // k-block of unit i
  int slot = 0;       // its activation slot: i mod KB
  int t = (int)(u0 / p.KB);
  const int t_first = t;
  long long seg_start = u0;

  auto step = [&](uint4 (&cur)[4], int i) {
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = cur[j];
    if (i + D < n_units) {
#pragma unroll
      for (int j = 0; j < 4; ++j) cur[j] = ldg_stream_v4(wp + (int64_t)(i + D) * 512 + j * 128);
    }
    gsk_dot_unit<MT>(w, xs + slot * (MT * 64), acc);

    if (i == n_units - 1 || kb == p.KB - 1) gsk_segment_end<MT>(p, acc, c, t, t_first, seg_start,
                                                               u0 + i + 1, tid, &s_ticket);
    if (kb == p.KB - 1) {
      seg_start = u0 + i + 1;
      ++t;
      kb = 0;
    } else {
      ++kb;
    }
    if (++slot == p.KB) slot = 0;
  };

  for (int i = 0; i < n_units; i += D) {
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (i + d < n_units) step(buf[d], i + d);
  }
}

// Dynamic shared memory the kernel needs for these sizes (activation slots).
size_t gemv_sk_smem_bytes(int mt, int KB, long long units, int grid) {
  const long long max_units = (units + grid - 1) / grid;
  const long long slots = max_units < KB ? max_units : KB;
  return (size_t)slots * mt * 64 * sizeof(float);
}

template <int MT, bool X_BF16, bool ROUND>
static cudaError_t gsk_launch(const GemvSkParams& gp, size_t smem, cudaStream_t st) {
  // smem <= kGemvSkSmemCap (48 KiB, the default limit), checked by the planner.
  constexpr int D = kGemvSkDepth;
  gemv_sk_kernel<MT, X_BF16, ROUND, D><<<gp.grid, 128, smem, st>>>(gp);
  return cudaGetLastError();
}

template <bool X_BF16, bool ROUND>
static cudaError_t gsk_by_mt(int mt, const GemvSkParams& gp, size_t smem, cudaStream_t st) {
  switch (mt) {
    case 1: return gsk_launch<1, X_BF16, ROUND>(gp, smem, st);
    case 2: return gsk_launch<2, X_BF16, ROUND>(gp, smem, st);
    case 3: return gsk_launch<3, X_BF16, ROUND>(gp, smem, st);
    case 4: return gsk_launch<4, X_BF16, ROUND>(gp, smem, st);
    case 5: return gsk_launch<5, X_BF16, ROUND>(gp, smem, st);
    case 6: return gsk_launch<6, X_BF16, ROUND>(gp, smem, st);
    case 7: return gsk_launch<7, X_BF16, ROUND>(gp, smem, st);
    case 8: return gsk_launch<8, X_BF16, ROUND>(gp, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_sk(const Plan& p, const void* X, int x_dtype, int64_t ldx, const void* packed,
                           const float* scale, const float* bias, float* Y, int64_t ldy,
                           void* workspace, cudaStream_t st) {
  GemvSkParams gp;
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
  gp.KB = p.kunits;
  gp.n_tiles = p.n_tiles;
  gp.units = (long long)p.n_tiles * p.kunits;
  gp.grid = p.grid;
  char* ws = static_cast<char*>(workspace);
  gp.counters = reinterpret_cast<unsigned*>(ws + p.off_counters);
  gp.partials = reinterpret_cast<float*>(ws + p.off_partials);
  const size_t smem = gemv_sk_smem_bytes((int)p.M, p.kunits, gp.units, p.grid);
  if (x_dtype == 1) return gsk_by_mt<true, false>((int)p.M, gp, smem, st);
  if (p.round_x) return gsk_by_mt<false, true>((int)p.M, gp, smem, st);
  return gsk_by_mt<false, false>((int)p.M, gp, smem, st);
}

}  // namespace mtrtq
