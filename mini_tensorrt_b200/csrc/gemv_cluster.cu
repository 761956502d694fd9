// Decode GEMV for the INT8 weight-only MatMul, M <= 64 (blocks of 8 tokens):
// split-K inside a thread-block cluster, reduced through distributed shared
// memory; optionally with each activation row layer-normalized first.
//
// Replaces, for the decode sites, the reference's scalar MatMulQ loop
// (src/ops/kernels_matmul.cpp:66-73) and the KV-cache decoder's fp32 GEMV
// (tools/run_gpt2.cpp:125-132, :189).
//
// Work: one cluster of CS CTAs per 128-channel tile; CTA rank s takes the s-th of
// CS equal ranges of the tile's 64-k units (8 KiB each, contiguous in the packed
// layout). A producer warp streams the CTA's units into a ring of shared memory
// stages with 1-D bulk async copies (TMA), so the bytes in flight are bounded by
// shared memory, not registers.
//
// Arithmetic: the int8 weights are used as they are, as the A operand of integer
// warp MMAs (m16n8k32, s8 x s8 -> s32, exact). Activations are re-expressed, per
// CTA and token m, as three int8 digits over the CTA's k range:
//     x = (s_m / 127) * (d0 + d1 / 2^7 + d2 / 2^14),   s_m = max |x[m, k range]|,
// d0 in [-127, 127], d1, d2 in [-64, 64], so each x is represented to within
// 2^-15 * s_m / 127 (about 2^-22 of the largest activation of the range; fp32
// itself carries 24 bits). Each digit plane is one MMA B operand (8 columns =
// the tokens); the three int32 accumulators are combined in fp32 at the end:
//     partial = (s_m / 127) * (acc0 + acc1 / 2^7 + acc2 / 2^14).
// In MTRTQ_MODE_BF16, fp32 activations are first rounded to bf16. Non-finite
// activations make the token's outputs NaN.
//
// Operand loads: the weight fragments of a unit's two k32 steps come from two
// ldmatrix.x4 (each 8 x 16 B matrix is eight consecutive rows of one 16-k slab,
// 128 contiguous bytes: no bank conflict), and the activation digits are stored
// in fragment order, so a lane's four B-fragment words are one 16-byte load.
//
// Partial sums never leave the SM cluster: each warp owns 16 channel rows, the CS
// ranks' partials are exchanged through distributed shared memory after a cluster
// barrier, and rank s sums rows [s*128/CS, (s+1)*128/CS) over the ranks in rank
// order -- a fixed order, so results do not depend on timing -- then applies
// y = sum * scale (+ bias), multiply then add, the reference's MatMulQ-then-Add
// order. No workspace, no atomics, no device-wide fences.
//
// Every mbarrier wait is bounded: a wait that gives up records MTRTQ_ERR_TIMEOUT
// in the device status word and stops the CTA's loops; the producer still waits
// (bounded) for the copies it issued before the CTA leaves.
#include "q8_common.cuh"
#include "q8_digits.cuh"
#include "q8_internal.h"

namespace mtrtq {

namespace {

constexpr int kClWarps = 8;                // consumers: one 16-row group each
constexpr int kClThreads = kClWarps * 32;  // consumer threads
constexpr int kClBlock = kClThreads + 32;  // + the producer warp
constexpr uint32_t kUnitBytes = 8192;      // 64 k x 128 channels of int8
constexpr int kDigits = 3;
constexpr int kClMaxTokens = kGemvClMaxM;  // 8 blocks of 8 tokens
// Weight units issued before the activations land (at most the ring's stages).
// After them the weight stream waits until every consumer warp has read its
// activations, so that those loads do not queue behind weight traffic; under
// programmatic dependent launch the early units are fetched while the grid
// ahead finishes. Measured on B200 with overlapped launches (conflict-free
// operand loads): 6 units against 4 gives 768 x 50257 M = 1 9.41 / 9.83 us,
// 3072 x 768 M = 8 5.05 / 5.48 us, 4096 x 14336 M = 1 14.18 / 14.5 us, and the
// same at M = 8 on the large shapes; 8 units is no better than 6.
constexpr int kClEarlyUnits = 6;
constexpr int kClEarlyUnitsPdl = 6;

struct GemvClParams {
  const void* X;
  int64_t ldx;
  const char* W;   // packed: tile t, unit u (64 k) at byte (t * KB + u) * 8192
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  Epilogue epi;
  int M, K, N;
  int KB;          // 64-k units per tile
  int stages;      // shared memory ring stages (2..kGemvClMaxStages)
  int early_units; // weight units issued before the activations have arrived
  unsigned* status;
  // LayerNorm of each activation row before the product (null: none); fp32 X only.
  const float* ln_gamma;
  const float* ln_beta;
  float ln_eps;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n"
               "barrier.cluster.wait.aligned;" ::: "memory");
}

// Address of `p` (this CTA's shared memory) in the shared memory of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Four consecutive activations of row m from k (zeros past K) as fp32.
template <bool X_BF16>
__device__ __forceinline__ float4 cl_load_x4(const GemvClParams& p, int m, int k, bool vec) {
  return load_x4<X_BF16>(p.X, p.ldx, p.K, m, k, vec);
}

// LayerNorm of four consecutive activations of token m at k, with the token's
// mean and 1 / sqrt(var + eps) in ln[m] and ln[kClMaxTokens + m] (the reference's
// (x - mean) * inv * gamma + beta, src/ops/kernels_transformer.cpp:50-51); those
// past K stay zero. No-op when ln is null.
__device__ __forceinline__ float4 cl_ln4(const GemvClParams& p, float4 v, int m, int k, const float* ln) {
  if (!ln) return v;
  const float mean = ln[m], inv = ln[kClMaxTokens + m];
  float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
    a[i] = k + i < p.K ? (a[i] - mean) * inv * __ldg(p.ln_gamma + k + i) + __ldg(p.ln_beta + k + i) : 0.0f;
  return make_float4(a[0], a[1], a[2], a[3]);
}

// Loads groups g0, g0 + 32, ... (kB of them, those below gend) of token m's range
// as fp32 (layer-normalized when ln is set, then rounded to bf16 when ROUND);
// zeros elsewhere.
template <int kB, bool X_BF16, bool ROUND>
__device__ __forceinline__ void cl_load_groups(const GemvClParams& p, float4 (&v)[kB], int m, int kbase,
                                               int g0, int gend, bool vec, const float* ln) {
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const int g = g0 + b * 32, k = kbase + g * 4;
    v[b] = g < gend ? cl_round<ROUND>(cl_ln4(p, cl_load_x4<X_BF16>(p, m, k, vec), m, k, ln))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Issues the loads of groups g0, g0 + 32, ... (kB of them, those below gend) that
// a single vector load can fetch, keeping the raw bits; nothing else waits on them.
template <int kB, bool X_BF16>
__device__ __forceinline__ void cl_issue_groups(const GemvClParams& p, uint4 (&raw)[kB], int m, int kbase,
                                                int g0, int gend, bool vec) {
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const int g = g0 + b * 32, k = kbase + g * 4;
    if (g < gend && vec && k + 3 < p.K) {
      const int64_t off = (int64_t)m * p.ldx + k;
      if (X_BF16) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p.X) + off));
        raw[b] = make_uint4(u.x, u.y, 0u, 0u);
      } else {
        raw[b] = __ldg(reinterpret_cast<const uint4*>(static_cast<const float*>(p.X) + off));
      }
    }
  }
}

// The values of the groups cl_issue_groups covered, from their raw bits; the
// others (past the row's end or at a stride that rules out vector loads) are
// read here element by element. Layer-normalized when ln is set, then rounded to
// bf16 when ROUND.
template <int kB, bool X_BF16, bool ROUND>
__device__ __forceinline__ void cl_decode_groups(const GemvClParams& p, const uint4 (&raw)[kB], float4 (&v)[kB],
                                                 int m, int kbase, int g0, int gend, bool vec,
                                                 const float* ln) {
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const int g = g0 + b * 32, k = kbase + g * 4;
    if (g >= gend) {
      v[b] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (vec && k + 3 < p.K) {
      const uint4 r = raw[b];
      v[b] = X_BF16 ? make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u),
                                  __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u))
                    : make_float4(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z),
                                  __uint_as_float(r.w));
    } else {
      v[b] = cl_load_x4<X_BF16>(p, m, k, vec);
    }
    if (g < gend) v[b] = cl_ln4(p, v[b], m, k, ln);
    v[b] = cl_round<ROUND>(v[b]);
  }
}

template <int kB>
__device__ __forceinline__ void cl_max_groups(const float4 (&v)[kB], float& mx, bool& bad) {
#pragma unroll
  for (int b = 0; b < kB; ++b) mx = fmaxf(mx, cl_group_max(v[b], bad));
}

// Writes the three digit planes of groups g0, g0 + 32, ... (those below gend).
template <int kB>
__device__ __forceinline__ void cl_store_digits(const float4 (&v)[kB], float inv, int8_t* xd, int plane,
                                                int mt, int m, int g0, int gend) {
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const int g = g0 + b * 32;
    if (g < gend) cl_store_digit_group(v[b], inv, xd, plane, mt, m, g);
  }
}

// Activation digits over the CTA's units [u0, u0 + nu): plane d at xd + d * plane,
// unit u, token m, k at ((u * mt + m) * 64 + k). Token m is staged by the consumer
// warps w with w % mt == m, each taking an equal share of the range's 4-element
// groups. s_max[m] gets max |x| over the range (atomically, as ordered bits) and
// s_bad[m] flags a non-finite value.
//
// begin() issues the loads of a share of up to 32 * RES groups, whose raw bits
// then stay in registers (the kernel calls it before its barrier setup, and
// nothing waits on the loads until finish(), so their latency overlaps the
// setup); finish() decodes them, completes the maxima across warps (one named
// barrier) and writes the digits. A longer share is read twice, in batches, in finish():
// the second time from the caches the first pass filled.
// MANY: the kernel instance takes more tokens than it has consumer warps (NB > 1);
// without it the many-token staging is not compiled in.
template <bool X_BF16, bool ROUND, int RES, bool MANY>
struct ClStager {
  static constexpr int kRes = RES;  // groups per lane held in registers
  static constexpr int kBatch = 6;  // groups per lane per batch otherwise
  int m, gbeg, gend, kbase, warp_, nu_;
  bool vec, resident;
  const float* ln = nullptr;  // per-token LayerNorm statistics in shared memory, if any
  uint4 raw[kRes];

  __device__ __forceinline__ void begin(const GemvClParams& p, int u0, int nu, int warp, int lane) {
    const int mt = p.M;
    warp_ = warp;
    nu_ = nu;
    kbase = u0 * 64;
    vec = (p.ldx & 3) == 0;
    if (mt > kClWarps) {  // more tokens than warps: finish() stages them whole
      resident = false;
      return;
    }
    m = warp % mt;
    const int share_warps = (kClWarps - 1 - m) / mt + 1;  // warps staging token m
    const int j = warp / mt;
    const int n4 = nu * 16;  // 4-element groups of the range
    gbeg = (int)((int64_t)j * n4 / share_warps);
    gend = (int)((int64_t)(j + 1) * n4 / share_warps);
    resident = gend - gbeg <= 32 * kRes;
    if (resident) cl_issue_groups<kRes, X_BF16>(p, raw, m, kbase, gbeg + lane, gend, vec);
  }

  // More tokens than warps: the consumer threads take the 4-element groups of all
  // tokens together (group e of the M x n4: token e / n4, group e % n4), kMany per
  // thread per pass with all of a pass's loads in flight at once (one warp per token
  // in turn would wait for one round trip per token). The maxima go to shared
  // memory atomically. A range that fits one pass keeps its values in registers
  // for the digits; a longer one is read again, from the caches the first read
  // filled.
  static constexpr int kMany = 8;
  __device__ __forceinline__ void many_load(const GemvClParams& p, float4 (&v)[kMany], int base, int ct, int n4,
                                            int total) {
#pragma unroll
    for (int i = 0; i < kMany; ++i) {
      const int e = base + i * kClThreads + ct;
      if (e < total) {
        const int t = e / n4, g = e - t * n4, k = kbase + g * 4;
        v[i] = cl_round<ROUND>(cl_ln4(p, cl_load_x4<X_BF16>(p, t, k, vec), t, k, ln));
      } else {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }

  __device__ __forceinline__ void finish_many(const GemvClParams& p, int8_t* xd, int plane, int* s_max,
                                              int* s_bad, uint64_t* xready, int lane) {
    const int mt = p.M, n4 = nu_ * 16, total = mt * n4;
    const int ct = warp_ * 32 + lane;
    constexpr int kPass = kClThreads * kMany;
    const bool one_pass = total <= kPass;
    float4 v[kMany];
    for (int base = 0; base < total; base += kPass) {
      many_load(p, v, base, ct, n4, total);
#pragma unroll
      for (int i = 0; i < kMany; ++i) {
        const int e = base + i * kClThreads + ct;
        if (e < total) {
          bool bad = false;
          const float a = cl_group_max(v[i], bad);
          const int t = e / n4;
          atomicMax(&s_max[t], __float_as_int(a));  // a >= 0: bit order is value order
          if (bad) atomicOr(&s_bad[t], 1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(xready);  // this warp's activations have been read
    named_bar_sync(1, kClThreads);
    for (int base = 0; base < total; base += kPass) {
      if (!one_pass) many_load(p, v, base, ct, n4, total);
#pragma unroll
      for (int i = 0; i < kMany; ++i) {
        const int e = base + i * kClThreads + ct;
        if (e < total) {
          const int t = e / n4, g = e - t * n4;
          const float smax = __int_as_float(s_max[t]);
          const float inv = (smax > 0.0f && !s_bad[t]) ? 127.0f / smax : 0.0f;
          cl_store_digit_group(v[i], inv, xd, plane, mt, t, g);
        }
      }
    }
  }

  __device__ __forceinline__ void finish(const GemvClParams& p, int8_t* xd, int plane, int* s_max,
                                         int* s_bad, uint64_t* xready, int lane) {
    const int mt = p.M;
    if (MANY && mt > kClWarps) {
      finish_many(p, xd, plane, s_max, s_bad, xready, lane);
      return;
    }
    float mx = 0.0f;
    bool bad = false;
    float4 v[kRes];
    if (resident) {
      cl_decode_groups<kRes, X_BF16, ROUND>(p, raw, v, m, kbase, gbeg + lane, gend, vec, ln);
      cl_max_groups<kRes>(v, mx, bad);
    } else {
      for (int g0 = gbeg + lane; g0 < gend; g0 += 32 * kBatch) {
        float4 w[kBatch];
        cl_load_groups<kBatch, X_BF16, ROUND>(p, w, m, kbase, g0, gend, vec, ln);
        cl_max_groups<kBatch>(w, mx, bad);
      }
    }
    // This warp's activations have been read: the weight stream may resume while
    // the maxima and digits are computed.
    __syncwarp();
    if (lane == 0) mbar_arrive(xready);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      bad |= __shfl_xor_sync(0xffffffffu, (int)bad, o) != 0;
    }
    if (lane == 0) {
      atomicMax(&s_max[m], __float_as_int(mx));  // mx >= 0: bit order is value order
      if (bad) atomicOr(&s_bad[m], 1);
    }
    named_bar_sync(1, kClThreads);
    const float smax = __int_as_float(s_max[m]);
    const float inv = (smax > 0.0f && !s_bad[m]) ? 127.0f / smax : 0.0f;
    if (resident) {
      cl_store_digits<kRes>(v, inv, xd, plane, mt, m, gbeg + lane, gend);
      return;
    }
    for (int g0 = gbeg + lane; g0 < gend; g0 += 32 * kBatch) {
      float4 w[kBatch];
      cl_load_groups<kBatch, X_BF16, ROUND>(p, w, m, kbase, g0, gend, vec, ln);
      cl_store_digits<kBatch>(w, inv, xd, plane, mt, m, g0, gend);
    }
  }
};

// Per-token LayerNorm statistics over the whole row, with the reference's formula
// (src/ops/kernels_transformer.cpp:38-49): the mean, then the biased variance of
// the centred values, inv = 1 / sqrt(var + eps); ln[t] = mean, ln[kClMaxTokens + t] = inv.
// Warp w takes tokens w, w + 8, ...; each lane adds its elements in k order and
// the lanes are added in a fixed tree order. Every CTA of a split computes the
// same statistics from the same row.
__device__ void cl_ln_stats(const GemvClParams& p, float* ln, int warp, int lane) {
  const float* X = static_cast<const float*>(p.X);
  for (int t = warp; t < p.M; t += kClWarps) {
    const float* row = X + (int64_t)t * p.ldx;
    float s = 0.0f;
    for (int k = lane; k < p.K; k += 32) s += __ldg(row + k);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)p.K;
    float q = 0.0f;
    for (int k = lane; k < p.K; k += 32) {  // the row again, from L1
      const float c = __ldg(row + k) - mean;
      q += c * c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    if (lane == 0) {
      ln[t] = mean;
      ln[kClMaxTokens + t] = 1.0f / sqrtf(q / (float)p.K + p.ln_eps);
    }
  }
}

// NB: blocks of 8 tokens (M <= 8 * NB); more blocks need more registers, so fewer
// CTAs fit an SM (3 for one block, 2 for up to four, 1 for eight).
// LN: the LayerNorm prologue (p.ln_gamma) is compiled in (fp32 X only).
template <bool X_BF16, bool ROUND, int RES, int NB, bool LN>
__global__ void __launch_bounds__(kClBlock, NB == 1 ? kGemvClCtasPerSm
                                             : NB <= 4 ? kGemvClCtasPerSmWide : kGemvClCtasPerSmWide8)
    gemv_cluster_kernel(const GemvClParams p) {
  // Shared memory: ring [stages][8 KiB] (the exchange buffer part[8 * NB][128] fp32
  // reuses it at the end) | full[8], empty[8], xready (+ pad) barriers |
  // digits [3][nu][M][64] s8.
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_abort;
  __shared__ int s_max[kClMaxTokens], s_bad[kClMaxTokens];  // per token: max |x| (fp32 bits), non-finite flag
  __shared__ float s_sb[2][128];      // scale and bias of the rows this CTA finishes
  __shared__ float s_ln[2 * kClMaxTokens];  // LayerNorm mean and 1 / std per token
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int CS = (int)gridDim.x;  // the cluster spans x
  const int t = blockIdx.y;
  const int nst = p.stages;
  const int mt = p.M;

  // This CTA's units [u0, u1) of tile t.
  const int u0 = (int)((int64_t)rank * p.KB / CS), u1 = (int)((int64_t)(rank + 1) * p.KB / CS);
  const int nu = u1 - u0;
  unsigned char* ring = smem;
  const size_t ring_bytes = max((size_t)nst * kUnitBytes, (size_t)8 * NB * 128 * sizeof(float));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_bytes);
  uint64_t* empty = full + kGemvClMaxStages;
  uint64_t* xready = empty + kGemvClMaxStages;
  int8_t* xd = reinterpret_cast<int8_t*>(xready + 2);
  const int plane = nu * mt * 64;
  const int r0 = (int)(rank * 128 / CS), r1 = (int)((rank + 1) * 128 / CS);  // rows finished here

  // Roles before the block barrier:
  //  * producer thread: barrier setup, then the first weight units into the ring
  //    (weights are never written by a kernel this launch may overlap);
  //  * consumers: wait for the grid this launch depends on (a no-op unless it was
  //    launched with programmatic stream serialization), then issue the
  //    activation loads, whose latency overlaps the rest of the setup.
  ClStager<X_BF16, ROUND, RES, (NB > 1)> stager;
  const char* src = p.W + ((int64_t)t * p.KB + u0) * kUnitBytes;
  int issued = 0, st_p = 0;
  uint32_t ph_p = 0;
  const int prefill = min(min(p.early_units, nst), nu);
  if (tid == 0) grid_launch_dependents();
  if (warp == kClWarps) {
    if (lane == 0) {
      for (int i = 0; i < nst; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], kClWarps);
      }
      mbar_init(xready, kClWarps);
      s_abort = 0;
      for (int i = 0; i < kClMaxTokens; ++i) s_max[i] = s_bad[i] = 0;
      fence_barrier_init();
      for (; issued < prefill; ++issued) {
        mbar_arrive_expect_tx(&full[st_p], kUnitBytes);
        bulk_g2s(ring + (size_t)st_p * kUnitBytes, src + (int64_t)issued * kUnitBytes, kUnitBytes,
                 &full[st_p]);
        if (++st_p == nst) { st_p = 0; ph_p ^= 1u; }
      }
    }
  } else {
    grid_dependency_wait();
    stager.begin(p, u0, nu, warp, lane);
  }
  __syncthreads();

  int acc[NB][kDigits][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int d = 0; d < kDigits; ++d)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[nb][d][j] = 0;

  if (warp == kClWarps) {
    // Producer: one thread keeps up to nst units in flight. The activations are
    // read while the memory system is quiet: after early_units units the weight
    // stream waits until they have arrived.
    if (lane == 0) {
      for (int u = issued; u < nu; ++u) {
        if (u == p.early_units && !mbar_wait_bounded(xready, 0, &s_abort, p.status)) break;
        if (u >= nst && !mbar_wait_bounded(&empty[st_p], ph_p ^ 1u, &s_abort, p.status)) break;
        mbar_arrive_expect_tx(&full[st_p], kUnitBytes);
        bulk_g2s(ring + (size_t)st_p * kUnitBytes, src + (int64_t)u * kUnitBytes, kUnitBytes, &full[st_p]);
        ++issued;
        if (++st_p == nst) { st_p = 0; ph_p ^= 1u; }
      }
      // Every issued copy lands before the CTA moves on (and, on an abort, leaves).
      volatile int no_abort = 0;
      for (int u = issued > nst ? issued - nst : 0; u < issued; ++u)
        mbar_wait_bounded(&full[u % nst], (uint32_t)(u / nst) & 1u, &no_abort, p.status);
    } else {
      // The other producer lanes fetch the epilogue's scales and biases meanwhile
      // (weights-like data, as above).
      for (int r = r0 + lane - 1; r < r1; r += 31) {
        const int n = t * kTileN + r;
        s_sb[0][r] = n < p.N ? p.scale[n] : 0.0f;
        s_sb[1][r] = (p.bias && n < p.N) ? p.bias[n] : 0.0f;
      }
    }
    __syncwarp();
  } else {
    // Consumers: activation digits first (the weights are already in flight),
    // after the LayerNorm statistics when the call asks for them.
    if (LN && !X_BF16) {
      cl_ln_stats(p, s_ln, warp, lane);
      named_bar_sync(1, kClThreads);
      stager.ln = s_ln;
    }
    stager.finish(p, xd, plane, s_max, s_bad, xready, lane);
    named_bar_sync(1, kClThreads);
    // Warp w: channel rows w*16 + g and w*16 + g + 8 (g = lane / 4). MMA step i
    // of a unit covers k = 32i .. 32i + 31 (slabs 2i, 2i + 1); lane (g, c) holds
    // the activation words of token g at k = 4c + 16j (j = 0..3) as one 16-byte
    // load, words 2i and 2i + 1 feeding step i.
    const int g = lane >> 2, c = lane & 3;
    const int8_t* xg = xd + g * 64 + c * 16;  // token g of block 0; block nb adds 8 * nb tokens
    int st = 0;
    uint32_t ph = 0;
    for (int u = 0; u < nu; ++u) {
      if (!mbar_wait_bounded(&full[st], ph, &s_abort, p.status)) break;
      uint32_t a1[4], a2[4];
      ld_weight_frag(ring + (size_t)st * kUnitBytes, warp * 16, 0, lane, a1);
      ld_weight_frag(ring + (size_t)st * kUnitBytes, warp * 16, 2, lane, a2);
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        uint4 xv[kDigits];
        const bool has_x = 8 * nb + g < mt;
#pragma unroll
        for (int d = 0; d < kDigits; ++d)
          xv[d] = has_x ? *reinterpret_cast<const uint4*>(xg + d * plane + (u * mt + 8 * nb) * 64)
                        : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int d = 0; d < kDigits; ++d) {
          mma_s8(acc[nb][d], a1[0], a1[1], a1[2], a1[3], xv[d].x, xv[d].y);
          mma_s8(acc[nb][d], a2[0], a2[1], a2[2], a2[3], xv[d].z, xv[d].w);
        }
      }
      // The stage goes back to the producer only after the MMAs have consumed the
      // weights read from it: a shared memory read is not finished when issued, and
      // the next bulk copy into the stage must not overtake it.
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      if (++st == nst) { st = 0; ph ^= 1u; }
    }
  }
  __syncthreads();  // the ring is idle: every copy has landed and been read

  // Accumulators -> fp32 partials part[token][row] in this CTA's shared memory.
  // Element j of a warp's C fragment: row ra (j < 2) or ra + 8, token 2c + (j & 1).
  float* part = reinterpret_cast<float*>(smem);  // [8 * NB][128], read by the other ranks
  if (warp < kClWarps) {
    const int g = lane >> 2, c = lane & 3;
    const int ra = warp * 16 + g;
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = 8 * nb + 2 * c + (j & 1), row = ra + (j >> 1) * 8;
        float v = 0.0f;
        if (m < mt) {
          const float sm =
              s_bad[m] ? __int_as_float(0x7fc00000) : __int_as_float(s_max[m]) * (1.0f / 127.0f);
          v = sm * ((float)acc[nb][0][j] + (float)acc[nb][1][j] * (1.0f / 128.0f) +
                    (float)acc[nb][2][j] * (1.0f / 16384.0f));
        }
        part[m * 128 + row] = v;
      }
    }
  }

  // Rank s finishes rows [s * 128 / CS, (s + 1) * 128 / CS), summing the ranks'
  // partials in rank order.
  if (CS > 1) cluster_sync_all();
  else __syncthreads();
  const int nr = r1 - r0;
  for (int e = tid; e < nr * mt; e += kClBlock) {
    const int m = e / nr, r = r0 + (e - m * nr);
    const int n = t * kTileN + r;
    float sum;
    if (CS > 1) {
      // All ranks' values are requested before the first is used.
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < CS) v[q] = ld_dsmem_f32(dsmem_addr(part + m * 128 + r, (uint32_t)q));
      sum = 0.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < CS) sum += v[q];
    } else {
      sum = part[m * 128 + r];
    }
    if (n < p.N) {
      float y = __fmul_rn(sum, s_sb[0][r]);
      if (p.bias) y = __fadd_rn(y, s_sb[1][r]);
      p.Y[(int64_t)m * p.ldy + n] = epi_apply(p.epi, y, m, n);
    }
  }
  // No CTA leaves while another rank may still read its shared memory. Those
  // reads have returned (their values are summed above), so the arrival needs
  // no release ordering.
  if (CS > 1) cluster_sync_relaxed();
}

template <bool X_BF16, bool ROUND, int RES, int NB, bool LN = false>
cudaError_t cl_launch(const GemvClParams& gp, int cs, int n_tiles, size_t smem, bool pdl, cudaStream_t st) {
  auto kern = gemv_cluster_kernel<X_BF16, ROUND, RES, NB, LN>;
  // Always raised (once per device and instance): the 48 KiB default covers dynamic
  // and static shared memory together, so a dynamic size just under 48 KiB can
  // still exceed it.
  if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern),
                                        (int)(NB == 1 ? kGemvClSmemCap
                                              : NB <= 4 ? kGemvClSmemCapWide : kGemvClSmemCapWide8)))
    return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cs, (unsigned)n_tiles, 1);
  cfg.blockDim = dim3(kClBlock, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, gp);
}

}  // namespace

// Blocks of 8 tokens of the kernel instance that serves m tokens (its NB).
static int cl_token_blocks(int m) { return m <= 8 ? 1 : m <= 16 ? 2 : m <= 32 ? 4 : 8; }

size_t gemv_cluster_smem_bytes(int m, int64_t units, int cs, int stages) {
  const int64_t nu = (units + cs - 1) / cs;  // the largest CTA range
  const size_t ring = (size_t)stages * kUnitBytes;
  // The exchange buffer part[8 * NB][128] (it reuses the ring): the kernel writes
  // all 8 * NB token rows, so it is sized by NB, not by m.
  const size_t exch = (size_t)cl_token_blocks(m) * 8 * 128 * sizeof(float);
  return (ring > exch ? ring : exch) + (2 * kGemvClMaxStages + 2) * sizeof(uint64_t) +
         (size_t)kDigits * (size_t)nu * (size_t)m * 64;
}

cudaError_t launch_gemv_cluster(const Plan& p, const void* X, int x_dtype, int64_t ldx,
                                const void* packed, const float* scale, const float* bias, float* Y,
                                int64_t ldy, unsigned* status, bool pdl, const Epilogue& epi,
                                cudaStream_t st, const float* ln_gamma, const float* ln_beta,
                                float ln_eps) {
  GemvClParams gp;
  gp.ln_gamma = ln_gamma;
  gp.ln_beta = ln_beta;
  gp.ln_eps = ln_eps;
  gp.epi = epi;
  gp.X = X;
  gp.ldx = ldx;
  gp.W = static_cast<const char*>(packed);
  gp.scale = scale;
  gp.bias = bias;
  gp.Y = Y;
  gp.ldy = ldy;
  gp.M = (int)p.M;
  gp.K = (int)p.K;
  gp.N = (int)p.N;
  gp.KB = p.kunits;
  gp.stages = p.stages;
  gp.early_units = min(pdl ? kClEarlyUnitsPdl : kClEarlyUnits, p.stages);
  gp.status = status;
  const size_t smem = gemv_cluster_smem_bytes((int)p.M, p.kunits, p.splits, p.stages);
  // Activation groups a staging lane holds: 6 unless some warp's share needs
  // more to be staged in one pass (a token has floor(8 / M) warps; M > 8 stages
  // whole tokens per warp in batches).
  const int nb = cl_token_blocks((int)p.M);
  bool wide = false;
  if (p.M <= 8) {
    const int64_t nu_max = (p.kunits + p.splits - 1) / p.splits;
    const int64_t share = (nu_max * 16 + kClWarps / p.M - 1) / (kClWarps / p.M);
    wide = share > 32 * 6;
  }
#define MTRTQ_CL_LAUNCH(XB, RD)                                                                     \
  (nb == 1 ? (wide ? cl_launch<XB, RD, 12, 1>(gp, p.splits, p.n_tiles, smem, pdl, st)               \
                   : cl_launch<XB, RD, 6, 1>(gp, p.splits, p.n_tiles, smem, pdl, st))               \
   : nb == 2 ? cl_launch<XB, RD, 6, 2>(gp, p.splits, p.n_tiles, smem, pdl, st)                      \
   : nb == 4 ? cl_launch<XB, RD, 6, 4>(gp, p.splits, p.n_tiles, smem, pdl, st)                      \
             : cl_launch<XB, RD, 6, 8>(gp, p.splits, p.n_tiles, smem, pdl, st))
  if (ln_gamma) {
    // The LayerNorm prologue: fp32 X, six-group staging (longer shares are read twice).
    if (x_dtype == 1) return cudaErrorInvalidValue;
#define MTRTQ_CL_LAUNCH_LN(RD)                                                               \
  (nb == 1 ? cl_launch<false, RD, 6, 1, true>(gp, p.splits, p.n_tiles, smem, pdl, st)        \
   : nb == 2 ? cl_launch<false, RD, 6, 2, true>(gp, p.splits, p.n_tiles, smem, pdl, st)      \
   : nb == 4 ? cl_launch<false, RD, 6, 4, true>(gp, p.splits, p.n_tiles, smem, pdl, st)      \
             : cl_launch<false, RD, 6, 8, true>(gp, p.splits, p.n_tiles, smem, pdl, st))
    return p.round_x ? MTRTQ_CL_LAUNCH_LN(true) : MTRTQ_CL_LAUNCH_LN(false);
#undef MTRTQ_CL_LAUNCH_LN
  }
  if (x_dtype == 1) return MTRTQ_CL_LAUNCH(true, false);
  if (p.round_x) return MTRTQ_CL_LAUNCH(false, true);
  return MTRTQ_CL_LAUNCH(false, false);
#undef MTRTQ_CL_LAUNCH
}

}  // namespace mtrtq
