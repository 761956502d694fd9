// Persistent, balanced decode GEMV over a group of independent INT8 weight-only
// MatMulQ problems (M <= 8 tokens each) in one launch.
//
// Replaces, for a set of decode-size calls that do not depend on one another
// (the Q, K and V projections the reference's KV decoder runs one after another,
// tools/run_gpt2.cpp:142-150, or any batch of independent Linears), the
// reference's scalar MatMulQ loop (src/ops/kernels_matmul.cpp:66-73) called once
// per problem. Arithmetic is that of the cluster GEMV (gemv_cluster.cu): int8
// weights, unconverted, times three int8 digits of each activation on
// m16n8k32 s8 warp MMAs with exact int32 sums, combined in fp32, then
// (sum * scale) + bias, multiply then add.
//
// Work: the problems' 64-k weight units (8 KiB each, contiguous per problem in the
// packed layout: tile-major, then k) form one global list of U units. The grid is
// persistent -- three CTAs per SM, G <= U -- and CTA c takes the contiguous units
// [floor(c U / G), floor((c + 1) U / G)): every CTA streams the same number of
// bytes give or take one unit, whatever the problems' shapes, so no SM finishes
// early and the launch's fixed costs are paid once for the whole group.
//
// A CTA walks its range as segments (the part of one 128-channel tile it owns),
// each cut into chunks of at most kSChunk units whose activations are staged as
// digits together. A segment that is a whole tile is finished by its CTA; the
// parts of a tile cut between CTAs go to a workspace slot each, and the CTA that
// arrives last (a ticket per tile) sums them in CTA order -- a fixed order, so
// results do not depend on timing -- then applies scale, bias and the epilogue.
//
// Roles: one producer thread streams the CTA's units into a ring of shared memory
// stages with 1-D bulk async copies (no multicast); eight consumer warps, each
// owning 16 channel rows, stage the digits of a chunk, run the MMAs and keep the
// segment's fp32 partial sums in registers.
//
// Every mbarrier wait is bounded; a wait that gives up records MTRTQ_ERR_TIMEOUT
// in the device status word and the CTA stops doing work but keeps its barrier
// sequence, and the producer waits (bounded) for its own copies before leaving.
#include "q8_common.cuh"
#include "q8_digits.cuh"
#include "q8_internal.h"

namespace mtrtq {

namespace {

constexpr int kSWarps = 8;                 // consumers: one 16-row group each
constexpr int kSThreads = kSWarps * 32;    // consumer threads
constexpr int kSBlock = kSThreads + 32;    // + the producer warp
constexpr uint32_t kSUnit = 8192;          // 64 k x 128 channels of int8
constexpr int kSDigits = 3;
constexpr int kSRes = 6;                   // staged groups per lane: kSChunk * 16 / 32
constexpr int kSPlane = kSChunk * 8 * 64;  // one digit plane: [unit][token][64 k]

struct StreamParams {
  GroupProblem prob[kGroupMax];
  int count;
  int64_t units;      // U
  int grid;           // G
  unsigned* counters; // one ticket per tile of the group
  float* partials;    // [G][2][8 tokens][128 rows]
  unsigned* status;
  int producers;      // producer lanes (1, 2, 3 or 6: a divisor of the stage count)
};

__host__ __device__ __forceinline__ int64_t range_start(int64_t c, int64_t U, int64_t G) { return c * U / G; }

// The CTA whose range holds unit u: the largest c with range_start(c) <= u.
__device__ __forceinline__ int64_t cta_of_unit(int64_t u, int64_t U, int64_t G) {
  return ((u + 1) * G + U - 1) / U - 1;
}

// Stages the digits of tokens [0, M) over units [ku, ku + nu) of problem P into
// xd (plane d at xd + d * kSPlane, unit i, token m at ((i * M + m) * 64)), with
// each token's max |x| (ordered bits) in smax[m] and a non-finite flag in sbad[m].
// Token m is staged by the warps w with w % M == m, each taking an equal share of
// the chunk's 4-element groups (at most kSRes per lane).
template <bool X_BF16, bool ROUND>
__device__ __forceinline__ void stage_chunk(const GroupProblem& P, int ku, int nu, int8_t* xd, int* smax,
                                            int* sbad, int* snext_max, int* snext_bad, int warp, int lane,
                                            int tid) {
  const int M = P.M;
  const int m = warp % M;
  const int share = (kSWarps - 1 - m) / M + 1;  // warps staging token m
  const int j = warp / M;
  const int n4 = nu * 16;
  const int gbeg = j * n4 / share, gend = (j + 1) * n4 / share;
  const int kbase = ku * 64;
  const bool vec = (P.ldx & 3) == 0;
  float4 v[kSRes];
  float mx = 0.0f;
  bool bad = false;
#pragma unroll
  for (int b = 0; b < kSRes; ++b) {
    const int g = gbeg + lane + 32 * b;
    v[b] = g < gend ? cl_round<ROUND>(load_x4<X_BF16>(P.X, P.ldx, P.K, m, kbase + g * 4, vec))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int b = 0; b < kSRes; ++b) mx = fmaxf(mx, cl_group_max(v[b], bad));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, (int)bad, o) != 0;
  }
  if (lane == 0) {
    atomicMax(&smax[m], __float_as_int(mx));  // mx >= 0: bit order is value order
    if (bad) atomicOr(&sbad[m], 1);
  }
  named_bar_sync(1, kSThreads);
  // Every consumer has finished the previous chunk (its fold read the other
  // buffer's maxima): clear that buffer for the next chunk.
  if (tid < 8) {
    snext_max[tid] = 0;
    snext_bad[tid] = 0;
  }
  const float s = __int_as_float(smax[m]);
  const float inv = (s > 0.0f && !sbad[m]) ? 127.0f / s : 0.0f;
#pragma unroll
  for (int b = 0; b < kSRes; ++b) {
    const int g = gbeg + lane + 32 * b;
    if (g < gend) cl_store_digit_group(v[b], inv, xd, kSPlane, M, m, g);
  }
  named_bar_sync(1, kSThreads);
}

template <bool X_BF16, bool ROUND>
__global__ void __launch_bounds__(kSBlock, kSCtasPerSm) gemv_stream_kernel(const __grid_constant__ StreamParams p) {
  // Shared memory: ring [stages][8 KiB] | full[stages], empty[stages] | digits [3][kSPlane].
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int s_abort;
  __shared__ int s_max[2][8], s_bad[2][8];
  __shared__ unsigned s_last[1];  // ticket of the cut tile being handed over
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nst = kSStages;
  unsigned char* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)nst * kSUnit);
  uint64_t* empty = full + nst;
  int8_t* xd = reinterpret_cast<int8_t*>(empty + nst);

  const int64_t U = p.units, G = p.grid, cta = blockIdx.x;
  const int64_t ub = range_start(cta, U, G), ue = range_start(cta + 1, U, G);

  if (tid == 0) grid_launch_dependents();
  if (tid == kSThreads) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSWarps);
    }
    s_abort = 0;
    for (int i = 0; i < 8; ++i) s_max[0][i] = s_bad[0][i] = s_max[1][i] = s_bad[1][i] = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kSWarps) {
    // Producer: weights only (never written by a kernel this launch may overlap),
    // so no wait for the grid ahead.
    // Lane l < np issues the CTA's units i = l, l + np, ... (np divides the stage
    // count, so a lane always refills the same stages): one thread's bulk copies
    // complete one after another, and several issuing lanes keep more of them in
    // flight.
    const int np = p.producers;
    if (lane < np) {
      int pi = 0;
      while (pi + 1 < p.count && p.prob[pi + 1].unit_begin <= ub) ++pi;
      const int64_t n = ue - ub;
      int64_t i = lane;
      for (; i < n; i += np) {
        const int st = (int)(i % nst);
        const uint32_t ph = (uint32_t)(i / nst) & 1u;
        if (i >= nst && !mbar_wait_bounded(&empty[st], ph ^ 1u, &s_abort, p.status)) break;
        const int64_t u = ub + i;
        while (pi + 1 < p.count && p.prob[pi + 1].unit_begin <= u) ++pi;
        const char* src = p.prob[pi].W + (u - p.prob[pi].unit_begin) * (int64_t)kSUnit;
        mbar_arrive_expect_tx(&full[st], kSUnit);
        bulk_g2s(ring + (size_t)st * kSUnit, src, kSUnit, &full[st]);
      }
      // Every copy this lane issued lands before the CTA leaves.
      volatile int no_abort = 0;
      for (int64_t j = i - np; j >= 0 && j >= i - (int64_t)nst; j -= np)
        mbar_wait_bounded(&full[j % nst], (uint32_t)(j / nst) & 1u, &no_abort, p.status);
    }
    __syncwarp();
  } else {
    grid_dependency_wait();  // X, Y, the workspace: after the grid ahead
    const int g = lane >> 2, c = lane & 3;
    const int ra = warp * 16 + g;
    int pi = 0;
    while (pi + 1 < p.count && p.prob[pi + 1].unit_begin <= ub) ++pi;
    int64_t rem = ue - ub;
    int64_t lu = ub - p.prob[pi].unit_begin;  // unit within the problem
    int t = (int)(lu / p.prob[pi].KB);
    int ku = (int)(lu - (int64_t)t * p.prob[pi].KB);
    int seg_start = ku;
    bool seg_first = true;
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    int st = 0, chunk = 0;
    uint32_t ph = 0;
    bool ok = true;
    while (rem > 0) {
      const GroupProblem& P = p.prob[pi];
      const int nu = (int)min((int64_t)min(kSChunk, P.KB - ku), rem);
      const int buf = chunk & 1;
      stage_chunk<X_BF16, ROUND>(P, ku, nu, xd, s_max[buf], s_bad[buf], s_max[buf ^ 1], s_bad[buf ^ 1], warp,
                                 lane, tid);
      int acc[kSDigits][4];
#pragma unroll
      for (int d = 0; d < kSDigits; ++d)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[d][jj] = 0;
      const bool has_x = g < P.M;
      const int8_t* xg = xd + g * 64 + c * 16;
      for (int i = 0; i < nu; ++i) {
        ok = ok && mbar_wait_bounded(&full[st], ph, &s_abort, p.status);
        if (ok) {
          uint32_t a1[4], a2[4];
          ld_weight_frag(ring + (size_t)st * kSUnit, warp * 16, 0, lane, a1);
          ld_weight_frag(ring + (size_t)st * kSUnit, warp * 16, 2, lane, a2);
          uint4 xv[kSDigits];
#pragma unroll
          for (int d = 0; d < kSDigits; ++d)
            xv[d] = has_x ? *reinterpret_cast<const uint4*>(xg + d * kSPlane + i * P.M * 64)
                          : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int d = 0; d < kSDigits; ++d) {
            mma_s8(acc[d], a1[0], a1[1], a1[2], a1[3], xv[d].x, xv[d].y);
            mma_s8(acc[d], a2[0], a2[1], a2[2], a2[3], xv[d].z, xv[d].w);
          }
        }
        // The stage goes back to the producer after the MMAs that read it.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (++st == nst) { st = 0; ph ^= 1u; }
      }
      // Fold the chunk's integer sums into the segment's fp32 partials. C fragment
      // element jj: row ra (jj < 2) or ra + 8, token 2c + (jj & 1).
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int m = 2 * c + (jj & 1);
        if (m < P.M) {
          const float sm = s_bad[buf][m] ? __int_as_float(0x7fc00000)
                                         : __int_as_float(s_max[buf][m]) * (1.0f / 127.0f);
          part[jj] += sm * ((float)acc[0][jj] + (float)acc[1][jj] * (1.0f / 128.0f) +
                            (float)acc[2][jj] * (1.0f / 16384.0f));
        }
      }
      ku += nu;
      rem -= nu;
      ++chunk;
      if (ku < P.KB && rem > 0) continue;  // the segment goes on

      // ---- the segment ends: finish the tile, or store this CTA's part of it ----
      if (seg_start == 0 && ku == P.KB) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int m = 2 * c + (jj & 1), row = ra + (jj >> 1) * 8;
          const int n = t * kTileN + row;
          if (m < P.M && n < P.N) {
            float y = __fmul_rn(part[jj], __ldg(P.scale + n));
            if (P.bias) y = __fadd_rn(y, __ldg(P.bias + n));
            P.Y[(int64_t)m * P.ldy + n] = epi_apply(P.epi, y, m, n);
          }
        }
      } else {
        const int sl = seg_first ? 0 : 1;
        float* slot = p.partials + ((cta * 2 + sl) * 8) * kTileN;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int m = 2 * c + (jj & 1), row = ra + (jj >> 1) * 8;
          if (m < P.M) __stcg(slot + m * kTileN + row, part[jj]);
        }
        named_bar_sync(1, kSThreads);  // every part of this CTA is stored
        unsigned* counter = p.counters + P.tile_begin + t;
        if (tid == 0) s_last[0] = ticket_acq_rel(counter);
        named_bar_sync(1, kSThreads);
        const int64_t T0 = P.unit_begin + (int64_t)t * P.KB;  // the tile's first unit
        const int64_t c_lo = cta_of_unit(T0, U, G), c_hi = cta_of_unit(T0 + P.KB - 1, U, G);
        if (s_last[0] == (unsigned)(c_hi - c_lo)) {
          // The last CTA to arrive sums the parts in CTA order. The first part is
          // the lowest CTA's last segment unless the tile starts its range; every
          // later CTA's part is its first segment.
          const int first_slot = range_start(c_lo, U, G) == T0 ? 0 : 1;
          for (int e = tid; e < kTileN * P.M; e += kSThreads) {
            const int m = e / kTileN, row = e - m * kTileN;
            const int n = t * kTileN + row;
            float sum = 0.0f;
            for (int64_t cc = c_lo; cc <= c_hi; ++cc) {
              const int csl = cc == c_lo ? first_slot : 0;
              sum += __ldcg(p.partials + ((cc * 2 + csl) * 8 + m) * kTileN + row);
            }
            if (n < P.N) {
              float y = __fmul_rn(sum, __ldg(P.scale + n));
              if (P.bias) y = __fadd_rn(y, __ldg(P.bias + n));
              P.Y[(int64_t)m * P.ldy + n] = epi_apply(P.epi, y, m, n);
            }
          }
          if (tid == 0) *counter = 0u;  // left at zero for the next call
        }
      }
      seg_first = false;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) part[jj] = 0.0f;
      if (ku == P.KB) {  // the next tile, or the next problem's first
        ku = 0;
        if (++t == P.n_tiles) {
          t = 0;
          ++pi;
        }
      }
      seg_start = ku;
    }

  }
  __syncthreads();  // the ring is idle: every copy has landed and been read
}

template <bool X_BF16, bool ROUND>
cudaError_t stream_launch(const StreamParams& sp, bool pdl, cudaStream_t st) {
  auto kern = gemv_stream_kernel<X_BF16, ROUND>;
  if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), (int)kStreamSmemBytes)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sp.grid, 1, 1);
  cfg.blockDim = dim3(kSBlock, 1, 1);
  cfg.dynamicSmemBytes = kStreamSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, sp);
}

}  // namespace

cudaError_t launch_gemv_stream(const GroupProblem* probs, int count, int64_t units, int grid, int x_dtype,
                               bool round_x, void* workspace, unsigned* status, bool pdl, int producers,
                               cudaStream_t st) {
  StreamParams sp;
  sp.producers = producers;
  for (int i = 0; i < count; ++i) sp.prob[i] = probs[i];
  sp.count = count;
  sp.units = units;
  sp.grid = grid;
  sp.counters = static_cast<unsigned*>(workspace);
  sp.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kStreamCounterBytes);
  sp.status = status;
  if (x_dtype == 1) return stream_launch<true, false>(sp, pdl, st);
  if (round_x) return stream_launch<false, true>(sp, pdl, st);
  return stream_launch<false, false>(sp, pdl, st);
}

}  // namespace mtrtq
