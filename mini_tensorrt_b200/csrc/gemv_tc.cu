// Tensor-core digit GEMV: INT8 weight-only MatMulQ for up to 64 tokens, a group
// of independent problems in one persistent launch, on tcgen05 kind::i8 MMAs.
//
// Replaces, for decode-size calls (the projections, FFN and LM head of the
// reference's KV decoder, tools/run_gpt2.cpp:142-187, and any batch of
// independent Linears), the reference's scalar MatMulQ loop
// (src/ops/kernels_matmul.cpp:66-73): Y[m, n] = (sum_k X[m, k] * q[k, n]) *
// scale[n] + bias[n], the sum first, then the scale, then the bias.
//
// Arithmetic. Each activation row m is written as four int8 digits,
//   X[m, k] ~ (s_m / 127) * (d0 + d1 / 2^7 + d2 / 2^14 + d3 / 2^21),
// s_m = max_k |X[m, k]|, every digit in [-127, 127]; the representation error is
// at most 2^-22 * s_m / 127 per element (fp32 itself keeps 24 bits). The int8
// weights are multiplied by each digit exactly on the tensor cores (s32 sums,
// no overflow below K = 2^31 / 127^2 ~ 133k), and the four sums are combined in
// fp32. In bf16 mode X is rounded to bf16 first; the digits then hold it exactly.
//
// Launches. digitize_kernel: one block per (token, problem) reads the row once for
// its max and once for its digits, and writes them straight into the MMA's
// operand layout (below), so the GEMV streams them with bulk copies like the
// weights. gemv_tc_kernel: persistent, one CTA per SM; the group's 64-k weight
// units (8 KiB each) form one list, and CTA c takes the contiguous units
// [c U / G, (c + 1) U / G), so every SM streams the same number of bytes whatever
// the problems' shapes. Both launch with programmatic dependent launch when
// asked: the GEMV's producer starts streaming weights (never written by a kernel)
// while the digitize kernel runs, and waits for it only before the first digits.
//
// Roles (192 threads): warp 0 lane 0 is the producer, which keeps a ring of
// stages full, each stage one weight unit plus the unit's digits; warp 1 holds the
// tensor memory and its lane 0 issues the MMAs: for every unit two
// tcgen05.mma.kind::i8 (M = 128 channels, N = 4 x NT, K = 32) read both operands
// from the stage, and a tcgen05.commit hands the stage back to the producer;
// warps 2..5 are the epilogue, one TMEM lane quarter (32 channels) each. A CTA's
// range is a sequence of segments (its part of one 128-channel tile); each
// segment accumulates in one of up to eight TMEM buffers, so the MMAs of later
// segments run while the epilogue drains the earlier ones. A segment that is a
// whole tile is finished in place (scale, bias, epilogue); of a tile cut between
// CTAs, the CTA holding its last unit adds the others' parts (from workspace
// slots, counted on a per-tile counter) in CTA order ahead of its own -- a fixed
// order, so results do not depend on timing.
//
// Operand layouts (K-major, no swizzle: 8-row x 16-byte core matrices). A: the
// packed weight unit as it is in memory, 16-k slabs of 128 channel rows x 16
// bytes (leading byte offset 2048, stride byte offset 128). B: the digits of one
// unit, 16-k slabs of 4 NT rows (row d * NT + m: digit d of token m) x 16 bytes
// (leading byte offset 64 NT, stride byte offset 128). D[channel, d * NT + m] is
// then the digit-d sum of token m, in TMEM lane = channel, column = d * NT + m.
//
// Every wait is bounded (mbarriers, a finisher's wait for the parts); a wait that
// gives up records MTRTQ_ERR_TIMEOUT in the device status word and the CTA stops
// issuing work but keeps every named barrier and counts its parts, so it ends; the
// producer waits (bounded) for its own copies and the MMA thread for its own MMAs
// before the CTA leaves. After a timeout the workspace is to be zero-filled again.
#include "q8_common.cuh"
#include "q8_digits.cuh"
#include "q8_internal.h"

namespace mtrtq {

namespace {

constexpr int kTcThreads = 192;  // producer warp, MMA warp, four epilogue warps
constexpr int kTcEpiThreads = 128;
constexpr uint32_t kTcUnit = 8192;  // 64 k x 128 channels of int8
constexpr int kTcMaxStages = 24;
constexpr int kTcEarlyStages = 4;  // weight stages issued before the wait for the digits
constexpr size_t kTcSmemPerSm = 220 * 1024;

// Two CTAs per SM up to NT = 32 (two independent rings stream faster than one
// ring twice as deep: B200, the decode set, 26.6 us against 36.9 us), one at 64.
template <int NT>
struct TcCfg {
  static constexpr int kCtas = NT == 64 ? 1 : 2;
  static constexpr int kRows = 4 * NT;                        // B rows: 4 digits x NT tokens
  static constexpr uint32_t kDigitBytes = 256u * NT;          // B of one 64-k unit
  static constexpr uint32_t kStage = kTcUnit + kDigitBytes;
  static constexpr int kAccCols = 4 * NT;                     // s32 columns of one accumulator
  // Accumulator buffers: the CTA's share of the 512 TMEM columns, one segment
  // each, so that the MMAs run up to kBufs - 1 segments ahead of the epilogue.
  static constexpr uint32_t kTmemCols = 512 / kCtas;
  static constexpr int kBufs = (int)kTmemCols / kAccCols;     // 8, 4, 2 (NT = 8, 16, 32), 2 (64)
  static constexpr size_t kBudget = kTcSmemPerSm / kCtas;
  static constexpr int kStages = (int)(kBudget / kStage) < kTcMaxStages ? (int)(kBudget / kStage) : kTcMaxStages;
  static constexpr size_t kSmem = (size_t)kStages * kStage;
  static_assert(kBufs >= 2 && kBufs <= 8 && kStages >= 4, "tensor memory or shared memory too small");
};

struct TcParams {
  GroupProblem prob[kGroupMax];
  int8_t* digits[kGroupMax];  // per problem: KB units of TcCfg::kDigitBytes
  float* scales;                    // [kGroupMax][kTcMaxTokens]: s_m, NaN for a non-finite row
  int count;
  int nt;
  int64_t units;  // U
  int grid;       // G
  unsigned* counters;
  float* partials;  // [G][2][nt][128]
  unsigned* status;
  const float* ln_gamma;  // non-null: the rows of X (fp32, one problem) are layer-normalized first
  const float* ln_beta;
  float ln_eps;
  TcExchange xc;          // the fused all-gather (xc.world > 1)
};

__host__ __device__ __forceinline__ int64_t tc_range_start(int64_t c, int64_t U, int64_t G) { return c * U / G; }

// The CTA whose range holds unit u: the largest c with tc_range_start(c) <= u.
__device__ __forceinline__ int64_t tc_cta_of_unit(int64_t u, int64_t U, int64_t G) {
  return ((u + 1) * G + U - 1) / U - 1;
}

// Four int8 digits of v (|v| <= 127), each residual exact in fp32 (the difference
// of two nearby values, scaled by a power of two); the bit patterns of the four
// rounding sums go to w[0..3], whose low bytes are the digits.
__device__ __forceinline__ void tc_digits4(float v, uint32_t (&w)[4]) {
  float r = v;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const float t = __fadd_rn(r, kRoundMagic);
    w[d] = __float_as_uint(t);
    r = __fmul_rn(__fsub_rn(r, __fsub_rn(t, kRoundMagic)), 128.0f);
  }
}

// Digitize blocks are small, so that one fits beside two GEMV CTAs on an SM
// (registers) while the two launches overlap.
constexpr int kDigitizeThreads = 128;
constexpr int kDigitizeWarps = kDigitizeThreads / 32;

// Sum over the block in a fixed order: a shuffle tree in each warp, then the warp
// sums in warp order.
__device__ __forceinline__ float block_sum(float v, float* red, int warp, int lane) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red is free (an earlier sum has been read)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kDigitizeWarps; ++w) t += red[w];
  return t;
}

// Four activations of row m from k, layer-normalized when LN (the reference's
// (x - mean) * inv * gamma + beta, src/ops/kernels_transformer.cpp:50-51; zeros
// past K), then rounded to bf16 when ROUND.
template <bool X_BF16, bool ROUND, bool LN>
__device__ __forceinline__ float4 tc_load4(const TcParams& p, const GroupProblem& P, int m, int k, bool vec,
                                           float mean, float inv) {
  float4 v = load_x4<X_BF16>(P.X, P.ldx, P.K, m, k, vec);
  if (LN) {
    float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      a[i] = k + i < P.K ? (a[i] - mean) * inv * __ldg(p.ln_gamma + k + i) + __ldg(p.ln_beta + k + i) : 0.0f;
    v = make_float4(a[0], a[1], a[2], a[3]);
  }
  return cl_round<ROUND>(v);
}

// One block per (token m, problem): s_m and the four digit planes of row m (zeros
// for m >= M and for k >= K), written as B operand units. With LN the row's
// statistics come first, with the reference's formula
// (src/ops/kernels_transformer.cpp:38-49): the mean, then the biased variance of
// the centred values, inv = 1 / sqrt(var + eps).
template <bool X_BF16, bool ROUND, bool LN>
__global__ void __launch_bounds__(kDigitizeThreads) digitize_kernel(const __grid_constant__ TcParams p) {
  __shared__ float s_red[kDigitizeThreads / 32];
  __shared__ int s_bad[kDigitizeThreads / 32];
  const int m = blockIdx.x, pi = blockIdx.y;
  const GroupProblem& P = p.prob[pi];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nt = p.nt;
  grid_launch_dependents();
  grid_dependency_wait();  // X comes from the grid ahead; the digits may still be read by it
  if (p.xc.world > 1 && p.xc.epoch == 0 && m == 0 && pi == 0 && tid == 0) {
    unsigned* e = p.xc.flags[p.xc.rank] + kShardFlagEpoch;  // this call's count, read by the GEMV's last CTA
    *e = *e + 1u;
  }
  const bool live = m < P.M;
  const int groups = P.KB * 16;  // 4-element groups over the padded row
  const bool vec = (P.ldx & 3) == 0;
  float ln_mean = 0.0f, ln_inv = 1.0f;
  if (LN) {
    const float* row = static_cast<const float*>(P.X) + (int64_t)(live ? m : 0) * P.ldx;
    float s = 0.0f;
    if (live)
      for (int k = tid; k < P.K; k += kDigitizeThreads) s += __ldg(row + k);
    ln_mean = block_sum(s, s_red, warp, lane) / (float)P.K;
    float q = 0.0f;
    if (live)
      for (int k = tid; k < P.K; k += kDigitizeThreads) {
        const float c = __ldg(row + k) - ln_mean;
        q += c * c;
      }
    ln_inv = 1.0f / sqrtf(block_sum(q, s_red, warp, lane) / (float)P.K + p.ln_eps);
    __syncthreads();  // s_red is reused below
  }
  float mx = 0.0f;
  bool bad = false;
  if (live) {
    for (int g = tid; g < groups; g += kDigitizeThreads)
      mx = fmaxf(mx, cl_group_max(tc_load4<X_BF16, ROUND, LN>(p, P, m, 4 * g, vec, ln_mean, ln_inv), bad));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, (int)bad, o) != 0;
  }
  if (lane == 0) {
    s_red[warp] = mx;
    s_bad[warp] = bad;
  }
  __syncthreads();
  float s = 0.0f;
  bool any_bad = false;
#pragma unroll
  for (int w = 0; w < kDigitizeWarps; ++w) {
    s = fmaxf(s, s_red[w]);
    any_bad |= s_bad[w] != 0;
  }
  if (tid == 0) p.scales[pi * kTcMaxTokens + m] = any_bad ? __int_as_float(0x7fc00000) : s;
  const float inv = (s > 0.0f && !any_bad) ? 127.0f / s : 0.0f;
  int8_t* out = p.digits[pi];
  const int plane = 64 * nt;  // bytes of one 16-k slab of B
  for (int g = tid; g < groups; g += kDigitizeThreads) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = tc_load4<X_BF16, ROUND, LN>(p, P, m, 4 * g, vec, ln_mean, ln_inv);
    uint32_t a[4], b[4], c[4], e[4];
    tc_digits4(__fmul_rn(v.x, inv), a);
    tc_digits4(__fmul_rn(v.y, inv), b);
    tc_digits4(__fmul_rn(v.z, inv), c);
    tc_digits4(__fmul_rn(v.w, inv), e);
    // group g: unit g / 16, slab (g / 4) % 4, bytes 4 (g % 4) .. + 3 of the row
    int8_t* base = out + (size_t)(g >> 4) * (256 * nt) + ((g >> 2) & 3) * plane + (g & 3) * 4;
#pragma unroll
    for (int d = 0; d < 4; ++d)
      *reinterpret_cast<uint32_t*>(base + (d * nt + m) * 16) = cl_pack_low_bytes(a[d], b[d], c[d], e[d]);
  }
}

__device__ __forceinline__ int tc_problem_of(const TcParams& p, int64_t u) {
  int pi = 0;
  while (pi + 1 < p.count && p.prob[pi + 1].unit_begin <= u) ++pi;
  return pi;
}

// The order in which a CTA takes its range [ub, ue): the last segment first (the
// part of the tile it shares with the next CTA), then [ub, ls) from the start, so
// that the parts of every cut tile are done early and the tile's hand-off
// overlaps the streaming of the whole tiles; the launch then ends on a whole
// tile. Returns ls, the last segment's first unit
// (ub when the range lies inside one tile).
__device__ __forceinline__ int64_t tc_last_segment(const TcParams& p, int64_t ub, int64_t ue) {
  const int pi = tc_problem_of(p, ue - 1);
  const GroupProblem& P = p.prob[pi];
  const int64_t tile_start = P.unit_begin + (ue - 1 - P.unit_begin) / P.KB * P.KB;
  return tile_start > ub ? tile_start : ub;
}

// A CTA's walk over its units as segments, in the order above: units
// [ku, ku + seg_units()) of tile t of problem pi, starting at unit u; the MMA
// thread and the epilogue each walk it.
struct TcWalk {
  int pi, t, ku;
  int64_t u, rem;
  int64_t next_b, next_e;  // the second part of the range, once the first is done
  __device__ __forceinline__ void start(const TcParams& p, int64_t b, int64_t e) {
    pi = tc_problem_of(p, b);
    const int64_t lu = b - p.prob[pi].unit_begin;
    t = (int)(lu / p.prob[pi].KB);
    ku = (int)(lu - (int64_t)t * p.prob[pi].KB);
    u = b;
    rem = e - b;
  }
  __device__ __forceinline__ void init(const TcParams& p, int64_t ub, int64_t ue) {
    const int64_t ls = tc_last_segment(p, ub, ue);
    start(p, ls, ue);
    next_b = ub;
    next_e = ls;
  }
  __device__ __forceinline__ int seg_units(const TcParams& p) const {
    const int64_t left = p.prob[pi].KB - ku;
    return (int)(left < rem ? left : rem);
  }
  __device__ __forceinline__ void advance(const TcParams& p, int nu) {
    ku += nu;
    u += nu;
    rem -= nu;
    if (rem == 0 && next_b < next_e) {
      start(p, next_b, next_e);
      next_b = next_e;
      return;
    }
    if (ku == p.prob[pi].KB) {
      ku = 0;
      if (++t == p.prob[pi].n_tiles) {
        t = 0;
        ++pi;
      }
    }
  }
};

// The producer's position in the same order, one unit at a time: the problem,
// the unit's index lu within it and its 64-k index ku within its tile, kept
// without a division except when it enters another problem or range part.
struct TcCursor {
  int pi, ku;
  int64_t u, lu, end, next_b, next_e;
  __device__ __forceinline__ void start(const TcParams& p, int64_t b, int64_t e) {
    u = b;
    end = e;
    pi = tc_problem_of(p, b);
    lu = b - p.prob[pi].unit_begin;
    ku = (int)(lu % p.prob[pi].KB);
  }
  __device__ __forceinline__ void init(const TcParams& p, int64_t ub, int64_t ue) {
    const int64_t ls = tc_last_segment(p, ub, ue);
    start(p, ls, ue);
    next_b = ub;
    next_e = ls;
  }
  __device__ __forceinline__ void step(const TcParams& p) {
    ++u;
    ++lu;
    if (u == end) {
      if (next_b < next_e) {
        start(p, next_b, next_e);
        next_b = next_e;
      }
      return;
    }
    if (pi + 1 < p.count && p.prob[pi + 1].unit_begin <= u) {
      ++pi;
      lu = 0;
      ku = 0;
    } else if (++ku == p.prob[pi].KB) {
      ku = 0;
    }
  }
  __device__ __forceinline__ const char* weights(const TcParams& p) const {
    return p.prob[pi].W + lu * (int64_t)kTcUnit;
  }
  __device__ __forceinline__ const int8_t* digits(const TcParams& p, uint32_t unit_bytes) const {
    return p.digits[pi] + (size_t)ku * unit_bytes;
  }
};

// t = (s_m / 127 * v) * scale[n] (+ bias[n]), then the call's epilogue.
__device__ __forceinline__ float tc_finish(const GroupProblem& P, float v, float s_m, int m, int n) {
  float y = __fmul_rn(__fmul_rn(s_m * (1.0f / 127.0f), v), __ldg(P.scale + n));
  if (P.bias) y = __fadd_rn(y, __ldg(P.bias + n));
  return epi_apply(P.epi, y, m, n);
}

// Y[m, n] = y here, and at the same offset in every peer's output buffer when the
// group's all-gather is fused (stores over NVLink, released by the last CTA).
__device__ __forceinline__ void tc_store(const TcParams& p, const GroupProblem& P, int m, int n, float y) {
  float* dst = P.Y + (int64_t)m * P.ldy + n;
  *dst = y;
  if (p.xc.world > 1) {
    const int64_t off = reinterpret_cast<const char*>(dst) - p.xc.own_base;
    for (int r = 0; r < p.xc.world; ++r)
      if (r != p.xc.rank) *reinterpret_cast<float*>(p.xc.peer_base[r] + off) = y;
  }
}

__device__ __forceinline__ void fence_acq_rel_sys_tc() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_relaxed_sys_tc(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys_tc(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The fused all-gather's end, by one thread of each CTA after all its stores
// (a barrier of the threads that made them comes first): the CTA's stores are
// released to this GPU with the rank's ticket; the last CTA acquires them all,
// releases them to the peers with one system-scope fence, adds one arrival to every
// peer's data flag, then waits, bounded, until every peer's arrival for this call is
// in its own (it signalled first, so no rank waits on one that has not signalled).
// The launch ends when this rank holds every rank's outputs.
__device__ __noinline__ void tc_exchange_end(const TcParams& p) {
  const TcExchange& xc = p.xc;
  unsigned* own = xc.flags[xc.rank];
  if (ticket_acq_rel(own + kShardFlagTicket) != (unsigned)(p.grid - 1)) return;
  fence_acq_rel_sys_tc();
  own[kShardFlagTicket] = 0u;
  const unsigned epoch = xc.epoch != 0 ? xc.epoch : *reinterpret_cast<volatile unsigned*>(own + kShardFlagEpoch);
  for (int r = 0; r < xc.world; ++r)
    if (r != xc.rank) red_add_relaxed_sys_tc(xc.flags[r] + kShardFlagData, 1u);
  const unsigned target = epoch * (unsigned)(xc.world - 1);
  const long long t0 = clock64();
  while ((int)(ld_relaxed_sys_tc(own + kShardFlagData) - target) < 0) {
    if (clock64() - t0 > kSpinLimitCycles) {
      atomicExch(p.status, 6u /* MTRTQ_ERR_TIMEOUT */);
      return;
    }
  }
  fence_acq_rel_sys_tc();
}

__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits, bounded, until *counter reaches want (the parts of the other CTAs of a
// cut tile are stored); false after recording MTRTQ_ERR_TIMEOUT, or once another
// role of the CTA has given up.
__device__ __noinline__ bool tc_wait_parts(const unsigned* counter, unsigned want, volatile int* abort_flag,
                                           unsigned* status) {
  const long long t0 = clock64();
  while (ld_acquire(counter) < want) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kSpinLimitCycles) {
      *abort_flag = 1;
      atomicExch(status, 6u /* MTRTQ_ERR_TIMEOUT */);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

// The fp32 sums of tokens 8g .. 8g + 7 from this thread's TMEM lane: the four
// digit sums of each, combined from the smallest digit up.
template <int NT>
__device__ __forceinline__ void tc_load8(uint32_t ta, int g, float (&v8)[8]) {
  uint32_t a[4][8];
#pragma unroll
  for (int d = 0; d < 4; ++d) tmem_ld_32x32b_x8(ta + (uint32_t)(d * NT + g * 8), a[d]);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 8; ++j)
    v8[j] = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn((float)(int)a[3][j], 0x1p-21f),
                                          __fmul_rn((float)(int)a[2][j], 0x1p-14f)),
                                __fmul_rn((float)(int)a[1][j], 0x1p-7f)),
                      (float)(int)a[0][j]);
}

// Epilogue warps (128 threads; thread = channel row = TMEM lane). For each segment,
// eight tokens at a time (the code does not grow with NT): the sums from TMEM,
// then the tile is finished, or, for a tile cut between CTAs, the CTA holding the
// tile's last unit (its finisher) adds the other CTAs' parts, in CTA order, ahead
// of its own; the other CTAs store their part to their slot and count it on the
// tile's counter with one release, without waiting. The accumulator goes back to
// the MMA thread once read. The walk takes each CTA's shared tiles first, so a
// finisher's wait is normally over when it comes to it; CTAs are dispatched in
// index order and all are resident (the grid is at most the CTAs that fit), and a
// finisher only waits for lower-numbered CTAs.
template <int NT>
__device__ __forceinline__ void tc_epilogue(const TcParams& p, uint32_t tmem, uint64_t* accf, uint64_t* acce,
                                            volatile int* s_abort, int64_t ub, int64_t ue, int warp, int lane,
                                            int tid) {
  using C = TcCfg<NT>;
  grid_dependency_wait();  // the scales, Y and the workspace: after the grid ahead
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int etid = tid - (kTcThreads - kTcEpiThreads);
  const int64_t U = p.units, G = p.grid, cta = blockIdx.x;
  TcWalk w;
  w.init(p, ub, ue);
  int seg = 0;
  bool ok = true;
  while (w.rem > 0) {
    const GroupProblem& P = p.prob[w.pi];
    const float* sc = p.scales + w.pi * kTcMaxTokens;
    const int nu = w.seg_units(p);
    const int ab = seg % C::kBufs;
    const int n = w.t * kTileN + row;
    const bool whole = w.ku == 0 && nu == P.KB;
    const bool finisher = !whole && w.ku + nu == P.KB;
    unsigned* counter = p.counters + P.tile_begin + w.t;
    const int64_t T0 = P.unit_begin + (int64_t)w.t * P.KB;  // the tile's first unit
    const int64_t c_lo = tc_cta_of_unit(T0, U, G), c_hi = tc_cta_of_unit(T0 + P.KB - 1, U, G);
    // slot 0 for the segment at the start of the range, 1 for the one at its end
    float* slot = p.partials + ((size_t)(cta * 2 + (w.u == ub ? 0 : 1)) * NT) * kTileN;
    // The lowest CTA's part of a cut tile is its last segment unless the tile
    // starts its range; every later CTA's part is its first segment.
    const int first_slot = tc_range_start(c_lo, U, G) == T0 ? 0 : 1;
    // A finisher adds the other CTAs' parts first: every token's load of one CTA's
    // part in flight at once, the CTAs in order.
    float s[NT];
#pragma unroll
    for (int m = 0; m < NT; ++m) s[m] = 0.0f;
    if (finisher) {
      if (etid == 0) tc_wait_parts(counter, (unsigned)(c_hi - c_lo), s_abort, p.status);
      named_bar_sync(1, kTcEpiThreads);  // the parts are visible to every thread (acquired above)
      for (int64_t cc = c_lo; cc < c_hi; ++cc) {
        const float* part = p.partials + ((size_t)(cc * 2 + (cc == c_lo ? first_slot : 0)) * NT) * kTileN + row;
        float t[NT];
#pragma unroll
        for (int m = 0; m < NT; ++m) t[m] = m < P.M ? __ldcg(part + m * kTileN) : 0.0f;
#pragma unroll
        for (int m = 0; m < NT; ++m) s[m] += t[m];
      }
    }
    ok = ok && mbar_wait_bounded(&accf[ab], (uint32_t)(seg / C::kBufs) & 1u, s_abort, p.status);
    tc_fence_after();
    const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(ab * C::kAccCols);
    const int groups = (P.M + 7) >> 3;
#pragma unroll
    for (int g = 0; g < NT / 8; ++g) {
      if (g >= groups) break;
      float v8[8];
      if (ok) {
        tc_load8<NT>(ta, g, v8);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v8[j] = 0.0f;
      }
      if (!whole && !finisher) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (g * 8 + j < P.M) __stcg(slot + (g * 8 + j) * kTileN + row, v8[j]);
        continue;
      }
      if (n < P.N) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int m = g * 8 + j;
          if (m < P.M) tc_store(p, P, m, n, tc_finish(P, finisher ? s[m] + v8[j] : v8[j], __ldg(sc + m), m, n));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acce[ab]);  // the accumulator goes back to the MMA thread
    if (!whole && !finisher) {
      named_bar_sync(1, kTcEpiThreads);  // every part of this CTA is stored
      if (etid == 0) red_release_add(counter, 1u);  // releases the parts (cumulative over the barrier)
    } else if (finisher && etid == 0) {
      *counter = 0u;  // left at zero for the next call
    }
    w.advance(p, nu);
    ++seg;
  }
  if (p.xc.world > 1) {
    named_bar_sync(1, kTcEpiThreads);  // every store of this CTA is made
    if (etid == 0) tc_exchange_end(p);
  }
}

template <int NT>
__global__ void __launch_bounds__(kTcThreads, TcCfg<NT>::kCtas) gemv_tc_kernel(const __grid_constant__ TcParams p) {
  using C = TcCfg<NT>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[S], empty[S], accf[C::kBufs], acce[C::kBufs], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  unsigned char* wring = smem;                         // S x 8 KiB of weights
  unsigned char* dring = smem + (size_t)S * kTcUnit;  // S x kDigitBytes of digits
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t U = p.units, G = p.grid, cta = blockIdx.x;
  const int64_t ub = tc_range_start(cta, U, G), ue = tc_range_start(cta + 1, U, G);

  if (tid == 0) {
    grid_launch_dependents();
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < C::kBufs; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], kTcEpiThreads / 32);
    }
    mbar_init(&done, 1);
    s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // Producer, in the walk's order. Weights first: they are never written by a
      // kernel, so the first few stages' weights go out before the wait for the
      // digitize kernel -- a few only, so that the digitize kernel's loads do not
      // queue behind every CTA's whole ring (B200, the decode set: 4 stages 28.4 us,
      // the whole ring 29.1, none 31.0).
      const int64_t n = ue - ub;
      const int64_t pre = n < S ? n : S;
      const int64_t pre_w = pre < kTcEarlyStages ? pre : kTcEarlyStages;
      TcCursor c;
      c.init(p, ub, ue);
      {
        TcCursor c0 = c;
        for (int64_t i = 0; i < pre_w; ++i) {
          mbar_arrive_expect_tx(&full[i], C::kStage);
          bulk_g2s(wring + (size_t)i * kTcUnit, c0.weights(p), kTcUnit, &full[i]);
          c0.step(p);
        }
      }
      grid_dependency_wait();  // the digits of this call are written
      int64_t i = 0;
      for (; i < pre; ++i) {
        if (i >= pre_w) {
          mbar_arrive_expect_tx(&full[i], C::kStage);
          bulk_g2s(wring + (size_t)i * kTcUnit, c.weights(p), kTcUnit, &full[i]);
        }
        bulk_g2s(dring + (size_t)i * C::kDigitBytes, c.digits(p, C::kDigitBytes), C::kDigitBytes, &full[i]);
        c.step(p);
      }
      for (; i < n; ++i) {
        const int st = (int)(i % S);
        if (!mbar_wait_bounded(&empty[st], ((uint32_t)(i / S) & 1u) ^ 1u, &s_abort, p.status)) break;
        mbar_arrive_expect_tx(&full[st], C::kStage);
        bulk_g2s(wring + (size_t)st * kTcUnit, c.weights(p), kTcUnit, &full[st]);
        bulk_g2s(dring + (size_t)st * C::kDigitBytes, c.digits(p, C::kDigitBytes), C::kDigitBytes, &full[st]);
        c.step(p);
      }
      // Every copy issued lands before the CTA leaves (the last S at most are
      // outstanding; earlier ones were waited for through their stage's reuse).
      volatile int no_abort = 0;
      for (int64_t j = i - 1; j >= 0 && j >= i - (int64_t)S; --j)
        mbar_wait_bounded(&full[j % S], (uint32_t)(j / S) & 1u, &no_abort, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.
      constexpr uint32_t idesc = umma_idesc_s8(kTileN, C::kRows);
      constexpr uint32_t b_lbo = C::kRows * 16;  // the two 16-k halves of one K = 32 step
      TcWalk w;
      w.init(p, ub, ue);
      int64_t i = 0;
      int seg = 0;
      bool ok = true;
      while (ok && w.rem > 0) {
        const int nu = w.seg_units(p);
        const int ab = seg % C::kBufs;
        if (seg >= C::kBufs)
          ok = mbar_wait_bounded(&acce[ab], (uint32_t)(seg / C::kBufs - 1) & 1u, &s_abort, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * C::kAccCols);
        for (int q = 0; q < nu; ++q, ++i) {
          const int st = (int)(i % S);
          if (!mbar_wait_bounded(&full[st], (uint32_t)(i / S) & 1u, &s_abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wa = smem_u32(wring + (size_t)st * kTcUnit);
          const uint32_t da = smem_u32(dring + (size_t)st * C::kDigitBytes);
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)  // the segment's first MMA overwrites the buffer
            umma_i8_ss(d, umma_desc_interleave(wa + kk * 2 * 2048, 2048, 128),
                       umma_desc_interleave(da + kk * 2 * b_lbo, b_lbo, 128), idesc, (q > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[st]);  // the stage goes back once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&accf[ab]);  // the segment's sums are complete
        w.advance(p, nu);
        ++seg;
      }
      // Every MMA this thread issued completes before the tensor memory is freed.
      umma_commit(&done);
      volatile int no_abort = 0;
      mbar_wait_bounded(&done, 0u, &no_abort, p.status);
    }
  } else {
    tc_epilogue<NT>(p, tmem, accf, acce, &s_abort, ub, ue, warp, lane, tid);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int NT>
cudaError_t tc_launch(const TcParams& tp, int x_dtype, bool round_x, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;

  cudaLaunchConfig_t dc = {};
  dc.gridDim = dim3((unsigned)NT, (unsigned)tp.count, 1);
  dc.blockDim = dim3(kDigitizeThreads, 1, 1);
  dc.stream = st;
  dc.attrs = attr;
  dc.numAttrs = pdl ? 1 : 0;
  void (*dk)(TcParams);
  if (x_dtype == 1)
    dk = digitize_kernel<true, false, false>;
  else if (tp.ln_gamma)
    dk = round_x ? digitize_kernel<false, true, true> : digitize_kernel<false, false, true>;
  else
    dk = round_x ? digitize_kernel<false, true, false> : digitize_kernel<false, false, false>;
  cudaError_t e = ensure_max_carveout(reinterpret_cast<const void*>(dk));
  if (e != cudaSuccess) return e;
  if ((e = cudaLaunchKernelEx(&dc, dk, tp)) != cudaSuccess) return e;

  auto kern = gemv_tc_kernel<NT>;
  if ((e = ensure_smem_limit(reinterpret_cast<const void*>(kern), (int)TcCfg<NT>::kSmem))) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tp.grid, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = TcCfg<NT>::kSmem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, tp);
}

}  // namespace

cudaError_t launch_gemv_tc(const GroupProblem* probs, int count, int64_t units, int grid, int nt, int x_dtype,
                           bool round_x, void* workspace, unsigned* status, bool pdl, cudaStream_t st,
                           const float* ln_gamma, const float* ln_beta, float ln_eps, const TcExchange* xc) {
  if (ln_gamma && (count != 1 || x_dtype != 0)) return cudaErrorInvalidValue;
  TcParams tp;
  tp.xc = xc ? *xc : TcExchange();
  tp.ln_gamma = ln_gamma;
  tp.ln_beta = ln_beta;
  tp.ln_eps = ln_eps;
  const TcLayout lay = gemv_tc_layout(probs, count, grid, nt);
  char* ws = static_cast<char*>(workspace);
  size_t doff = lay.off_digits;
  for (int i = 0; i < count; ++i) {
    tp.prob[i] = probs[i];
    tp.digits[i] = reinterpret_cast<int8_t*>(ws + doff);
    doff += (size_t)probs[i].KB * 256 * nt;
  }
  for (int i = count; i < kGroupMax; ++i) tp.digits[i] = nullptr;
  tp.scales = reinterpret_cast<float*>(ws + lay.off_scales);
  tp.count = count;
  tp.nt = nt;
  tp.units = units;
  tp.grid = grid;
  tp.counters = reinterpret_cast<unsigned*>(ws);
  tp.partials = reinterpret_cast<float*>(ws + lay.off_partials);
  tp.status = status;
  switch (nt) {
    case 8: return tc_launch<8>(tp, x_dtype, round_x, pdl, st);
    case 16: return tc_launch<16>(tp, x_dtype, round_x, pdl, st);
    case 32: return tc_launch<32>(tp, x_dtype, round_x, pdl, st);
    case 64: return tc_launch<64>(tp, x_dtype, round_x, pdl, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mtrtq
