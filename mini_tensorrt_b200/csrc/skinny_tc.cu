// Stream-K tensor-core kernel for skinny INT8 weight-only MatMuls: M <= 32 token
// rows (decode GEMV and small prefill), MTRTQ_MODE_BF16.
//
// Replaces, for these shapes, the reference's scalar MatMulQ loop
// (src/ops/kernels_matmul.cpp:66-73) and the decode loop's fp32 GEMV
// (tools/run_gpt2.cpp:125-132, :189).
//
// Why stream-K: a skinny MatMul is a stream over the int8 weights (K*N bytes),
// and the work is the same per 64-k block of a 128-channel tile (a "unit": 8 KiB
// of packed weights, contiguous in memory because the packed layout is
// [tile][slab]). The grid is one persistent CTA per SM; CTA c takes the units
// [c*U/G, (c+1)*U/G), i.e. one contiguous byte range of the weights, so every SM
// streams the same amount with no tail wave. A tile cut by a CTA boundary gets
// one fp32 partial per CTA that touches it; the last of those CTAs to finish (an
// atomic ticket per tile) sums them in CTA order -- deterministic -- and writes Y.
//
// Units travel in batches of four (units 4b..4b+3 of a CTA: 32 KiB contiguous in
// memory): one bulk copy, one mbarrier round and one commit per batch. Measured on
// B200, a single thread issues a small (N <= 64) tcgen05.mma only every ~50-80
// cycles, and a barrier wait with its tcgen05.fence costs ~400 cycles and a commit
// ~100, so the single-thread roles' bookkeeping, not bandwidth, bounds a skinny
// kernel; batching amortizes it over four units.
//
// Activations: with X_RES the whole [TM x K] activation matrix is rounded to bf16
// once per CTA into shared memory (128-byte-swizzled K-major tiles, one per 64-k
// block) by the twelve worker warps before their main loops; otherwise every unit
// brings its own activation tile by TMA (fp32 rounded to bf16 by the dequantizers,
// or bf16 straight into the swizzled tile).
//
// Warp roles (14 warps):
//   warp 0        producer: per batch, the weight bulk copy (and, without X_RES, the
//                 activation tiles) into a ring of shared-memory stages;
//   warp 1        allocates TMEM; one lane issues tcgen05.mma (kind::f16, A from
//                 TMEM, B = activations from shared memory, four independent
//                 sub-accumulators, one per 16-k step) and tcgen05.commit;
//   warps 2..5    dequantizer group 0 (even units), warps 6..9 group 1 (odd units):
//                 each thread owns one channel row, converts its 64 int8 weights
//                 exactly to bf16 and stores them into a TMEM A stage (tcgen05.st);
//   warps 10..13  the epilogue: tcgen05.ld of a
//                 finished accumulator (double-buffered in TMEM, so the next
//                 segment's MMAs proceed meanwhile), scale and bias into Y, or an
//                 fp32 partial plus the ticketed reduction.
// Every wait is bounded (~1 s); on timeout the kernel records MTRTQ_ERR_TIMEOUT in
// the device status word, drains its copies and MMAs, frees TMEM and returns.
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

struct SkinnyParams {
  const uint8_t* W;       // packed weights; unit u = (tile, k-block) lives at u * 8 KiB
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  Epilogue epi;
  const void* X;          // activations (X_RES staging), row stride ldx elements
  int64_t ldx;
  int x_bf16;             // X element type for X_RES staging
  int M, N, K, n_pad;
  int KB;                 // 64-k blocks per tile
  int n_tiles;
  long long units;        // n_tiles * KB
  int grid;               // CTAs (G)
  float* partials;        // [G][2][M][128]
  unsigned* counters;     // [n_tiles]
  unsigned* status;
};

constexpr int kSkinnyThreads = 14 * 32;
constexpr int kSkinnyBatch = 4;               // units per producer/MMA round (P)
constexpr int kSkinnyAStages = 2 * kSkinnyBatch;  // TMEM A stages: two batches in flight
constexpr int kSkinnyXResBytes = 96 * 1024;   // largest resident activation matrix

template <int TM, bool X_F32, bool X_RES>
struct SkinnyCfg {
  static constexpr int XB_BYTES = TM * 128;                           // bf16 B tile (SW128)
  static constexpr int W_BYTES = kTileN * kBlockK;                    // 8 KiB
  static constexpr int XR_BYTES = (!X_RES && X_F32) ? TM * kBlockK * 4 : 0;  // raw fp32 tile
  static constexpr int STAGE = W_BYTES + (X_RES ? 0 : XB_BYTES + XR_BYTES);
  static constexpr int X_REGION = X_RES ? kSkinnyXResBytes : 0;
  static constexpr int STAGES_RAW = (200 * 1024 - X_REGION) / STAGE;
  static constexpr int STAGES = (STAGES_RAW > 16 ? 16 : STAGES_RAW) / kSkinnyBatch * kSkinnyBatch;
  static constexpr int SB = STAGES / kSkinnyBatch;                     // batch slots
  // Per stage: [W 8 KiB][bf16 B tile][raw fp32 tile]; with X_RES a stage is just
  // the 8 KiB of weights, so the four stages of a batch take one 32 KiB copy.
  static constexpr int OFF_RING = X_REGION;
  static constexpr int OFF_W = 0;
  static constexpr int OFF_XB = W_BYTES;
  static constexpr int OFF_XR = W_BYTES + XB_BYTES;
  static constexpr int OFF_BAR = OFF_RING + STAGES * STAGE;
  static constexpr int NUM_BARS = 2 * SB + 2 + 2 + 2 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 64 + 1024;
  // Independent accumulation chains: the k-th MMA (k = 0..3) of every unit of a
  // segment accumulates into sub-accumulator k, so the four MMAs of a unit do not
  // wait on one another in the tensor pipe; the epilogue sums the four
  // sub-accumulators in a fixed order.
  static constexpr int R = kBlockK / 16;
  static constexpr int ACC_COL = kSkinnyAStages * 32;
  static constexpr int ACC_BUF = R * TM;                     // columns per buffer
  static constexpr int NEED_COLS = ACC_COL + 2 * ACC_BUF;
  static constexpr int TMEM_COLS = NEED_COLS <= 256 ? 256 : 512;
  static_assert(STAGE % 1024 == 0 && X_REGION % 1024 == 0, "1024-byte aligned tiles");
  static_assert(SB >= 2, "the ring must hold two batches");
  static_assert(TM % 16 == 0 && TM >= 16 && TM <= 32, "TM in {16, 32}");
  static_assert(NEED_COLS <= 512, "TMEM has 512 columns");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ bool sk_warp_wait(uint64_t* bar, uint32_t parity, volatile int* ab,
                                             unsigned* status) {
  const bool ok = mbar_wait_bounded(bar, parity, ab, status);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void sk_drain(uint64_t* bar, uint32_t parity, unsigned* status) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) {
      atomicExch(status, 6u);
      return;
    }
  }
}

// CTA that owns unit u: r(c) = floor(c*U/G) <= u < r(c+1).
__device__ __forceinline__ int sk_owner(long long u, long long U, int G) {
  return (int)(((u + 1) * (long long)G - 1) / U);
}

// 8 consecutive activations of row m starting at k (zero past K or M), rounded
// to bf16 (round to nearest even) and packed as 4 bf16x2 words.
__device__ __forceinline__ uint4 sk_load_x8(const SkinnyParams& p, int m, int k) {
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float x = 0.0f;
    if (m < p.M && k + j < p.K) {
      if (p.x_bf16)
        x = __bfloat162float(static_cast<const __nv_bfloat16*>(p.X)[(int64_t)m * p.ldx + k + j]);
      else
        x = static_cast<const float*>(p.X)[(int64_t)m * p.ldx + k + j];
    }
    v[j] = x;
  }
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]);
  __nv_bfloat162 h3 = __floats2bfloat162_rn(v[6], v[7]);
  uint4 r;
  r.x = *reinterpret_cast<uint32_t*>(&h0);
  r.y = *reinterpret_cast<uint32_t*>(&h1);
  r.z = *reinterpret_cast<uint32_t*>(&h2);
  r.w = *reinterpret_cast<uint32_t*>(&h3);
  return r;
}

template <int TM, bool X_F32, bool X_RES>
__global__ void __launch_bounds__(kSkinnyThreads, 1)
    skinny_q8_tc_kernel(const __grid_constant__ CUtensorMap xmap, const SkinnyParams p) {
  using C = SkinnyCfg<TM, X_F32, X_RES>;
  constexpr int S = C::STAGES;
  constexpr int SB = C::SB;
  constexpr int SA = kSkinnyAStages;
  constexpr int P = kSkinnyBatch;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem + C::OFF_RING;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  //   full[b % SB]     batch b's copies landed (producer tx)
  //   done[b % SB]     batch b's MMAs completed (one commit): frees its units'
  //                    shared-memory stages (the dequantizers finished reading them
  //                    before signalling a_full) and their TMEM A stages
  //   a_full[b % 2]    batch b's A operands written (4 arrivals per unit)
  //   x_ready          resident activations staged (12 worker warps)
  uint64_t* full = bars;                   // [SB]
  uint64_t* done = bars + SB;              // [SB]
  uint64_t* a_full = bars + 2 * SB;        // [2]
  uint64_t* acc_full = a_full + 2;         // [2] 1 commit
  uint64_t* acc_empty = acc_full + 2;      // [2] 4 epilogue warps
  uint64_t* x_ready = acc_empty + 2;       // [1]
  uint64_t* drain = x_ready + 1;           // [1] abort drain, 1 commit
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  volatile unsigned* s_ticket = reinterpret_cast<volatile unsigned*>(smem + C::OFF_MISC + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int c = blockIdx.x;
  const long long U = p.units;
  const int G = p.grid;
  const long long u0 = (long long)c * U / G;
  const long long u1 = (long long)(c + 1) * U / G;
  const int n_units = (int)(u1 - u0);
  const int n_batches = (n_units + P - 1) / P;

  if (tid == 0) {
    for (int s = 0; s < SB; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&done[s], 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(&a_full[s], 4 * P);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(x_ready, 12);
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (!X_RES && warp == 0 && lane == 0) prefetch_tensormap(&xmap);
  if (warp == 1) {
    tmem_alloc(s_tmem, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  // X_RES: the 12 worker warps (w = 0..11) round the whole [TM x K_pad] activation
  // matrix to bf16 into one swizzled K-major tile per 64-k block (chunk (kb, row, ch)
  // holds k = kb*64 + ch*8 .. +7), four chunks' loads in flight per thread.
  auto stage_x = [&](int w) {
    const int et = w * 32 + lane;                 // 0..383
    const int chunks = p.KB * TM * 8;
    for (int c0 = et; c0 < chunks; c0 += 4 * 384) {
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cidx = c0 + j * 384;
        const int ch = cidx & 7, row = (cidx >> 3) % TM, kb = cidx / (8 * TM);
        v[j] = cidx < chunks ? sk_load_x8(p, row, kb * kBlockK + ch * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cidx = c0 + j * 384;
        if (cidx < chunks) {
          const int ch = cidx & 7, row = (cidx >> 3) % TM, kb = cidx / (8 * TM);
          *reinterpret_cast<uint4*>(smem + kb * C::XB_BYTES + row * 128 + ((ch ^ (row & 7)) << 4)) =
              v[j];
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(x_ready);
  };

  if (warp == 0) {
    // ---------------- producer: one round per batch ----------------
    if (lane == 0) {
      int issued = 0;  // batches
      int kb = (int)(u0 % p.KB);
      for (int b = 0; b < n_batches; ++b) {
        const int sb = b % SB;
        if (!mbar_wait_bounded(&done[sb], ((b / SB) & 1) ^ 1, s_abort, p.status)) break;
        const int i0 = P * b;
        const int nu = min(P, n_units - i0);
        uint8_t* st = ring + (i0 % S) * C::STAGE;
        const uint32_t x_bytes = X_RES ? 0u : (uint32_t)(X_F32 ? C::XR_BYTES : C::XB_BYTES);
        mbar_arrive_expect_tx(&full[sb], (uint32_t)nu * (C::W_BYTES + x_bytes));
        if (X_RES) {
          // The batch's weights are adjacent in memory and in the ring.
          bulk_g2s(st + C::OFF_W, p.W + (u0 + i0) * (long long)C::W_BYTES,
                   (uint32_t)nu * C::W_BYTES, &full[sb]);
        } else {
          for (int j = 0; j < nu; ++j) {
            uint8_t* sj = st + j * C::STAGE;
            bulk_g2s(sj + C::OFF_W, p.W + (u0 + i0 + j) * (long long)C::W_BYTES, C::W_BYTES,
                     &full[sb]);
            tma_load_2d(sj + (X_F32 ? C::OFF_XR : C::OFF_XB), &xmap, kb * kBlockK, 0, &full[sb]);
            if (++kb == p.KB) kb = 0;
          }
        }
        ++issued;
      }
      for (int j = max(0, issued - SB); j < issued; ++j)
        sk_drain(&full[j % SB], (j / SB) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: one round per batch ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kTileN, TM);
      int seg = -1;
      bool ok = true;
      int kb = (int)(u0 % p.KB);
      if (X_RES && !mbar_wait_bounded(x_ready, 0, s_abort, p.status)) ok = false;
      for (int b = 0; b < n_batches && ok; ++b) {
        if (!mbar_wait_bounded(&a_full[b & 1], (b >> 1) & 1, s_abort, p.status)) { ok = false; break; }
        // bf16 activation tiles arrive by TMA straight into the B tile: observe
        // those copies. (fp32 tiles are written by the dequantizers before a_full.)
        if (!X_RES && !X_F32 &&
            !mbar_wait_bounded(&full[b % SB], (b / SB) & 1, s_abort, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int i_end = min(P * b + P, n_units);
        for (int i = P * b; i < i_end; ++i, kb = (kb + 1 == p.KB) ? 0 : kb + 1) {
          const bool first = (i == 0) || kb == 0;
          const bool last = (i == n_units - 1) || kb == p.KB - 1;
          if (first) {
            ++seg;
            if (!mbar_wait_bounded(&acc_empty[seg & 1], ((seg >> 1) & 1) ^ 1, s_abort, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const uint32_t acc = tmem_base + C::ACC_COL + (seg & 1) * C::ACC_BUF;
          const uint32_t xaddr =
              X_RES ? smem_u32(smem + kb * C::XB_BYTES)
                    : smem_u32(ring + (i % S) * C::STAGE + C::OFF_XB);
          const uint32_t a_tm = tmem_base + (i % SA) * 32;
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k)
            umma_ts(acc + k * TM, a_tm + k * 8, umma_desc_sw128(xaddr + k * 32), idesc,
                    first ? 0u : 1u);
          if (last) umma_commit(&acc_full[seg & 1]);
        }
        if (!ok) break;
        umma_commit(&done[b % SB]);
      }
      if (!ok) {
        // Let every MMA already issued finish before TMEM is freed.
        umma_commit(drain);
        sk_drain(drain, 0, p.status);
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---------------- dequantizers (group g handles units i = g, g+2, ...) ----------------
    const int group = (warp - 2) >> 2;     // 0: warps 2..5, 1: warps 6..9
    const int q4 = warp & 3;               // TMEM lane quadrant
    const int r = q4 * 32 + lane;          // channel row in the tile
    const int gt = (warp - 2 - 4 * group) * 32 + lane;  // 0..127 within the group
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    if (X_RES) stage_x(warp - 2);
    for (int i = group; i < n_units; i += 2) {
      const int s = i % S, sa = i % SA, b = i / P;
      if (!sk_warp_wait(&full[b % SB], (b / SB) & 1, s_abort, p.status)) break;
      uint8_t* st = ring + s * C::STAGE;
      uint4 wv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wv[j] = *reinterpret_cast<const uint4*>(st + C::OFF_W + j * kSlabBytes + r * 16);
      if (!X_RES && X_F32) {
        // Round the fp32 activation tile [TM][64] to bf16 into the swizzled B tile.
        const float* xr = reinterpret_cast<const float*>(st + C::OFF_XR);
        uint8_t* xb = st + C::OFF_XB;
#pragma unroll
        for (int cidx = gt; cidx < TM * 8; cidx += 128) {
          const int row = cidx >> 3, ch = cidx & 7;
          const float4 a = *reinterpret_cast<const float4*>(xr + row * 64 + ch * 8);
          const float4 b = *reinterpret_cast<const float4*>(xr + row * 64 + ch * 8 + 4);
          __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y);
          __nv_bfloat162 h1 = __floats2bfloat162_rn(a.z, a.w);
          __nv_bfloat162 h2 = __floats2bfloat162_rn(b.x, b.y);
          __nv_bfloat162 h3 = __floats2bfloat162_rn(b.z, b.w);
          uint4 v;
          v.x = *reinterpret_cast<uint32_t*>(&h0);
          v.y = *reinterpret_cast<uint32_t*>(&h1);
          v.z = *reinterpret_cast<uint32_t*>(&h2);
          v.w = *reinterpret_cast<uint32_t*>(&h3);
          *reinterpret_cast<uint4*>(xb + row * 128 + ((ch ^ (row & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
      }
      uint32_t a[32];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        i8x4_to_bf16x4(wv[j].x, a[8 * j + 0], a[8 * j + 1]);
        i8x4_to_bf16x4(wv[j].y, a[8 * j + 2], a[8 * j + 3]);
        i8x4_to_bf16x4(wv[j].z, a[8 * j + 4], a[8 * j + 5]);
        i8x4_to_bf16x4(wv[j].w, a[8 * j + 6], a[8 * j + 7]);
      }
      // A stage sa was last used by unit i - SA (batch b - 2): free once that batch is done.
      if (b >= 2 && !sk_warp_wait(&done[(b - 2) % SB], ((b - 2) / SB) & 1, s_abort, p.status)) break;
      tmem_st_32x32b_x32(tmem_base + lane_off + sa * 32, a);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      // Four arrivals per unit; the CTA's last unit also stands in for the units its
      // (short) final batch lacks, so every batch completes a_full with 4*P.
      if (lane == 0)
        mbar_arrive_cnt(&a_full[b & 1], i == n_units - 1 ? 1u + (uint32_t)(P * (b + 1) - n_units) : 1u);
    }
  } else {
    // ---------------- (X_RES: activation staging, then) epilogue ----------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    if (X_RES) stage_x(warp - 2);
    int seg = -1;
    long long u = u0;
    while (u < u1) {
      const int t = (int)(u / p.KB);
      const long long seg_end = min(u1, (long long)(t + 1) * p.KB);
      const bool full_tile = (u == (long long)t * p.KB) && (seg_end == (long long)(t + 1) * p.KB);
      ++seg;
      const int b = seg & 1;
      float v[TM];
      const bool ok = sk_warp_wait(&acc_full[b], (seg >> 1) & 1, s_abort, p.status);
      if (ok) {
        tc_fence_after();
        // The four sub-accumulators, summed 0, 1, 2, 3.
#pragma unroll
        for (int j = 0; j < TM; ++j) v[j] = 0.0f;
#pragma unroll
        for (int sub = 0; sub < C::R; ++sub) {
#pragma unroll
          for (int c0 = 0; c0 < TM; c0 += 16) {
            uint32_t raw[16];
            tmem_ld_32x32b_x16(tmem_base + lane_off + C::ACC_COL + b * C::ACC_BUF + sub * TM + c0,
                               raw);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[c0 + j] += __uint_as_float(raw[j]);
          }
        }
        tc_fence_before();
      } else {
#pragma unroll
        for (int j = 0; j < TM; ++j) v[j] = 0.0f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);

      const int n = t * kTileN + r;
      const bool n_ok = n < p.N;
      const float sc = n_ok ? p.scale[n] : 0.0f;
      const float bi = (n_ok && p.bias) ? p.bias[n] : 0.0f;
      if (full_tile) {
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < TM; ++j) {
            if (j < p.M) {
              float y = __fmul_rn(v[j], sc);
              if (p.bias) y = __fadd_rn(y, bi);
              p.Y[(int64_t)j * p.ldy + n] = epi_apply(p.epi, y, j, n);
            }
          }
        }
      } else {
        // Partial of tile t: this CTA's slot 0 if t is its first tile, else slot 1.
        const int t_first = (int)(u0 / p.KB);
        const int slot = (t == t_first) ? 0 : 1;
        float* part = p.partials + ((int64_t)(c * 2 + slot) * p.M) * kTileN + r;
#pragma unroll
        for (int j = 0; j < TM; ++j)
          if (j < p.M) __stcg(part + (int64_t)j * kTileN, v[j]);
        named_bar_sync(1, 128);
        const int c_first = sk_owner((long long)t * p.KB, U, G);
        const int c_last = sk_owner((long long)(t + 1) * p.KB - 1, U, G);
        const unsigned nslots = (unsigned)(c_last - c_first + 1);
        unsigned* counter = p.counters + t;
        if (warp == 10 && lane == 0) *s_ticket = ticket_acq_rel(counter);
        named_bar_sync(1, 128);
        if (*s_ticket == nslots - 1) {
          if (n_ok) {
            // Slots are summed in CTA order (= k order), 16 rows at a time; the
            // loads of four slots are issued together.
            constexpr int SL = 4;
            for (int j0 = 0; j0 < TM && j0 < p.M; j0 += 16) {
              float sum[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) sum[j] = 0.0f;
              for (int cc0 = c_first; cc0 <= c_last; cc0 += SL) {
                float v2[SL][16];
#pragma unroll
                for (int k = 0; k < SL; ++k) {
                  const int cc = min(cc0 + k, c_last);
                  const int sl = ((int)((long long)cc * U / G / p.KB) == t) ? 0 : 1;
                  const float* src =
                      p.partials + ((int64_t)(cc * 2 + sl) * p.M + j0) * kTileN + r;
#pragma unroll
                  for (int j = 0; j < 16; ++j)
                    v2[k][j] = (j0 + j < p.M) ? __ldcg(src + (int64_t)j * kTileN) : 0.0f;
                }
#pragma unroll
                for (int k = 0; k < SL; ++k)
                  if (cc0 + k <= c_last) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) sum[j] += v2[k][j];
                  }
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (j0 + j < p.M) {
                  float y = __fmul_rn(sum[j], sc);
                  if (p.bias) y = __fadd_rn(y, bi);
                  p.Y[(int64_t)(j0 + j) * p.ldy + n] = epi_apply(p.epi, y, j0 + j, n);
                }
              }
            }
          }
          if (warp == 10 && lane == 0) *counter = 0u;
        }
      }
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int TM, bool X_F32, bool X_RES>
static cudaError_t sk_launch(const SkinnyParams& sp, const CUtensorMap& xmap, cudaStream_t st) {
  using C = SkinnyCfg<TM, X_F32, X_RES>;
  if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(skinny_q8_tc_kernel<TM, X_F32, X_RES>),
                                         C::SMEM_BYTES))
    return e;
  skinny_q8_tc_kernel<TM, X_F32, X_RES><<<sp.grid, kSkinnyThreads, C::SMEM_BYTES, st>>>(xmap, sp);
  return cudaGetLastError();
}

bool skinny_x_resident(int tile_m, int64_t k_pad) {
  return k_pad * tile_m * 2 <= kSkinnyXResBytes;
}

cudaError_t launch_skinny_tc(const Plan& p, const float* scale, const float* bias, float* Y,
                             int64_t ldy, const void* packed, void* workspace,
                             const CUtensorMap& xmap, bool x_f32, const void* X, int64_t ldx,
                             int x_dtype, unsigned* status, const Epilogue& epi, cudaStream_t st) {
  SkinnyParams sp;
  sp.epi = epi;
  sp.W = static_cast<const uint8_t*>(packed);
  sp.scale = scale;
  sp.bias = bias;
  sp.Y = Y;
  sp.ldy = ldy;
  sp.X = X;
  sp.ldx = ldx;
  sp.x_bf16 = x_dtype == 1 ? 1 : 0;
  sp.M = (int)p.M;
  sp.N = (int)p.N;
  sp.K = (int)p.K;
  sp.n_pad = (int)p.n_pad;
  sp.KB = p.kunits;
  sp.n_tiles = p.n_tiles;
  sp.units = (long long)p.n_tiles * p.kunits;
  sp.grid = p.grid;
  char* ws = static_cast<char*>(workspace);
  sp.counters = reinterpret_cast<unsigned*>(ws + p.off_counters);
  sp.partials = reinterpret_cast<float*>(ws + p.off_partials);
  sp.status = status;
  const bool res = skinny_x_resident(p.tile_m, p.k_pad);
  switch (p.tile_m) {
    case 16:
      if (res) return sk_launch<16, true, true>(sp, xmap, st);
      return x_f32 ? sk_launch<16, true, false>(sp, xmap, st) : sk_launch<16, false, false>(sp, xmap, st);
    case 32:
      if (res) return sk_launch<32, true, true>(sp, xmap, st);
      return x_f32 ? sk_launch<32, true, false>(sp, xmap, st) : sk_launch<32, false, false>(sp, xmap, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace mtrtq
