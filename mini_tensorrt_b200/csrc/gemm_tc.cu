// Prefill GEMM for the INT8 weight-only MatMul on 5th-generation tensor cores.
//
// Replaces, for M > 8 token rows, the reference's scalar MatMulQ loop
// (src/ops/kernels_matmul.cpp:66-73). Swap-AB orientation: the MMA's M side is
// 128 output channels (one channel tile of the packed weights), its N side is a
// tile of TM tokens, K advances 64 at a time, so the per-channel scale and bias
// are per-TMEM-lane constants in the epilogue and Y stores are coalesced along
// channels.
//
// One CTA = 6 warps, warp-specialised, one output tile of 128 channels x TM
// tokens over a k range:
//   warp 0      producer: per stage one TMA tensor copy of the bf16 activation
//               tile (128-byte swizzle) and one 8 KiB bulk copy of the int8 weight
//               tile, both completing on the stage's `full` mbarrier;
//   warp 1      allocates TMEM; one lane issues tcgen05.mma (kind::f16, fp32
//               accumulators in TMEM) and tcgen05.commit to release stages;
//   warps 2..5  dequantize: each thread owns one channel row, reads its 64 int8
//               weights of the stage from shared memory, converts them exactly to
//               bf16 and writes them as the MMA's A operand -- into TMEM with
//               tcgen05.st (A_TMEM) or into a 128-byte-swizzled shared tile;
//               afterwards the same warps run the epilogue (tcgen05.ld, scale,
//               bias, store or split-K partial).
// Every mbarrier wait is bounded (~1 s); on timeout the kernel records
// MTRTQ_ERR_TIMEOUT in the device status word, drains its own copies and MMAs,
// frees TMEM and returns.
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

struct GemmParams {
  const uint8_t* W;       // packed weights
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  Epilogue epi;
  int M, N, n_pad;
  int KB;                 // k blocks of 64 in K_pad
  int kb_per_split;
  int splits;
  int n_tiles, m_tiles;
  float* partials;        // [splits][M][n_pad]
  unsigned* counters;     // [m_tiles][n_tiles]
  unsigned* status;       // device status word (MTRTQ_ERR_TIMEOUT on a failed wait)
};

template <int TM, bool A_TMEM, int STAGES>
struct GemmCfg {
  static constexpr int X_STAGE = TM * 128;                  // TM rows x 64 bf16
  static constexpr int W_STAGE = kTileN * kBlockK;          // 8192 int8
  static constexpr int A_STAGE = A_TMEM ? 0 : kTileN * 128; // 128 rows x 64 bf16
  static constexpr int OFF_X = 0;
  static constexpr int OFF_A = OFF_X + STAGES * X_STAGE;
  static constexpr int OFF_W = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_BAR = OFF_W + STAGES * W_STAGE;
  static constexpr int NUM_BARS = 4 * STAGES + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 32 + 1024;   // + alignment slack
  static constexpr int TMEM_A_COLS = A_TMEM ? STAGES * 32 : 0;
  static constexpr int ACC_COL = TMEM_A_COLS;
  static constexpr int NEED_COLS = TMEM_A_COLS + TM;
  static constexpr int TMEM_COLS = NEED_COLS <= 32 ? 32 : NEED_COLS <= 64 ? 64
                                 : NEED_COLS <= 128 ? 128 : NEED_COLS <= 256 ? 256 : 512;
  static_assert(TM % 16 == 0 && TM >= 16 && TM <= 256, "MMA N must be 16..256, multiple of 16");
  static_assert(X_STAGE % 1024 == 0, "swizzle atoms need 1024-byte aligned stages");
  static_assert(NEED_COLS <= 512, "TMEM has 512 columns");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// Bounded wait by every lane of a warp; the result is warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned* status) {
  const bool ok = mbar_wait_bounded(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait that ignores the abort flag (used to drain in-flight work).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, unsigned* status) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kSpinLimitCycles) {
      atomicExch(status, 6u);
      return;
    }
  }
}

template <int TM, bool A_TMEM, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
  using C = GemmCfg<TM, A_TMEM, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;                    // TMA landed (X + W), count 1 + tx
  uint64_t* empty = bars + STAGES;          // stage smem free: 4 converter warps + 1 commit
  uint64_t* a_full = bars + 2 * STAGES;     // A operand written: 4 converter warps
  uint64_t* a_empty = bars + 3 * STAGES;    // A operand consumed: 1 commit
  uint64_t* acc_full = bars + 4 * STAGES;   // accumulator final: 1 commit
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  volatile unsigned* s_ticket = reinterpret_cast<volatile unsigned*>(smem + C::OFF_MISC + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int mt = blockIdx.x;
  const int nt = blockIdx.y;
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.KB);
  const int nkb = kb1 - kb0;
  const int m0 = mt * TM;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&xmap);
  if (warp == 1) {
    tmem_alloc(s_tmem, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1, s_abort, p.status)) break;
        mbar_arrive_expect_tx(&full[s], C::X_STAGE + C::W_STAGE);
        const int kb = kb0 + i;
        tma_load_2d(smem + C::OFF_X + s * C::X_STAGE, &xmap, kb * kBlockK, m0, &full[s]);
        bulk_g2s(smem + C::OFF_W + s * C::W_STAGE,
                 p.W + ((int64_t)nt * p.KB + kb) * (int64_t)C::W_STAGE, C::W_STAGE, &full[s]);
        ++issued;
      }
      // No copy may still be in flight when the CTA exits.
      for (int j = max(0, issued - STAGES); j < issued; ++j)
        mbar_drain(&full[j % STAGES], (j / STAGES) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kTileN, TM);
      const uint32_t acc = tmem_base + C::ACC_COL;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait_bounded(&a_full[s], ph, s_abort, p.status)) break;
        if (!mbar_wait_bounded(&full[s], ph, s_abort, p.status)) break;
        tc_fence_after();
        const uint32_t xaddr = smem_u32(smem + C::OFF_X + s * C::X_STAGE);
#pragma unroll
        for (int k = 0; k < kBlockK / 16; ++k) {
          const uint64_t bdesc = umma_desc_sw128(xaddr + k * 32);
          const uint32_t accumulate = (i > 0 || k > 0) ? 1u : 0u;
          if (A_TMEM) {
            umma_ts(acc, tmem_base + s * 32 + k * 8, bdesc, idesc, accumulate);
          } else {
            const uint32_t aaddr = smem_u32(smem + C::OFF_A + s * C::A_STAGE);
            umma_ss(acc, umma_desc_sw128(aaddr + k * 32), bdesc, idesc, accumulate);
          }
        }
        umma_commit(&empty[s]);
        umma_commit(&a_empty[s]);
      }
      umma_commit(acc_full);
      if (*s_abort) mbar_drain(acc_full, 0, p.status);  // MMAs must finish before TMEM is freed
    }
    __syncwarp();
  } else {
    // ---------------- dequantizers, then epilogue ----------------
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;            // channel row within the tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      if (!warp_wait(&full[s], ph, s_abort, p.status)) { ok = false; break; }
      const uint8_t* wst = smem + C::OFF_W + s * C::W_STAGE;
      uint4 wv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wv[j] = *reinterpret_cast<const uint4*>(wst + j * kSlabBytes + r * 16);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      uint32_t a[32];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        i8x4_to_bf16x4(wv[j].x, a[8 * j + 0], a[8 * j + 1]);
        i8x4_to_bf16x4(wv[j].y, a[8 * j + 2], a[8 * j + 3]);
        i8x4_to_bf16x4(wv[j].z, a[8 * j + 4], a[8 * j + 5]);
        i8x4_to_bf16x4(wv[j].w, a[8 * j + 6], a[8 * j + 7]);
      }
      if (!warp_wait(&a_empty[s], ph ^ 1, s_abort, p.status)) { ok = false; break; }
      if (A_TMEM) {
        tmem_st_32x32b_x32(tmem_base + lane_off + s * 32, a);
        tmem_wait_st();
      } else {
        uint8_t* arow = smem + C::OFF_A + s * C::A_STAGE + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) =
              make_uint4(a[4 * c], a[4 * c + 1], a[4 * c + 2], a[4 * c + 3]);
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }

    const int n = nt * kTileN + r;
    const bool n_ok = n < p.N;
    const float sc = n_ok ? p.scale[n] : 0.0f;
    const float b = (n_ok && p.bias) ? p.bias[n] : 0.0f;
    if (ok && warp_wait(acc_full, 0, s_abort, p.status)) {
      tc_fence_after();
      for (int c0 = 0; c0 < TM; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem_base + lane_off + C::ACC_COL + c0, v);
        tmem_wait_ld();
        if (p.splits == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (n_ok && m < p.M) {
              float y = __fmul_rn(__uint_as_float(v[j]), sc);
              if (p.bias) y = __fadd_rn(y, b);
              p.Y[(int64_t)m * p.ldy + n] = epi_apply(p.epi, y, m, n);
            }
          }
        } else {
          float* part = p.partials + ((int64_t)split * p.M) * p.n_pad + n;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m < p.M) __stcg(part + (int64_t)m * p.n_pad, __uint_as_float(v[j]));
          }
        }
      }
    }
    if (p.splits > 1) {
      // Last CTA of this output tile sums the partials in split order. All four
      // epilogue warps reach both named barriers whatever happened above, and the
      // ticket is always taken, so the counter returns to zero even after a
      // timeout (whose output is then flagged by the device status word).
      named_bar_sync(1, 128);
      unsigned* counter = p.counters + (int64_t)mt * p.n_tiles + nt;
      if (warp == 2 && lane == 0) *s_ticket = ticket_acq_rel(counter);
      named_bar_sync(1, 128);
      if (*s_ticket == (unsigned)(p.splits - 1)) {
        if (n_ok) {
          // 8 tokens at a time: their loads (rows clamped to M-1, so always in
          // bounds) for one split are independent and issued together; each output
          // still sums splits 0, 1, 2, ... in order.
          const int64_t split_stride = (int64_t)p.M * p.n_pad;
          const float* base = p.partials + n;
          for (int c0 = 0; c0 < TM && m0 + c0 < p.M; c0 += 8) {
            int64_t off[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) off[j] = (int64_t)min(m0 + c0 + j, p.M - 1) * p.n_pad;
            float sum[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) sum[j] = 0.0f;
            const float* src = base;
#pragma unroll 2
            for (int sp = 0; sp < p.splits; ++sp, src += split_stride) {
#pragma unroll
              for (int j = 0; j < 8; ++j) sum[j] += __ldcg(src + off[j]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int m = m0 + c0 + j;
              if (m < p.M) {
                float y = __fmul_rn(sum[j], sc);
                if (p.bias) y = __fadd_rn(y, b);
                p.Y[(int64_t)m * p.ldy + n] = epi_apply(p.epi, y, m, n);
              }
            }
          }
        }
        if (warp == 2 && lane == 0) *counter = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- persistent variant: one CTA per SM over a static tile schedule ----------------
//
// For grids of at least one tile per SM and one k split. Ten warps: warp 0 the
// producer (as above), warp 1 the MMA issuer, warps 2..5 dequantize each weight tile
// into a 128-byte-swizzled shared memory ring (the A operand), warps 6..9 the
// epilogue. TMEM holds two 256-column fp32 accumulators: the MMAs of a CTA's next
// tile run while the epilogue drains the last one, so the per-tile epilogue (128
// KiB of fp32 Y) and set-up no longer stall the tensor pipe. CTA c takes tiles c,
// c + G, c + 2G, ..., token tiles fastest, so that the CTAs working at the same time
// share channel tiles (weights) and every token tile (X) in L2.
constexpr int kPgThreads = 320;
constexpr int kPgLoadStages = 4;  // X (32 KiB) + W (8 KiB) per stage
constexpr int kPgAStages = 2;     // dequantized A, 16 KiB per stage

struct PgCfg {
  static constexpr int TM = 256;
  static constexpr int X_STAGE = TM * 128;
  static constexpr int W_STAGE = kTileN * kBlockK;
  static constexpr int A_STAGE = kTileN * 128;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_A = OFF_X + kPgLoadStages * X_STAGE;
  static constexpr int OFF_W = OFF_A + kPgAStages * A_STAGE;
  static constexpr int OFF_BAR = OFF_W + kPgLoadStages * W_STAGE;
  static constexpr int NUM_BARS = 2 * kPgLoadStages + 2 * kPgAStages + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 32 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

__global__ void __launch_bounds__(kPgThreads, 1)
    gemm_q8_tc_persistent_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
  using C = PgCfg;
  constexpr int TM = C::TM;
  constexpr int SL = kPgLoadStages, SA = kPgAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;                    // X + W landed: 1 + tx
  uint64_t* empty = bars + SL;              // load stage free: 4 dequantizing warps + 1 commit
  uint64_t* a_full = bars + 2 * SL;         // A written: 4 dequantizing warps
  uint64_t* a_empty = a_full + SA;          // A consumed: 1 commit
  uint64_t* acc_full = a_empty + SA;        // [2] accumulator final: 1 commit
  uint64_t* acc_empty = acc_full + 2;       // [2] accumulator drained: 4 epilogue warps
  uint64_t* done = acc_empty + 2;           // every MMA of this CTA complete
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.m_tiles * p.n_tiles;
  const int KB = p.KB;

  if (tid == 0) {
    for (int s = 0; s < SL; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&xmap);
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      int64_t li = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < T; tile += gridDim.x) {
        const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
        for (int kb = 0; kb < KB; ++kb, ++li) {
          const int s = (int)(li % SL);
          if (li >= SL && !mbar_wait_bounded(&empty[s], ((uint32_t)(li / SL) & 1u) ^ 1u, s_abort, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::X_STAGE + C::W_STAGE);
          tma_load_2d(smem + C::OFF_X + s * C::X_STAGE, &xmap, kb * kBlockK, mt * TM, &full[s]);
          bulk_g2s(smem + C::OFF_W + s * C::W_STAGE, p.W + ((int64_t)nt * KB + kb) * (int64_t)C::W_STAGE,
                   C::W_STAGE, &full[s]);
        }
      }
      for (int64_t j = li - 1; j >= 0 && j >= li - SL; --j) mbar_drain(&full[j % SL], (uint32_t)(j / SL) & 1u, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kTileN, TM);
      int64_t li = 0, ai = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < T; tile += gridDim.x, ++it) {
        const int b = it & 1;
        if (it >= 2 && !mbar_wait_bounded(&acc_empty[b], (uint32_t)((it >> 1) - 1) & 1u, s_abort, p.status)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + (uint32_t)(b * TM);
        for (int kb = 0; kb < KB; ++kb, ++li, ++ai) {
          const int s = (int)(li % SL), sa = (int)(ai % SA);
          if (!mbar_wait_bounded(&a_full[sa], (uint32_t)(ai / SA) & 1u, s_abort, p.status) ||
              !mbar_wait_bounded(&full[s], (uint32_t)(li / SL) & 1u, s_abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(smem + C::OFF_X + s * C::X_STAGE);
          const uint32_t aaddr = smem_u32(smem + C::OFF_A + sa * C::A_STAGE);
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k)
            umma_ss(acc, umma_desc_sw128(aaddr + k * 32), umma_desc_sw128(xaddr + k * 32), idesc,
                    (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&a_empty[sa]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
      umma_commit(done);  // MMAs must finish before TMEM is freed
      mbar_drain(done, 0, p.status);
    }
  } else if (warp < 6) {
    // Dequantize each weight tile: thread = channel row, 64 int8 -> bf16, into a
    // 128-byte-swizzled row of the A stage.
    const int r = (warp - 2) * 32 + lane;
    int64_t li = 0, ai = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < T; tile += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++li, ++ai) {
        const int s = (int)(li % SL), sa = (int)(ai % SA);
        if (!warp_wait(&full[s], (uint32_t)(li / SL) & 1u, s_abort, p.status)) {
          ok = false;
          break;
        }
        const uint8_t* wst = smem + C::OFF_W + s * C::W_STAGE;
        uint4 wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const uint4*>(wst + j * kSlabBytes + r * 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        uint32_t a[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          i8x4_to_bf16x4(wv[j].x, a[8 * j + 0], a[8 * j + 1]);
          i8x4_to_bf16x4(wv[j].y, a[8 * j + 2], a[8 * j + 3]);
          i8x4_to_bf16x4(wv[j].z, a[8 * j + 4], a[8 * j + 5]);
          i8x4_to_bf16x4(wv[j].w, a[8 * j + 6], a[8 * j + 7]);
        }
        if (ai >= SA && !warp_wait(&a_empty[sa], ((uint32_t)(ai / SA) & 1u) ^ 1u, s_abort, p.status)) {
          ok = false;
          break;
        }
        uint8_t* arow = smem + C::OFF_A + sa * C::A_STAGE + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) =
              make_uint4(a[4 * c], a[4 * c + 1], a[4 * c + 2], a[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
    }
  } else {
    // Epilogue: thread = channel row = TMEM lane of its quarter.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    int it = 0;
    for (int tile = blockIdx.x; tile < T; tile += gridDim.x, ++it) {
      const int b = it & 1;
      const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
      const bool ok = warp_wait(&acc_full[b], (uint32_t)(it >> 1) & 1u, s_abort, p.status);
      tc_fence_after();
      const int n = nt * kTileN + r;
      const bool n_ok = n < p.N;
      const float sc = n_ok ? __ldg(p.scale + n) : 0.0f;
      const float bs = (n_ok && p.bias) ? __ldg(p.bias + n) : 0.0f;
      const int m0 = mt * TM;
      if (ok) {
        for (int c0 = 0; c0 < TM && m0 + c0 < p.M; c0 += 16) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(tmem_base + lane_off + (uint32_t)(b * TM + c0), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (n_ok && m < p.M) {
              float y = __fmul_rn(__uint_as_float(v[j]), sc);
              if (p.bias) y = __fadd_rn(y, bs);
              p.Y[(int64_t)m * p.ldy + n] = epi_apply(p.epi, y, m, n);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---- stream-K variant of the persistent kernel ---------------------------------------
//
// The same roles, but CTA c takes the contiguous run [c I / G, (c + 1) I / G) of the
// I = tiles x k-blocks iterations (tile-major, k fastest, token tiles fastest among
// tiles), so every SM gets the same number of MMAs whatever the tile count: no wave
// quantization (4096 x 4096 at M = 2048 is 256 tiles on 148 SMs). A run is a
// sequence of segments (its part of one tile); each segment accumulates in one of the
// two TMEM accumulators. A segment that is a whole tile is finished in place; of a
// tile cut between CTAs, the CTA holding its last k-block (the finisher) waits,
// bounded, for the other CTAs' fp32 parts (each stores its part to its workspace slot
// and counts it on the tile's counter with one release) and adds them in CTA order
// ahead of its own. A CTA takes the last segment of its run first (the tile it shares
// with the next CTA), so parts are ready early; all CTAs are resident (one per SM)
// and a finisher only waits for lower-numbered CTAs.
struct SkWalk {
  int tile, kb;         // the segment's tile and first k-block
  int64_t u, rem;       // its first iteration; iterations left in this part of the run
  int64_t next_b, next_e;
  __device__ __forceinline__ void start(int64_t b, int64_t e, int KB) {
    u = b;
    rem = e - b;
    tile = (int)(b / KB);
    kb = (int)(b - (int64_t)tile * KB);
  }
  __device__ __forceinline__ void init(int64_t ub, int64_t ue, int KB) {
    const int64_t last_tile_start = (ue - 1) / KB * KB;
    const int64_t ls = last_tile_start > ub ? last_tile_start : ub;
    start(ls, ue, KB);
    next_b = ub;
    next_e = ls;
  }
  __device__ __forceinline__ int seg_len(int KB) const {
    const int64_t left = KB - kb;
    return (int)(left < rem ? left : rem);
  }
  __device__ __forceinline__ void advance(int n, int KB) {
    u += n;
    rem -= n;
    kb += n;
    if (rem == 0 && next_b < next_e) {
      start(next_b, next_e, KB);
      next_b = next_e;
      return;
    }
    if (kb == KB) {
      kb = 0;
      ++tile;
    }
  }
};

__device__ __forceinline__ int64_t sk_range_start(int64_t c, int64_t I, int64_t G) { return c * I / G; }
__device__ __forceinline__ int64_t sk_cta_of(int64_t u, int64_t I, int64_t G) { return ((u + 1) * G + I - 1) / I - 1; }

__device__ __forceinline__ void sk_red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned sk_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __noinline__ void sk_wait_parts(const unsigned* counter, unsigned want, volatile int* abort_flag,
                                           unsigned* status) {
  const long long t0 = clock64();
  while (sk_ld_acquire(counter) < want) {
    if (*abort_flag) return;
    if (clock64() - t0 > kSpinLimitCycles) {
      *abort_flag = 1;
      atomicExch(status, 6u /* MTRTQ_ERR_TIMEOUT */);
      return;
    }
    __nanosleep(200);
  }
}

__global__ void __launch_bounds__(kPgThreads, 1)
    gemm_q8_tc_streamk_kernel(const __grid_constant__ CUtensorMap xmap, const GemmParams p) {
  using C = PgCfg;
  constexpr int TM = C::TM;
  constexpr int SL = kPgLoadStages, SA = kPgAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + SL;
  uint64_t* a_full = bars + 2 * SL;
  uint64_t* a_empty = a_full + SA;
  uint64_t* acc_full = a_empty + SA;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = p.KB;
  const int64_t I = (int64_t)p.m_tiles * p.n_tiles * KB, G = gridDim.x, cta = blockIdx.x;
  const int64_t ub = sk_range_start(cta, I, G), ue = sk_range_start(cta + 1, I, G);

  if (tid == 0) {
    for (int s = 0; s < SL; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&xmap);
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      SkWalk w;
      w.init(ub, ue, KB);
      int64_t li = 0;
      bool ok = true;
      while (ok && w.rem > 0) {
        const int n = w.seg_len(KB);
        const int mt = w.tile % p.m_tiles, nt = w.tile / p.m_tiles;
        for (int q = 0; q < n; ++q, ++li) {
          const int s = (int)(li % SL);
          if (li >= SL && !mbar_wait_bounded(&empty[s], ((uint32_t)(li / SL) & 1u) ^ 1u, s_abort, p.status)) {
            ok = false;
            break;
          }
          const int kb = w.kb + q;
          mbar_arrive_expect_tx(&full[s], C::X_STAGE + C::W_STAGE);
          tma_load_2d(smem + C::OFF_X + s * C::X_STAGE, &xmap, kb * kBlockK, mt * TM, &full[s]);
          bulk_g2s(smem + C::OFF_W + s * C::W_STAGE, p.W + ((int64_t)nt * KB + kb) * (int64_t)C::W_STAGE,
                   C::W_STAGE, &full[s]);
        }
        w.advance(n, KB);
      }
      for (int64_t j = li - 1; j >= 0 && j >= li - SL; --j) mbar_drain(&full[j % SL], (uint32_t)(j / SL) & 1u, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kTileN, TM);
      SkWalk w;
      w.init(ub, ue, KB);
      int64_t li = 0;
      int seg = 0;
      bool ok = true;
      while (ok && w.rem > 0) {
        const int n = w.seg_len(KB);
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait_bounded(&acc_empty[b], (uint32_t)((seg >> 1) - 1) & 1u, s_abort, p.status)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + (uint32_t)(b * TM);
        for (int q = 0; q < n; ++q, ++li) {
          const int s = (int)(li % SL), sa = (int)(li % SA);
          if (!mbar_wait_bounded(&a_full[sa], (uint32_t)(li / SA) & 1u, s_abort, p.status) ||
              !mbar_wait_bounded(&full[s], (uint32_t)(li / SL) & 1u, s_abort, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(smem + C::OFF_X + s * C::X_STAGE);
          const uint32_t aaddr = smem_u32(smem + C::OFF_A + sa * C::A_STAGE);
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k)
            umma_ss(acc, umma_desc_sw128(aaddr + k * 32), umma_desc_sw128(xaddr + k * 32), idesc,
                    (q > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&a_empty[sa]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
        w.advance(n, KB);
        ++seg;
      }
      umma_commit(done);
      mbar_drain(done, 0, p.status);
    }
  } else if (warp < 6) {
    const int r = (warp - 2) * 32 + lane;
    SkWalk w;
    w.init(ub, ue, KB);
    int64_t li = 0;
    bool ok = true;
    while (ok && w.rem > 0) {
      const int n = w.seg_len(KB);
      for (int q = 0; q < n; ++q, ++li) {
        const int s = (int)(li % SL), sa = (int)(li % SA);
        if (!warp_wait(&full[s], (uint32_t)(li / SL) & 1u, s_abort, p.status)) {
          ok = false;
          break;
        }
        const uint8_t* wst = smem + C::OFF_W + s * C::W_STAGE;
        uint4 wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const uint4*>(wst + j * kSlabBytes + r * 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        uint32_t a[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          i8x4_to_bf16x4(wv[j].x, a[8 * j + 0], a[8 * j + 1]);
          i8x4_to_bf16x4(wv[j].y, a[8 * j + 2], a[8 * j + 3]);
          i8x4_to_bf16x4(wv[j].z, a[8 * j + 4], a[8 * j + 5]);
          i8x4_to_bf16x4(wv[j].w, a[8 * j + 6], a[8 * j + 7]);
        }
        if (li >= SA && !warp_wait(&a_empty[sa], ((uint32_t)(li / SA) & 1u) ^ 1u, s_abort, p.status)) {
          ok = false;
          break;
        }
        uint8_t* arow = smem + C::OFF_A + sa * C::A_STAGE + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(arow + ((c ^ (r & 7)) << 4)) =
              make_uint4(a[4 * c], a[4 * c + 1], a[4 * c + 2], a[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
      w.advance(n, KB);
    }
  } else {
    // Epilogue: thread = channel row = TMEM lane of its quarter.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int etid = tid - 192;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    SkWalk w;
    w.init(ub, ue, KB);
    int seg = 0;
    bool ok = true;
    while (w.rem > 0) {
      const int nlen = w.seg_len(KB);
      const int b = seg & 1;
      const int mt = w.tile % p.m_tiles, nt = w.tile / p.m_tiles;
      const bool whole = w.kb == 0 && nlen == KB;
      const bool finisher = !whole && w.kb + nlen == KB;
      unsigned* counter = p.counters + w.tile;
      const int64_t T0 = (int64_t)w.tile * KB;
      const int64_t c_lo = sk_cta_of(T0, I, G), c_hi = sk_cta_of(T0 + KB - 1, I, G);
      const int first_slot = sk_range_start(c_lo, I, G) == T0 ? 0 : 1;
      float* slot = p.partials + (size_t)(cta * 2 + (w.u == ub ? 0 : 1)) * TM * kTileN;
      if (finisher) {
        if (etid == 0) sk_wait_parts(counter, (unsigned)(c_hi - c_lo), s_abort, p.status);
        named_bar_sync(1, 128);
      }
      ok = ok && warp_wait(&acc_full[b], (uint32_t)(seg >> 1) & 1u, s_abort, p.status);
      tc_fence_after();
      const int n = nt * kTileN + r;
      const bool n_ok = n < p.N;
      const float sc = n_ok ? __ldg(p.scale + n) : 0.0f;
      const float bs = (n_ok && p.bias) ? __ldg(p.bias + n) : 0.0f;
      const int m0 = mt * TM;
      for (int c0 = 0; c0 < TM && m0 + c0 < p.M; c0 += 16) {
        uint32_t v[16];
        if (ok) {
          tmem_ld_32x32b_x16(tmem_base + lane_off + (uint32_t)(b * TM + c0), v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0u;
        }
        if (!whole && !finisher) {
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(slot + (c0 + j) * kTileN + r, __uint_as_float(v[j]));
          continue;
        }
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
        if (finisher) {
          for (int64_t cc = c_lo; cc < c_hi; ++cc) {
            const float* part =
                p.partials + (size_t)(cc * 2 + (cc == c_lo ? first_slot : 0)) * TM * kTileN + (size_t)c0 * kTileN + r;
            float t[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) t[j] = __ldcg(part + j * kTileN);
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] += t[j];
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (n_ok && m < p.M) {
            float y = __fmul_rn(acc[j] + __uint_as_float(v[j]), sc);
            if (p.bias) y = __fadd_rn(y, bs);
            p.Y[(int64_t)m * p.ldy + n] = epi_apply(p.epi, y, m, n);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (!whole && !finisher) {
        named_bar_sync(1, 128);  // every part of this CTA is stored
        if (etid == 0) sk_red_release_add(counter, 1u);
      } else if (finisher && etid == 0) {
        *counter = 0u;  // left at zero for the next call
      }
      w.advance(nlen, KB);
      ++seg;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int TM, bool A_TMEM, int STAGES>
static cudaError_t launch_cfg(const GemmParams& gp, const CUtensorMap& xmap, cudaStream_t st) {
  using C = GemmCfg<TM, A_TMEM, STAGES>;
  if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(gemm_q8_tc_kernel<TM, A_TMEM, STAGES>),
                                         C::SMEM_BYTES))
    return e;
  const dim3 grid((unsigned)gp.m_tiles, (unsigned)gp.n_tiles, (unsigned)gp.splits);
  gemm_q8_tc_kernel<TM, A_TMEM, STAGES><<<grid, 192, C::SMEM_BYTES, st>>>(xmap, gp);
  return cudaGetLastError();
}

template <bool A_TMEM>
static cudaError_t launch_tm(int tm, const GemmParams& gp, const CUtensorMap& xmap, cudaStream_t st) {
  switch (tm) {
    case 16: return launch_cfg<16, A_TMEM, 4>(gp, xmap, st);
    case 32: return launch_cfg<32, A_TMEM, 4>(gp, xmap, st);
    case 64: return launch_cfg<64, A_TMEM, 4>(gp, xmap, st);
    case 128: return launch_cfg<128, A_TMEM, 4>(gp, xmap, st);
    case 256: return launch_cfg<256, A_TMEM, A_TMEM ? 4 : 3>(gp, xmap, st);
    default: return cudaErrorInvalidValue;
  }
}

bool gemm_tile_supported(int tile_m) {
  return tile_m == 16 || tile_m == 32 || tile_m == 64 || tile_m == 128 || tile_m == 256;
}

static cudaError_t launch_persistent(const GemmParams& gp, const CUtensorMap& xmap, int grid, bool stream_k,
                                     cudaStream_t st) {
  const void* k = stream_k ? reinterpret_cast<const void*>(gemm_q8_tc_streamk_kernel)
                           : reinterpret_cast<const void*>(gemm_q8_tc_persistent_kernel);
  if (cudaError_t e = ensure_smem_limit(k, PgCfg::SMEM_BYTES)) return e;
  if (stream_k)
    gemm_q8_tc_streamk_kernel<<<grid, kPgThreads, PgCfg::SMEM_BYTES, st>>>(xmap, gp);
  else
    gemm_q8_tc_persistent_kernel<<<grid, kPgThreads, PgCfg::SMEM_BYTES, st>>>(xmap, gp);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const Plan& p, const void* Xb, int64_t ldxb, const void* packed,
                           const float* scale, const float* bias, float* Y, int64_t ldy,
                           void* workspace, const CUtensorMap& xmap, int a_from_tmem,
                           unsigned* status, const Epilogue& epi, cudaStream_t st) {
  (void)Xb;
  (void)ldxb;
  GemmParams gp;
  gp.epi = epi;
  gp.W = static_cast<const uint8_t*>(packed);
  gp.scale = scale;
  gp.bias = bias;
  gp.Y = Y;
  gp.ldy = ldy;
  gp.M = (int)p.M;
  gp.N = (int)p.N;
  gp.n_pad = (int)p.n_pad;
  gp.KB = p.kunits;
  gp.kb_per_split = p.kunits_per_split;
  gp.splits = p.splits;
  gp.n_tiles = p.n_tiles;
  gp.m_tiles = p.m_tiles;
  char* ws = static_cast<char*>(workspace);
  gp.counters = ws ? reinterpret_cast<unsigned*>(ws + p.off_counters) : nullptr;
  gp.partials = ws ? reinterpret_cast<float*>(ws + p.off_partials) : nullptr;
  gp.status = status;
  if (p.persistent) return launch_persistent(gp, xmap, p.grid, p.stream_k, st);
  return a_from_tmem ? launch_tm<true>(p.tile_m, gp, xmap, st)
                     : launch_tm<false>(p.tile_m, gp, xmap, st);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

int make_x_tensor_map(CUtensorMap* map, const void* X, int64_t M, int64_t K, int64_t ldx,
                      int tile_m, bool x_f32) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -1;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * (x_f32 ? 4 : 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kBlockK, (cuuint32_t)tile_m};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      enc(map, x_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
          const_cast<void*>(X), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          x_f32 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

}  // namespace mtrtq
