// Shared device helpers for the INT8 weight-only MatMul kernels (sm_100a only).
//
// - int8 -> fp32 / bf16 conversion by the exponent-bias trick: the biased byte
//   u = q + 128 is placed in the low mantissa byte of 2^23 (0x4B0000uu), and
//   subtracting 2^23 + 128 leaves q exactly. |q| <= 128 has at most 8 significant
//   bits, so the fp32 value's upper half is also its exact bf16.
// - thin PTX wrappers for mbarriers, TMA bulk copies and tcgen05 (TMEM alloc,
//   tcgen05.mma / commit / ld / st / fences), written from the PTX ISA.
// - bounded mbarrier waits that set a device status word instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q8_internal.h"

namespace mtrtq {

// About one second of SM clock at B200 clocks: the cap on any spin-wait.
constexpr long long kSpinLimitCycles = 2000000000LL;

// ---- numeric conversion -------------------------------------------------------

__device__ __forceinline__ float i8_lane_to_f32(uint32_t biased_word, uint32_t sel) {
  // sel selects byte i (0..3) into byte 0 of 0x4B000000.
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, sel));
}

// 4 int8 (one 32-bit word) -> 4 exact floats, as two float2 pairs (k, k+1), (k+2, k+3).
__device__ __forceinline__ void i8x4_to_f32x4(uint32_t w, float2& lo, float2& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float2 a = make_float2(i8_lane_to_f32(u, 0x7540), i8_lane_to_f32(u, 0x7541));
  const float2 b = make_float2(i8_lane_to_f32(u, 0x7542), i8_lane_to_f32(u, 0x7543));
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  lo = __fadd2_rn(a, bias);  // packed fp32x2 add (sm_100)
  hi = __fadd2_rn(b, bias);
}

// Two exact small-integer floats -> one bf16x2 word (element 0 in the low half).
__device__ __forceinline__ uint32_t pack_bf16x2_exact(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

// 4 int8 -> 2 bf16x2 words (k, k+1) and (k+2, k+3), exact.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& p0, uint32_t& p1) {
  float2 lo, hi;
  i8x4_to_f32x4(w, lo, hi);
  p0 = pack_bf16x2_exact(lo.x, lo.y);
  p1 = pack_bf16x2_exact(hi.x, hi.y);
}

// d = a * b + c on both lanes (IEEE fp32 fma per lane, packed fp32x2 on sm_100).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// fp32 -> bf16 (round to nearest even) -> fp32.
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Streaming 16-byte global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- epilogue ----------------------------------------------------------------

// The epilogue (Epilogue, q8_internal.h) applied to t = (acc * scale) + bias
// before the store.
__device__ __forceinline__ float epi_apply(const Epilogue& e, float t, int64_t m, int64_t n) {
  if (e.kind == 1) {
    const float inner = 0.7978845608028654f * (t + 0.044715f * t * t * t);
    return 0.5f * t * (1.0f + tanhf(inner));
  }
  if (e.kind == 2) return __fadd_rn(e.residual[m * e.ldr + n], t);
  return t;
}

// ---- shared-memory addressing, mbarriers -------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Non-blocking test of the phase with the given parity (cheap when it has
// completed).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Tests the phase with the given parity. If it has not completed, the thread is
// suspended (not spinning, so it takes no issue slots from the warps doing the
// work) until the phase completes or about 0.1 ms passes.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false (after
// recording MTRTQ_ERR_TIMEOUT in the device status word *status and raising
// *abort) if the phase does not complete within kSpinLimitCycles, or if another
// role of the CTA has already raised *abort.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag, unsigned* status) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kSpinLimitCycles) {
      *abort_flag = 1;
      atomicExch(status, 6u /* MTRTQ_ERR_TIMEOUT */);
      return false;
    }
  }
}

// ---- split tiles: tickets ---------------------------------------------------------

// Ticket of a split tile, taken by ONE thread after a barrier of the threads that
// stored this CTA's part: the gpu-scope acq_rel atomic releases every part those
// threads stored before the barrier (release is cumulative over the barrier) and,
// for the last arriver, acquires the other CTAs' parts for the reads its threads
// make after the next barrier. One fence per CTA, where a __threadfence() by every
// thread is a sequentially consistent fence each (measured as the main stall,
// membar, of the grouped GEMV). The parts are read with ld.global.cg (L2), never
// from a stale L1 line.
__device__ __forceinline__ unsigned ticket_acq_rel(unsigned* counter) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

// ---- TMA (bulk async copies into shared memory) ------------------------------

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy global -> shared (coordinates: c0 innermost, in elements).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 / TMEM --------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// K-major operand in shared memory, 128-byte swizzle: rows of 128 bytes, 8-row
// groups 1024 bytes apart (SBO), version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (16 B, unused)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset
  d |= (uint64_t)1 << 46;                          // descriptor version
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B
  return d;
}

// K-major operand in shared memory without swizzle ("interleaved" canonical
// layout): 8 x 16-byte core matrices, the 8 rows of each at 16-byte stride; the
// two core matrices of one K = 32-byte step lbo bytes apart (leading byte
// offset), consecutive 8-row groups sbo bytes apart (stride byte offset); version
// 1 (sm_100), layout type 0 (SWIZZLE_NONE). The packed weight unit (16-k slabs of
// 128 rows x 16 bytes) is this layout with lbo = 2048 and sbo = 128.
__device__ __forceinline__ uint64_t umma_desc_interleave(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);    // start address
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;       // leading byte offset
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;       // stride byte offset
  d |= (uint64_t)1 << 46;                            // descriptor version
  return d;                                          // base offset 0, SWIZZLE_NONE
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::i8 (s8 inputs, s32 accumulate).
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::i8, A = B = signed 8-bit, D = s32, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
  return (2u << 4)                          // D format s32
         | (1u << 7)                        // A format signed 8-bit
         | (1u << 10)                       // B format signed 8-bit
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                          // D format f32
         | (1u << 7)                        // A format bf16
         | (1u << 10)                       // B format bf16
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// 32 lanes x 32 bits, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 32 bits, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- problem geometry shared by host and device ------------------------------------

constexpr int kTileN = 128;   // output channels per channel tile (MMA M)
constexpr int kSlabK = 16;    // k values per slab
constexpr int kBlockK = 64;   // k values per pipeline stage (4 slabs)
constexpr int kSlabBytes = kTileN * kSlabK;  // 2048

__host__ __device__ constexpr int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ constexpr int64_t round_up64(int64_t a, int64_t b) { return ceil_div64(a, b) * b; }

}  // namespace mtrtq
