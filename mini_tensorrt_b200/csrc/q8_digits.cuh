// Device helpers shared by the int8-weight GEMV kernels that multiply the int8
// weights, unconverted, by int8 digits of the activations on integer warp MMAs
// (gemv_cluster.cu, gemv_stream.cu). sm_100a only.
#pragma once

#include "q8_common.cuh"

namespace mtrtq {

// Programmatic dependent launch (no-ops unless the launch enabled it): wait for
// the grids this one depends on to complete and their writes to be visible; let
// the grids that depend on this one start launching.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// d[0..3] += A(16x32 s8) * B(32x8 s8), int32 accumulate (exact).
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Weight fragments of one m16n8k32 step from a unit in shared memory ([slab][128
// rows][16 B]): slabs s and s + 1 of rows ra0 .. ra0 + 15. Each of the four 8 x 16 B
// matrices is eight consecutive rows of one slab, 128 contiguous bytes, so the
// load has no bank conflict (16-byte loads of one row from four slabs 2 KiB
// apart, by the four lanes of an MMA group, would meet in the same banks); lane
// l addresses row l & 7 of matrix l >> 3, and lane (g, t) receives bytes
// 4t .. 4t + 3 of row g of each matrix: the A fragment (rows g and g + 8,
// k = 16 s + 4t .. and 16 (s + 1) + 4t ..).
__device__ __forceinline__ void ld_weight_frag(const unsigned char* unit_base, int ra0, int s, int lane,
                                               uint32_t (&a)[4]) {
  const int mat = lane >> 3;
  const uint32_t addr = smem_u32(unit_base + (size_t)(s + (mat >> 1)) * 2048 +
                                 (size_t)(ra0 + (lane & 7) + (mat & 1) * 8) * 16);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
               : "r"(addr));
}

// Four consecutive activations of row m from k (zeros past K) as fp32; a vector
// load when the row stride allows it and all four lie inside the row.
template <bool X_BF16>
__device__ __forceinline__ float4 load_x4(const void* X, int64_t ldx, int K, int m, int k, bool vec) {
  const int64_t off = (int64_t)m * ldx + k;
  if (X_BF16) {
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(X) + off;
    if (vec && k + 3 < K) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(x));
      return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                         __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    }
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = k + i < K ? __bfloat162float(x[i]) : 0.0f;
    return make_float4(v[0], v[1], v[2], v[3]);
  }
  const float* x = static_cast<const float*>(X) + off;
  if (vec && k + 3 < K) return __ldg(reinterpret_cast<const float4*>(x));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = k + i < K ? __ldg(x + i) : 0.0f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

template <bool ROUND>
__device__ __forceinline__ float4 cl_round(float4 v) {
  if (ROUND) {
    v.x = round_bf16(v.x);
    v.y = round_bf16(v.y);
    v.z = round_bf16(v.z);
    v.w = round_bf16(v.w);
  }
  return v;
}

// Three int8 digits of v (|v| <= 127): v ~ d0 + d1 / 2^7 + d2 / 2^14. Each
// residual is exact in fp32 (it is the difference of two nearby values, then
// scaled by a power of two); the last digit's rounding leaves |error| <= 2^-15.
//
// Rounding to the nearest integer (ties to even) is an add of 1.5 * 2^23: for
// |v| < 2^22 the sum's spacing is 1, so the sum holds round(v) as a two's
// complement offset in its low mantissa bits, and the low byte of its bit
// pattern is the int8 digit. Plain adds and multiplies, where a float-to-integer
// conversion would run on the narrower conversion pipe. w0, w1, w2 receive the
// three sums' bit patterns.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
__device__ __forceinline__ void cl_digits(float v, uint32_t& w0, uint32_t& w1, uint32_t& w2) {
  const float t0 = __fadd_rn(v, kRoundMagic);
  const float v1 = __fmul_rn(__fsub_rn(v, __fsub_rn(t0, kRoundMagic)), 128.0f);
  const float t1 = __fadd_rn(v1, kRoundMagic);
  const float v2 = __fmul_rn(__fsub_rn(v1, __fsub_rn(t1, kRoundMagic)), 128.0f);
  const float t2 = __fadd_rn(v2, kRoundMagic);
  w0 = __float_as_uint(t0);
  w1 = __float_as_uint(t1);
  w2 = __float_as_uint(t2);
}

// The low bytes of a, b, c, e as one word (a in byte 0).
__device__ __forceinline__ uint32_t cl_pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t e) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, e, 0x0040), 0x5410);
}

// max |v| over a group, and whether any of its values is NaN or infinite: fmaxf
// drops a NaN, so the sum of the four values (NaN if any of them is) is tested
// too; an infinity shows in the maximum.
__device__ __forceinline__ float cl_group_max(const float4 v, bool& bad) {
  const float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  const float sum = (v.x + v.y) + (v.z + v.w);
  bad |= !(a <= 3.402823466e38f) || sum != sum;
  return a;
}

// Writes the three digit planes of group g (k = 4g .. 4g + 3 of the CTA's range)
// of token m.
__device__ __forceinline__ void cl_store_digit_group(const float4 v, float inv, int8_t* xd, int plane, int mt,
                                                     int m, int g) {
  uint32_t a0, a1, a2, b0, b1, b2, c0, c1, c2, e0, e1, e2;
  cl_digits(__fmul_rn(v.x, inv), a0, a1, a2);
  cl_digits(__fmul_rn(v.y, inv), b0, b1, b2);
  cl_digits(__fmul_rn(v.z, inv), c0, c1, c2);
  cl_digits(__fmul_rn(v.w, inv), e0, e1, e2);
  // Group q = g & 15 of the unit (k = 4q .. 4q + 3) sits at byte (q & 3) * 16 +
  // (q >> 2) * 4 of the token's 64-byte row: lane t of an MMA group then finds
  // its four B-fragment words (k = 4t + 16j, j = 0..3) in one 16-byte load.
  const int u = g >> 4, q = g & 15;
  const int off = (u * mt + m) * 64 + (q & 3) * 16 + (q >> 2) * 4;
  *reinterpret_cast<uint32_t*>(xd + off) = cl_pack_low_bytes(a0, b0, c0, e0);
  *reinterpret_cast<uint32_t*>(xd + plane + off) = cl_pack_low_bytes(a1, b1, c1, e1);
  *reinterpret_cast<uint32_t*>(xd + 2 * plane + off) = cl_pack_low_bytes(a2, b2, c2, e2);
}

}  // namespace mtrtq
