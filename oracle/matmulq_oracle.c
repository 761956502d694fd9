/*
 * CPU oracle for the INT8 weight-only MatMul (MatMulQ) hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA path is
 * compared against; it is linked by tests/, by __graft_entry__.smoke() and by
 * the cpu_baseline leg of bench.py, never by the product library.
 *
 * Parity pin: every function here is compared bit-for-bit (tests/test_oracle.py)
 * against the reference's own code compiled from its sources by
 * oracle/build_ref.sh (oracle/_ref/libmtrt_ref.so), and against the reference's
 * Golden.MatMulQ fixture (tests/golden/).
 *
 * Arithmetic is plain IEEE fp32 in the same order as the reference; build with
 * -ffp-contract=off so no multiply-add is fused (the reference's x86-64 build
 * has no FMA either).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/*
 * Symmetric per-output-channel int8 quantization of W[K,N] (row-major, "in,out").
 * Follows the reference packer in tests/golden_kernel_test.cpp:163-170:
 *   amax_j = max_k |W[k,j]|           (running std::max over k, fp32)
 *   s_j    = amax_j / 127.0f          (fp32 division)
 *   q[k,j] = (int8_t) lround(W[k,j] / s_j)   (ties away from zero, no clamp)
 * A column of zeros has amax = 0; the reference then computes 0/0 and casts
 * lround(NaN) to int8, which is 0 on x86-64. This restatement writes s_j = 0
 * and q = 0 explicitly, which is the same bytes without the undefined step.
 * Returns the number of all-zero columns.
 */
int64_t oracle_quantize_per_channel(const float* W, int64_t K, int64_t N, int8_t* q,
                                    float* scale) {
  int64_t zero_cols = 0;
  for (int64_t j = 0; j < N; ++j) {
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      const float a = fabsf(W[k * N + j]);
      amax = amax < a ? a : amax; /* std::max(amax, |w|) */
    }
    const float sc = amax / 127.0f;
    scale[j] = sc;
    if (amax == 0.0f) {
      ++zero_cols;
      for (int64_t k = 0; k < K; ++k) q[k * N + j] = 0;
      continue;
    }
    for (int64_t k = 0; k < K; ++k) q[k * N + j] = (int8_t)lroundf(W[k * N + j] / sc);
  }
  return zero_cols;
}

/*
 * C[M,N] = A[M,K] (f32) x dequant(W[K,N] i8, scale[N]).
 * Follows src/ops/kernels_matmul.cpp:66-73: for each (i, j) an fp32 accumulator
 * sums a[i*K+k] * (float)w[k*N+j] in ascending k, and the scale multiplies the
 * finished sum once.
 */
void oracle_matmul_q8_f32(const float* A, const int8_t* W, const float* s, float* C,
                          int64_t M, int64_t K, int64_t N) {
  for (int64_t i = 0; i < M; ++i) {
    for (int64_t j = 0; j < N; ++j) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += A[i * K + k] * (float)W[k * N + j];
      C[i * N + j] = acc * s[j];
    }
  }
}

/*
 * Same arithmetic as oracle_matmul_q8_f32 for a subset of rows: rows[r] selects
 * the row of A and the row of C written (C is [n_rows, N]). Rows are
 * independent in the reference loop, so a sampled check is exact.
 */
void oracle_matmul_q8_f32_rows(const float* A, const int8_t* W, const float* s, float* C,
                               const int64_t* rows, int64_t n_rows, int64_t K, int64_t N) {
  for (int64_t r = 0; r < n_rows; ++r) {
    const float* a = A + rows[r] * K;
    for (int64_t j = 0; j < N; ++j) {
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k) acc += a[k] * (float)W[k * N + j];
      C[r * N + j] = acc * s[j];
    }
  }
}

/*
 * Bias broadcast over rows: Y[i,j] += b[j].
 * Follows src/ops/kernels_elementwise.cpp:31-35 (out = a + b[i % N]).
 */
void oracle_add_bias(float* Y, const float* b, int64_t M, int64_t N) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) Y[i * N + j] = Y[i * N + j] + b[j];
}

/*
 * Round-to-nearest-even fp32 -> bf16 -> fp32, the activation rounding the
 * bf16 mode of the CUDA path applies to X before the product. Used to build the
 * "after bf16 activation rounding" comparison input. NaN is passed through.
 */
void oracle_round_bf16(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &x[i], 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
      y[i] = x[i];
      continue;
    }
    const uint32_t lsb = (u >> 16) & 1u;
    u = (u + 0x7fffu + lsb) & 0xffff0000u;
    memcpy(&y[i], &u, 4);
  }
}
