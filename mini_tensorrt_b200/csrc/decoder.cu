// Device kernels of the GPT-2 KV-cache decode loop around MatMulQ.
//
// They restate, one launch each, the steps of the reference's KVDecoder::step
// (tools/run_gpt2.cpp:135-191) that are not MatMulQ: token + position embedding
// (:138-140), LayerNorm with biased variance and eps 1e-5 (:113-122), attention
// of the new query over the cached keys and values (:146-172), gelu_new
// (:178-181), the residual adds (:174, :183) and the greedy argmax
// (:42-47, first index of the maximum; the residual adds and gelu_new are also
// available fused into MatMulQ, mtrtq_matmul_ex). All sequences of a batch sit at the same
// position, which lives in device memory so that one CUDA graph replays every
// step; the embedding reads the prompt while the position is inside it, and the
// previous step's argmax after it.
//
// The arithmetic is fp32 with the reference's formulas (mean, then the biased
// variance of the centred values; max-subtracted exponentials; weights times
// values); sums over a row or over keys are split across threads and added in a
// fixed tree order, so results do not depend on timing.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "../../include/mtrtq.h"

namespace mtrtq {
// MTRTQ_OPT_OVERLAP_LAUNCH (abi.cu).
bool overlap_launch_enabled();

namespace {

// Programmatic dependent launch. Every kernel here starts with pdl_begin(): it
// waits until the grid ahead of it in the stream has completed and its writes are
// visible (a no-op when the launch did not ask for programmatic serialization),
// and only then touches global memory; it then lets the grid behind it start
// launching, so that grid's set-up overlaps this one.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block (blockDim.x a multiple of 32, <= 1024); every thread gets it.
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  t = warp_sum(t);
  return t;
}

// x[b, :] = wte[tok, :] + wpe[pos, :], tok = prompt[b, pos] while pos < prompt_len,
// else next_tok[b].
__global__ void embed_kernel(const int32_t* prompt, int64_t prompt_len, const int32_t* next_tok,
                             const int32_t* pos_p, const float* wte, const float* wpe, float* x,
                             int64_t D, int64_t V, int64_t n_pos) {
  pdl_begin();
  const int64_t b = blockIdx.x;
  const int pos = *pos_p;
  if (pos < 0 || pos >= n_pos) {  // past the position table: zeros, no read out of bounds
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) x[b * D + i] = 0.0f;
    return;
  }
  int64_t tok = pos < prompt_len ? prompt[b * prompt_len + pos] : next_tok[b];
  if (tok < 0 || tok >= V) tok = 0;  // ids outside the vocabulary read row 0
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x)
    x[b * D + i] = wte[tok * D + i] + wpe[(int64_t)pos * D + i];
}

// One block per row: y = (x - mean) / sqrt(var + eps) * gamma + beta. Rows of up
// to kLnRegs * blockDim.x elements stay in registers (one read of x); longer rows
// are read again for each pass.
constexpr int kLnRegs = 8;

__global__ void layernorm_kernel(const float* x, int64_t ldx, const float* g, const float* bta, float* y,
                                 int64_t D, float eps) {
  __shared__ float red[32];
  pdl_begin();
  const float* xr = x + blockIdx.x * ldx;
  float* yr = y + blockIdx.x * D;
  const bool in_regs = D <= (int64_t)kLnRegs * blockDim.x;
  float v[kLnRegs];
  float s = 0.0f;
  if (in_regs) {
#pragma unroll
    for (int c = 0; c < kLnRegs; ++c) {
      const int64_t i = threadIdx.x + (int64_t)c * blockDim.x;
      v[c] = i < D ? xr[i] : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < kLnRegs; ++c) s += v[c];
  } else {
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) s += xr[i];
  }
  const float mean = block_sum(s, red) / (float)D;
  float q = 0.0f;
  if (in_regs) {
#pragma unroll
    for (int c = 0; c < kLnRegs; ++c) {
      const int64_t i = threadIdx.x + (int64_t)c * blockDim.x;
      const float cv = v[c] - mean;
      if (i < D) q += cv * cv;
    }
  } else {
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
      const float c = xr[i] - mean;
      q += c * c;
    }
  }
  const float var = block_sum(q, red) / (float)D;
  const float inv = 1.0f / sqrtf(var + eps);
  if (in_regs) {
#pragma unroll
    for (int c = 0; c < kLnRegs; ++c) {
      const int64_t i = threadIdx.x + (int64_t)c * blockDim.x;
      if (i < D) yr[i] = (v[c] - mean) * inv * g[i] + bta[i];
    }
  } else {
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) yr[i] = (xr[i] - mean) * inv * g[i] + bta[i];
  }
}

// One block of kAttnThreads per (head, sequence). qkv: [B, 3D] rows (q | k | v).
// Appends this position's k and v (its head slice) to the caches [B, max_ctx, D],
// then out[b, head slice] = softmax(q . K / sqrt(d)) V over cached positions
// 0..pos. Decode attention is a chain of dependent memory reads, so every step
// keeps many reads in flight instead of walking keys one after another:
// * scores: a thread per key, its dot product over head_dim in k order (16-byte
//   loads when the rows allow them, all issued before they are used);
// * softmax: the max and the sum of exponentials as block reductions (fixed tree
//   order);
// * weighted sum: thread (g, c) adds keys g, g + G, ... for column chunk c (4
//   columns, or 1), and the G groups' partial sums are added in group order.
// Every sum has a fixed order, so results do not depend on timing.
// Dynamic shared memory: head_dim + max_ctx (rounded up to a multiple of 4) +
// max(head_dim, kAttnThreads * 4) floats.
constexpr int kAttnThreads = 256;

__device__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const float* qkv, float* kc, float* vc,
                                                                 const int32_t* pos_p, float* out,
                                                                 int64_t H, int64_t hd, int64_t max_ctx) {
  extern __shared__ float sm[];
  __shared__ float red[32];
  pdl_begin();
  const int64_t h = blockIdx.x, b = blockIdx.y;
  const int64_t D = H * hd;
  const int pos = *pos_p;
  const int tid = threadIdx.x;
  if (pos < 0 || pos >= max_ctx) {  // past the cache: zeros, no access out of bounds
    for (int64_t t = tid; t < hd; t += blockDim.x) out[b * D + h * hd + t] = 0.0f;
    return;
  }
  float* qs = sm;                 // [hd]
  float* sc = sm + hd;            // [max_ctx]
  float* part = sm + ((hd + max_ctx + 3) & ~(int64_t)3);  // [G][hd], 16-byte aligned
  const float* row = qkv + b * 3 * D;
  float* kb = kc + b * max_ctx * D + h * hd;
  float* vb = vc + b * max_ctx * D + h * hd;
  for (int64_t t = tid; t < hd; t += blockDim.x) {
    qs[t] = row[h * hd + t];
    kb[(int64_t)pos * D + t] = row[D + h * hd + t];
    vb[(int64_t)pos * D + t] = row[2 * D + h * hd + t];
  }
  __syncthreads();
  // 16-byte loads of cache rows when every row start is 16-byte aligned.
  const bool vec = (hd % 4 == 0) && (D % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) % 16 == 0);
  const float scale = 1.0f / sqrtf((float)hd);
  for (int j = tid; j <= pos; j += blockDim.x) {
    const float* kj = kb + (int64_t)j * D;
    float s = 0.0f;
    if (vec) {
      for (int64_t t = 0; t < hd; t += 16) {
        float4 k4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          k4[i] = t + 4 * i < hd ? *reinterpret_cast<const float4*>(kj + t + 4 * i)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (t + 4 * i < hd) {
            const float* qq = qs + t + 4 * i;
            s += qq[0] * k4[i].x;
            s += qq[1] * k4[i].y;
            s += qq[2] * k4[i].z;
            s += qq[3] * k4[i].w;
          }
        }
      }
    } else {
      for (int64_t t = 0; t < hd; ++t) s += qs[t] * kj[t];
    }
    sc[j] = s * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = tid; j <= pos; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = block_max(mx, red);
  float sum = 0.0f;
  for (int j = tid; j <= pos; j += blockDim.x) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = block_sum(sum, red);  // ends with the exponentials visible block-wide
  const float inv = 1.0f / sum;
  // Weighted sum over (key group, column chunk) threads.
  const int w = vec ? 4 : 1;
  const int nc = (int)((hd + w - 1) / w);            // column chunks
  const int G = nc >= blockDim.x ? 1 : blockDim.x / nc;  // key groups
  const int g = tid / nc;
  if (g < G) {
    for (int c = tid % nc; c < nc; c += (nc >= blockDim.x ? blockDim.x : nc)) {
      if (vec) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        int j = g;
        for (; j + 3 * G <= pos; j += 4 * G) {  // four keys' loads in flight
          float4 v4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) v4[i] = *reinterpret_cast<const float4*>(vb + (int64_t)(j + i * G) * D + 4 * c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = sc[j + i * G] * inv;
            a.x += p * v4[i].x;
            a.y += p * v4[i].y;
            a.z += p * v4[i].z;
            a.w += p * v4[i].w;
          }
        }
        for (; j <= pos; j += G) {
          const float4 v4 = *reinterpret_cast<const float4*>(vb + (int64_t)j * D + 4 * c);
          const float p = sc[j] * inv;
          a.x += p * v4.x;
          a.y += p * v4.y;
          a.z += p * v4.z;
          a.w += p * v4.w;
        }
        *reinterpret_cast<float4*>(part + (int64_t)g * hd + 4 * c) = a;
      } else {
        float a = 0.0f;
        for (int j = g; j <= pos; j += G) a += (sc[j] * inv) * vb[(int64_t)j * D + c];
        part[(int64_t)g * hd + c] = a;
      }
    }
  }
  __syncthreads();
  for (int64_t t = tid; t < hd; t += blockDim.x) {
    float a = 0.0f;
    for (int q = 0; q < G; ++q) a += part[(int64_t)q * hd + t];
    out[b * D + h * hd + t] = a;
  }
}

__global__ void gelu_tanh_kernel(const float* x, float* y, int64_t n) {
  pdl_begin();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float u = x[i];
    y[i] = 0.5f * u * (1.0f + tanhf(0.7978845608028654f * (u + 0.044715f * u * u * u)));
  }
}

__global__ void add_kernel(float* y, const float* a, int64_t n) {
  pdl_begin();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] += a[i];
}

// Greedy argmax in two launches. A 64-bit key orders (value, index) so that the
// larger key is the larger value and, between equal values, the lower index:
// high word = the float's bits made monotonic as an unsigned integer, low word =
// ~index. argmax_fold_kernel: one block per (chunk of 4096 logits, row) folds its
// chunk's best key into best[row] with atomicMax (order-free, so deterministic).
// NaN logits are skipped.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t hi = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)hi << 32) | (uint32_t)(~(uint32_t)idx);
}

constexpr int kArgmaxChunk = 4096;

__global__ void argmax_fold_kernel(const float* logits, int64_t V, int64_t ldl, unsigned long long* best) {
  __shared__ unsigned long long bk[32];
  pdl_begin();
  const float* r = logits + blockIdx.y * ldl;
  const int64_t j0 = (int64_t)blockIdx.x * kArgmaxChunk;
  const int64_t j1 = j0 + kArgmaxChunk < V ? j0 + kArgmaxChunk : V;
  unsigned long long k = 0;
  for (int64_t j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const float v = r[j];
    if (v == v) {
      const unsigned long long c = argmax_key(v, (int)j);
      k = c > k ? c : k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
    k = ok > k ? ok : k;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) bk[warp] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w) k = bk[w] > k ? bk[w] : k;
    if (k) atomicMax(best + blockIdx.y, k);
  }
}

// tok[r] = the index in best[r] (0 for a row with no finite logit), history[*pos *
// rows + r] too, best[r] = 0 for the next step; then *pos += 1.
__global__ void decode_next_kernel(unsigned long long* best, int64_t rows, int32_t* tok, int32_t* history,
                                   int64_t history_len, int32_t* pos) {
  pdl_begin();
  const int p = *pos;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    const unsigned long long k = best[r];
    const int idx = k ? (int)(~(uint32_t)(k & 0xffffffffu)) : 0;
    tok[r] = idx;
    if (history && p >= 0 && p < history_len) history[(int64_t)p * rows + r] = idx;
    best[r] = 0ull;
  }
  __syncthreads();
  if (threadIdx.x == 0) *pos = p + 1;
}

// ---- prefill of a whole prompt -------------------------------------------------

// x[b * P + i, :] = wte[ids[b, i], :] + wpe[i, :] for every prompt position i: one
// block per (position, sequence). Ids outside the vocabulary read row 0.
__global__ void prefill_embed_kernel(const int32_t* ids, int64_t P, const float* wte, const float* wpe,
                                     float* x, int64_t D, int64_t V) {
  pdl_begin();
  const int64_t i = blockIdx.x, b = blockIdx.y;
  int64_t tok = ids[b * P + i];
  if (tok < 0 || tok >= V) tok = 0;
  float* row = x + (b * P + i) * D;
  for (int64_t c = threadIdx.x; c < D; c += blockDim.x) row[c] = wte[tok * D + c] + wpe[i * D + c];
}

// Causal attention over a prompt of P positions, one block of kPrefillWarps warps
// per (head, sequence): the keys and values of positions 0..P-1 (the head's slice
// of qkv [B*P, 3D] rows q | k | v) go to the caches [B, max_ctx, D], and for every
// query position i a warp computes, as the reference does one position at a time
// (tools/run_gpt2.cpp:152-172): scores q_i . k_j * (1 / sqrt(d)) for j <= i (a lane
// per key, each dot product in k order), the max-subtracted exponentials and their
// sum (lane tree in fixed order), then out[b * P + i, head slice] = sum over j, in
// ascending j, of (e_j * (1 / sum)) v_j (a lane per column).
constexpr int kPrefillWarps = 8;
__global__ void __launch_bounds__(kPrefillWarps * 32)
    prefill_attention_kernel(const float* qkv, float* kc, float* vc, float* out, int64_t P, int64_t H,
                             int64_t d, int64_t max_ctx) {
  pdl_begin();
  extern __shared__ float sc[];  // [kPrefillWarps][P] scores
  const int64_t h = blockIdx.x, b = blockIdx.y, D = H * d;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = qkv + b * P * 3 * D;
  // k and v of every prompt position into the caches (this head's columns).
  for (int64_t e = threadIdx.x; e < P * d; e += blockDim.x) {
    const int64_t i = e / d, t = e - i * d;
    const float* r = base + i * 3 * D + h * d + t;
    kc[(b * max_ctx + i) * D + h * d + t] = r[D];
    vc[(b * max_ctx + i) * D + h * d + t] = r[2 * D];
  }
  const float scale = 1.0f / sqrtf((float)d);
  float* s = sc + warp * P;
  for (int64_t i = warp; i < P; i += kPrefillWarps) {
    const float* q = base + i * 3 * D + h * d;
    float mx = -INFINITY;
    for (int64_t j = lane; j <= i; j += 32) {
      const float* k = base + j * 3 * D + D + h * d;
      float acc = 0.0f;
      for (int64_t t = 0; t < d; ++t) acc += q[t] * k[t];
      acc *= scale;
      s[j] = acc;
      mx = fmaxf(mx, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int64_t j = lane; j <= i; j += 32) {
      const float e = expf(s[j] - mx);
      s[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    __syncwarp();
    for (int64_t t = lane; t < d; t += 32) {
      float acc = 0.0f;
      for (int64_t j = 0; j <= i; ++j) acc += (s[j] * inv) * base[j * 3 * D + 2 * D + h * d + t];
      out[(b * P + i) * D + h * d + t] = acc;
    }
    __syncwarp();
  }
}

int launch_status(cudaError_t e) { return e == cudaSuccess ? MTRTQ_OK : MTRTQ_ERR_CUDA; }

// Launches kern on `stream`, with programmatic stream serialization when
// MTRTQ_OPT_OVERLAP_LAUNCH is set (every kernel here waits for the grid ahead
// before it reads or writes global memory, so the attribute is safe for them).
template <typename... Params, typename... Args>
int launch_helper(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, void* stream,
                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap_launch_enabled() ? 1 : 0;
  return launch_status(cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...));
}

}  // namespace
}  // namespace mtrtq

using namespace mtrtq;

extern "C" {

int mtrtq_decode_embed(const int32_t* prompt, int64_t prompt_len, const int32_t* next_tok,
                       const int32_t* pos, const float* wte, const float* wpe, int64_t n_pos, float* x,
                       int64_t B, int64_t D, int64_t V, void* stream) {
  if (!pos || !wte || !wpe || !x || !next_tok || B <= 0 || D <= 0 || V <= 0 || n_pos <= 0 ||
      (prompt_len > 0 && !prompt) || B > 65535)
    return MTRTQ_ERR_INVALID_ARG;
  return launch_helper(embed_kernel, dim3((unsigned)B), dim3(256), 0, stream, prompt, prompt_len,
                       next_tok, pos, wte, wpe, x, D, V, n_pos);
}

int mtrtq_layernorm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                    int64_t D, float eps, void* stream) {
  if (!x || !gamma || !beta || !y || rows <= 0 || D <= 0 || rows > 2147483647) return MTRTQ_ERR_INVALID_ARG;
  return launch_helper(layernorm_kernel, dim3((unsigned)rows), dim3(256), 0, stream, x, D, gamma, beta, y,
                       D, eps);
}

int mtrtq_layernorm_strided(const float* x, int64_t ldx, const float* gamma, const float* beta, float* y,
                            int64_t rows, int64_t D, float eps, void* stream) {
  if (!x || !gamma || !beta || !y || rows <= 0 || D <= 0 || ldx < D || rows > 2147483647)
    return MTRTQ_ERR_INVALID_ARG;
  return launch_helper(layernorm_kernel, dim3((unsigned)rows), dim3(256), 0, stream, x, ldx, gamma, beta, y,
                       D, eps);
}

int mtrtq_decode_attention(const float* qkv, float* kcache, float* vcache, const int32_t* pos,
                           float* out, int64_t B, int64_t H, int64_t head_dim, int64_t max_ctx,
                           void* stream) {
  if (!qkv || !kcache || !vcache || !pos || !out || B <= 0 || H <= 0 || head_dim <= 0 ||
      max_ctx <= 0 || B > 65535 || H > 2147483647)
    return MTRTQ_ERR_INVALID_ARG;
  // q, the scores and the key groups' partial sums (at most kAttnThreads chunks of
  // up to 4 columns each, or one group of head_dim columns).
  const int64_t parts = head_dim > 4 * kAttnThreads ? head_dim : 4 * kAttnThreads;
  const size_t smem = (size_t)(((head_dim + max_ctx + 3) & ~(int64_t)3) + parts) * sizeof(float);
  if (smem > 48 * 1024) return MTRTQ_ERR_INVALID_ARG;  // contexts up to ~11k positions at d = 64
  return launch_helper(attention_kernel, dim3((unsigned)H, (unsigned)B), dim3(kAttnThreads), smem,
                       stream, qkv, kcache, vcache, pos, out, H, head_dim, max_ctx);
}

int mtrtq_prefill_embed(const int32_t* ids, int64_t B, int64_t P, const float* wte, const float* wpe,
                        int64_t n_pos, float* x, int64_t D, int64_t V, void* stream) {
  if (!ids || !wte || !wpe || !x || B <= 0 || P <= 0 || D <= 0 || V <= 0 || P > n_pos || B > 65535 ||
      P > 2147483647)
    return MTRTQ_ERR_INVALID_ARG;
  return launch_helper(prefill_embed_kernel, dim3((unsigned)P, (unsigned)B), dim3(256), 0, stream, ids, P,
                       wte, wpe, x, D, V);
}

int mtrtq_prefill_attention(const float* qkv, float* kcache, float* vcache, float* out, int64_t B, int64_t P,
                            int64_t H, int64_t head_dim, int64_t max_ctx, void* stream) {
  if (!qkv || !kcache || !vcache || !out || B <= 0 || P <= 0 || H <= 0 || head_dim <= 0 || P > max_ctx ||
      B > 65535 || H > 65535)
    return MTRTQ_ERR_INVALID_ARG;
  const size_t smem = (size_t)kPrefillWarps * (size_t)P * sizeof(float);
  if (smem > 48 * 1024) return MTRTQ_ERR_INVALID_ARG;  // prompts up to 1536 positions
  return launch_helper(prefill_attention_kernel, dim3((unsigned)H, (unsigned)B), dim3(kPrefillWarps * 32), smem,
                       stream, qkv, kcache, vcache, out, P, H, head_dim, max_ctx);
}

int mtrtq_gelu_tanh(const float* x, float* y, int64_t n, void* stream) {
  if (!x || !y || n <= 0) return MTRTQ_ERR_INVALID_ARG;
  const int64_t blocks = n / 256 + 1 < 4096 ? n / 256 + 1 : 4096;
  return launch_helper(gelu_tanh_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, x, y, n);
}

int mtrtq_add_inplace(float* y, const float* a, int64_t n, void* stream) {
  if (!y || !a || n <= 0) return MTRTQ_ERR_INVALID_ARG;
  const int64_t blocks = n / 256 + 1 < 4096 ? n / 256 + 1 : 4096;
  return launch_helper(add_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, y, a, n);
}

int mtrtq_argmax_rows(const float* logits, int64_t rows, int64_t V, int64_t ldl,
                      unsigned long long* best, void* stream) {
  if (!logits || !best || rows <= 0 || V <= 0 || ldl < V || rows > 65535 || V > 2147483647)
    return MTRTQ_ERR_INVALID_ARG;
  const int64_t chunks = (V + kArgmaxChunk - 1) / kArgmaxChunk;
  return launch_helper(argmax_fold_kernel, dim3((unsigned)chunks, (unsigned)rows), dim3(256), 0, stream,
                       logits, V, ldl, best);
}

int mtrtq_decode_next(unsigned long long* best, int64_t rows, int32_t* tok, int32_t* history,
                      int64_t history_len, int32_t* pos, void* stream) {
  if (!best || !tok || !pos || rows <= 0 || (history_len > 0 && !history)) return MTRTQ_ERR_INVALID_ARG;
  return launch_helper(decode_next_kernel, dim3(1), dim3(256), 0, stream, best, rows, tok, history,
                       history_len, pos);
}

}  // extern "C"
