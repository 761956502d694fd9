// Device kernels of the GPT-2 KV-cache decode loop around MatMulQ.
//
// They restate, one launch each, the steps of the reference's KVDecoder::step
// (tools/run_gpt2.cpp:135-191) that are not MatMulQ: token + position embedding
// (:138-140), LayerNorm with biased variance and eps 1e-5 (:113-122), attention
// of the new query over the cached keys and values (:146-172), gelu_new
// (:178-181), the residual adds (:174, :183) and the greedy argmax
// (:42-47, first index of the maximum). All sequences of a batch sit at the same
// position, which lives in device memory so that one CUDA graph replays every
// step; the embedding reads the prompt while the position is inside it, and the
// previous step's argmax after it.
//
// The arithmetic is fp32 in the reference's order where it has one (mean, then
// the biased variance of the centred values; scores, max, exp and sum in key
// order; weights times values in key order); block reductions add in a tree.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "../../include/mtrtq.h"

namespace mtrtq {
namespace {

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

// One block per row: y = (x - mean) / sqrt(var + eps) * gamma + beta.
__global__ void layernorm_kernel(const float* x, const float* g, const float* bta, float* y,
                                 int64_t D, float eps) {
  __shared__ float red[32];
  const float* xr = x + blockIdx.x * D;
  float* yr = y + blockIdx.x * D;
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s, red) / (float)D;
  float v = 0.0f;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    const float c = xr[i] - mean;
    v += c * c;
  }
  const float var = block_sum(v, red) / (float)D;
  const float inv = 1.0f / sqrtf(var + eps);
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) yr[i] = (xr[i] - mean) * inv * g[i] + bta[i];
}

// One block per (head, sequence). qkv: [B, 3D] rows (q | k | v). Appends this
// position's k and v (its head slice) to the caches [B, max_ctx, D], then
// out[b, head slice] = softmax(q . K / sqrt(d)) V over cached positions 0..pos.
// Dynamic shared memory: max_ctx + head_dim floats.
__global__ void attention_kernel(const float* qkv, float* kc, float* vc, const int32_t* pos_p,
                                 float* out, int64_t H, int64_t hd, int64_t max_ctx) {
  extern __shared__ float sm[];
  __shared__ float red[32];
  const int64_t h = blockIdx.x, b = blockIdx.y;
  const int64_t D = H * hd;
  const int pos = *pos_p;
  if (pos < 0 || pos >= max_ctx) {  // past the cache: zeros, no access out of bounds
    for (int64_t t = threadIdx.x; t < hd; t += blockDim.x) out[b * H * hd + h * hd + t] = 0.0f;
    return;
  }
  float* qs = sm;            // [hd]
  float* sc = sm + hd;       // [max_ctx]
  const float* row = qkv + b * 3 * D;
  float* kb = kc + b * max_ctx * D;
  float* vb = vc + b * max_ctx * D;
  for (int64_t t = threadIdx.x; t < hd; t += blockDim.x) {
    qs[t] = row[h * hd + t];
    kb[(int64_t)pos * D + h * hd + t] = row[D + h * hd + t];
    vb[(int64_t)pos * D + h * hd + t] = row[2 * D + h * hd + t];
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)hd);
  // scores: one warp per key, lanes over the head dimension
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int j = warp; j <= pos; j += nw) {
    const float* kj = kb + (int64_t)j * D + h * hd;
    float s = 0.0f;
    for (int64_t t = lane; t < hd; t += 32) s += qs[t] * kj[t];
    s = warp_sum(s);
    if (lane == 0) sc[j] = s * scale;
  }
  __syncthreads();
  // max, then exp and sum in key order (one thread: at most max_ctx terms)
  if (threadIdx.x == 0) {
    float mx = -1e30f;
    for (int j = 0; j <= pos; ++j) mx = sc[j] > mx ? sc[j] : mx;
    float sum = 0.0f;
    for (int j = 0; j <= pos; ++j) {
      sc[j] = expf(sc[j] - mx);
      sum += sc[j];
    }
    red[0] = 1.0f / sum;
  }
  __syncthreads();
  const float inv = red[0];
  for (int64_t t = threadIdx.x; t < hd; t += blockDim.x) {
    float a = 0.0f;
    for (int j = 0; j <= pos; ++j) a += (sc[j] * inv) * vb[(int64_t)j * D + h * hd + t];
    out[b * D + h * hd + t] = a;
  }
}

__global__ void gelu_tanh_kernel(const float* x, float* y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float u = x[i];
    y[i] = 0.5f * u * (1.0f + tanhf(0.7978845608028654f * (u + 0.044715f * u * u * u)));
  }
}

__global__ void add_kernel(float* y, const float* a, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] += a[i];
}

// One block per row: the first index of the row's maximum -> tok[row] and
// history[pos * rows + row].
__global__ void argmax_kernel(const float* logits, int64_t V, int64_t ldl, int32_t* tok,
                              int32_t* history, const int32_t* pos_p, int64_t history_len) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* r = logits + blockIdx.x * ldl;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = r[j];
    if (v > best) {  // strictly greater: the first (lowest) index of this thread's max
      best = v;
      idx = (int)j;
    }
  }
  // ties between threads go to the lower index
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    if (idx == 0x7fffffff) idx = 0;  // an all-NaN row
    tok[blockIdx.x] = idx;
    const int pos = *pos_p;
    if (history && pos < history_len) history[(int64_t)pos * gridDim.x + blockIdx.x] = idx;
  }
}

__global__ void advance_kernel(int32_t* pos) { *pos += 1; }

int launch_status(cudaError_t e) { return e == cudaSuccess ? MTRTQ_OK : MTRTQ_ERR_CUDA; }

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
  embed_kernel<<<(unsigned)B, 256, 0, static_cast<cudaStream_t>(stream)>>>(prompt, prompt_len, next_tok,
                                                                         pos, wte, wpe, x, D, V, n_pos);
  return launch_status(cudaGetLastError());
}

int mtrtq_layernorm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                    int64_t D, float eps, void* stream) {
  if (!x || !gamma || !beta || !y || rows <= 0 || D <= 0 || rows > 2147483647) return MTRTQ_ERR_INVALID_ARG;
  layernorm_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, gamma, beta, y, D, eps);
  return launch_status(cudaGetLastError());
}

int mtrtq_decode_attention(const float* qkv, float* kcache, float* vcache, const int32_t* pos,
                           float* out, int64_t B, int64_t H, int64_t head_dim, int64_t max_ctx,
                           void* stream) {
  if (!qkv || !kcache || !vcache || !pos || !out || B <= 0 || H <= 0 || head_dim <= 0 ||
      max_ctx <= 0 || B > 65535 || H > 2147483647)
    return MTRTQ_ERR_INVALID_ARG;
  const size_t smem = (size_t)(max_ctx + head_dim) * sizeof(float);
  if (smem > 48 * 1024) return MTRTQ_ERR_INVALID_ARG;  // contexts up to ~12k positions
  attention_kernel<<<dim3((unsigned)H, (unsigned)B), 128, smem, static_cast<cudaStream_t>(stream)>>>(
      qkv, kcache, vcache, pos, out, H, head_dim, max_ctx);
  return launch_status(cudaGetLastError());
}

int mtrtq_gelu_tanh(const float* x, float* y, int64_t n, void* stream) {
  if (!x || !y || n <= 0) return MTRTQ_ERR_INVALID_ARG;
  const int64_t blocks = n / 256 + 1 < 4096 ? n / 256 + 1 : 4096;
  gelu_tanh_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  return launch_status(cudaGetLastError());
}

int mtrtq_add_inplace(float* y, const float* a, int64_t n, void* stream) {
  if (!y || !a || n <= 0) return MTRTQ_ERR_INVALID_ARG;
  const int64_t blocks = n / 256 + 1 < 4096 ? n / 256 + 1 : 4096;
  add_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, a, n);
  return launch_status(cudaGetLastError());
}

int mtrtq_argmax_rows(const float* logits, int64_t rows, int64_t V, int64_t ldl, int32_t* tok,
                      int32_t* history, const int32_t* pos, int64_t history_len, void* stream) {
  if (!logits || !tok || !pos || rows <= 0 || V <= 0 || ldl < V || rows > 65535 ||
      V > 2147483647 || (history_len > 0 && !history))
    return MTRTQ_ERR_INVALID_ARG;
  argmax_kernel<<<(unsigned)rows, 512, 0, static_cast<cudaStream_t>(stream)>>>(logits, V, ldl, tok, history,
                                                                              pos, history_len);
  return launch_status(cudaGetLastError());
}

int mtrtq_decode_advance(int32_t* pos, void* stream) {
  if (!pos) return MTRTQ_ERR_INVALID_ARG;
  advance_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(pos);
  return launch_status(cudaGetLastError());
}

}  // extern "C"
