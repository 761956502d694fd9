// Host-side declarations shared by the launch files and the C ABI (abi.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mtrtq {

// What a MatMulQ call does with t = (acc * scale) + bias before it stores it:
//  kind 0: y = t;
//  kind 1: y = gelu_new(t), the reference's FusedMatMulBiasGeluTanh activation
//          (src/ops/kernels_fused.cpp:46-57);
//  kind 2: y = residual[m, n] + t, the decoder's residual add (tools/run_gpt2.cpp:174).
// residual may be Y itself: each element is read and written by the same thread.
struct Epilogue {
  int kind = 0;
  const float* residual = nullptr;
  int64_t ldr = 0;
};

// How one mtrtq_matmul call is carried out; computed by plan_matmul() from the
// problem alone (and the device's SM count), so the workspace query and the
// launch always agree.
struct Plan {
  enum Kind { kGemv = 0, kGemmTC = 1, kSkinnyTC = 2, kGemvCluster = 3, kGemvStream = 4, kGemvTC = 5 } kind = kGemv;
  int64_t M = 0, K = 0, N = 0;
  int64_t n_pad = 0, k_pad = 0;    // packed weight extents
  int n_tiles = 0;                 // channel tiles of 128
  int m_tiles = 0;                 // token tiles (GEMV: chunks of 8 rows)
  int tile_m = 0;                  // tokens per tile (GEMV: 8; GEMM: 16..256)
  int splits = 1;                  // k splits
  int kunits = 0;                  // k units (GEMV: slabs of 16; GEMM: blocks of 64)
  int kunits_per_split = 0;
  int chunk_units = 0;             // GEMV: slabs of activations staged at a time
  int grid = 0;                    // stream-K kernel: persistent CTAs
  int stages = 0;                  // cluster GEMV: shared memory ring stages
  bool x_to_bf16 = false;          // GEMM: X is staged as a bf16 copy in the workspace
  bool round_x = false;            // GEMV: round fp32 X to bf16 before the product
  bool persistent = false;         // GEMM: one CTA per SM over the tiles (grid CTAs), two accumulators
  bool stream_k = false;           // persistent GEMM: equal runs of (tile, k-block) iterations per CTA
  // workspace layout (byte offsets)
  size_t off_counters = 0, off_partials = 0, off_xb = 0, total = 0;
  int64_t ldxb = 0;                // row stride (elements) of the bf16 X copy
};

// GEMV weight loads in flight per thread (16-byte slabs); the activation
// staging chunk is a multiple of it.
constexpr int kGemvUnroll = 8;

// Cluster GEMV: the most activation rows (tokens) it takes.
constexpr int kGemvClMaxM = 64;

struct DeviceInfo {
  int device = -1;
  int sm_count = 148;
  int major = 0, minor = 0;
  size_t smem_optin = 0;
  unsigned* status = nullptr;  // this device's g_device_status (bounded-wait errors)
};

// Raises a kernel's dynamic shared memory limit to `bytes` on the current device,
// once per (device, kernel); later calls only look the pair up.
cudaError_t ensure_smem_limit(const void* kernel, int bytes);
// Asks for the largest shared memory carveout for a small kernel that runs
// between (or overlapped with) kernels using most of an SM's shared memory, so that
// an SM running it need not change its L1 / shared memory split before their next
// CTA can start there. Once per (device, kernel).
cudaError_t ensure_max_carveout(const void* kernel);

// Persistent grouped decode GEMV (gemv_stream.cu): up to kGroupMax independent
// problems of M <= 8 tokens in one launch, their 64-k weight units split evenly
// over kSCtasPerSm CTAs per SM.
constexpr int kGroupMax = 16;
constexpr int kSChunk = 12;       // units whose activation digits are staged together
constexpr int kSStages = 6;       // ring stages of 8 KiB
constexpr int kSCtasPerSm = 3;
constexpr size_t kStreamSmemBytes = (size_t)kSStages * 8192 + 2 * kSStages * 8 + 3 * (size_t)kSChunk * 8 * 64;
constexpr size_t kStreamCounterBytes = 4096;  // tickets: one per tile of the group
constexpr int kStreamMaxTiles = (int)(kStreamCounterBytes / 4);

struct GroupProblem {
  const void* X;
  int64_t ldx;
  const char* W;        // packed weights
  const float* scale;
  const float* bias;
  float* Y;
  int64_t ldy;
  Epilogue epi;
  int M, K, N;
  int KB;               // 64-k units per tile
  int n_tiles;
  int tile_begin;       // first ticket of this problem
  int64_t unit_begin;   // first unit of this problem in the group's unit list
};

// Workspace of a group launch: tickets, then [grid][2][8][128] fp32 partials.
inline size_t gemv_stream_workspace_bytes(int grid) {
  return kStreamCounterBytes + (size_t)grid * 2 * 8 * 128 * sizeof(float);
}
cudaError_t launch_gemv_stream(const GroupProblem* probs, int count, int64_t units, int grid, int x_dtype,
                               bool round_x, void* workspace, unsigned* status, bool pdl, int producers,
                               cudaStream_t st);

// A rank's flag words in peer-memory exchanges (shard.cu, and the digit GEMV's
// fused all-gather): arrivals at the entry barrier and of peers' data, the
// last-block ticket, the epoch of a call whose entry wait gave up, and the
// device-side call count (epoch 0).
constexpr int kShardFlagEntry = 0, kShardFlagData = 1, kShardFlagTicket = 2, kShardFlagAbort = 3,
              kShardFlagEpoch = 4;
constexpr int kShardMaxWorld = 8;

// The fused all-gather of a digit GEMV group: every output element is also stored
// at the same byte offset from each peer's output base; the last CTA then signals
// every peer's data flag and waits for theirs. world <= 1: no exchange.
struct TcExchange {
  int world = 1, rank = 0;
  const char* own_base = nullptr;           // this rank's output buffer
  char* peer_base[kShardMaxWorld] = {};     // each rank's output buffer (mapped here)
  unsigned* flags[kShardMaxWorld] = {};     // each rank's flag words
  unsigned epoch = 0;                       // 0: device-counted (advanced by the digitize kernel)
};

// Tensor-core digit GEMV (gemv_tc.cu): up to kGroupMax independent problems of
// M <= kTcMaxTokens tokens in one persistent launch, one CTA per SM, each CTA a
// contiguous range of the group's 64-k weight units as in the grouped GEMV. A
// digitize kernel first writes four int8 digits of every activation (per token,
// scaled by the row's max |x|) in the MMA's operand layout; tcgen05 kind::i8 MMAs
// then multiply the weight units, straight from the shared memory ring, by the
// digits into s32 accumulators in tensor memory.
constexpr int kTcMaxTokens = 64;
// Tokens per launch (the MMA's N is four digits x this): the smallest of 8, 16,
// 32 and 64 that holds the largest M of the group.
inline int gemv_tc_tokens(int max_m) { return max_m <= 8 ? 8 : max_m <= 16 ? 16 : max_m <= 32 ? 32 : 64; }
// CTAs per SM: two (each with half the shared memory ring and 256 TMEM columns)
// up to 32 tokens, one at 64 (its two 256-column accumulators fill TMEM).
inline int gemv_tc_ctas_per_sm(int nt) { return nt == 64 ? 1 : 2; }
// Persistent CTAs: at most gemv_tc_ctas_per_sm per SM, and none with fewer than
// four 64-k units (fewer parts for a small problem's cut tiles to add).
inline int gemv_tc_grid(int64_t units, int sm_count, int nt) {
  const int64_t by_units = (units + 3) / 4;
  const int64_t slots = (int64_t)sm_count * gemv_tc_ctas_per_sm(nt);
  return (int)(by_units < slots ? by_units : slots);
}
// Workspace: tickets | per-token scales [kGroupMax][64] | [grid][2][nt][128] fp32
// partials | each problem's digits, KB units of 256 * nt bytes.
struct TcLayout {
  size_t off_scales = 0, off_partials = 0, off_digits = 0, total = 0;
};
inline TcLayout gemv_tc_layout(const GroupProblem* probs, int count, int grid, int nt) {
  TcLayout l;
  l.off_scales = kStreamCounterBytes;
  l.off_partials = l.off_scales + (size_t)kGroupMax * kTcMaxTokens * sizeof(float);
  l.off_digits = l.off_partials + (((size_t)grid * 2 * nt * 128 * sizeof(float) + 255) & ~(size_t)255);
  size_t d = 0;
  for (int i = 0; i < count; ++i) d += (size_t)probs[i].KB * 256 * nt;
  l.total = l.off_digits + d;
  return l;
}
// ln_gamma non-null (one problem, fp32 X): each row of X is layer-normalized
// (ln_gamma, ln_beta, ln_eps) before the product.
cudaError_t launch_gemv_tc(const GroupProblem* probs, int count, int64_t units, int grid, int nt, int x_dtype,
                           bool round_x, void* workspace, unsigned* status, bool pdl, cudaStream_t st,
                           const float* ln_gamma = nullptr, const float* ln_beta = nullptr,
                           float ln_eps = 0.0f, const TcExchange* xc = nullptr);

// Cluster GEMV: CTAs resident per SM (registers are capped to allow it) and the
// shared memory a CTA may use so that they fit, for M <= 8 and for larger M (more
// accumulators: fewer, larger CTAs); the most ring stages.
constexpr int kGemvClCtasPerSm = 3;
constexpr size_t kGemvClSmemCap = 72 * 1024;  // 3 x (72 + static + 1 reserved) KiB <= 228 KiB
constexpr int kGemvClCtasPerSmWide = 2;     // 8 < M <= 32
constexpr size_t kGemvClSmemCapWide = 110 * 1024;
constexpr int kGemvClCtasPerSmWide8 = 1;    // 32 < M <= 64: 96 accumulator registers a thread
constexpr size_t kGemvClSmemCapWide8 = 200 * 1024;
constexpr int kGemvClMaxStages = 8;
size_t gemv_cluster_smem_bytes(int m, int64_t units, int cs, int stages);
// ln_gamma non-null: each row of X (fp32) is layer-normalized (ln_gamma,
// ln_beta, ln_eps) before the product.
cudaError_t launch_gemv_cluster(const Plan& p, const void* X, int x_dtype, int64_t ldx,
                                const void* packed, const float* scale, const float* bias, float* Y,
                                int64_t ldy, unsigned* status, bool pdl, const Epilogue& epi,
                                cudaStream_t st, const float* ln_gamma = nullptr,
                                const float* ln_beta = nullptr, float ln_eps = 0.0f);

// Launchers (return cudaError_t of the launch).
cudaError_t launch_prepack(const int8_t* q, int64_t K, int64_t N, void* packed, cudaStream_t st);
cudaError_t launch_x_to_bf16(const void* X, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                             void* Xb, int64_t ldxb, cudaStream_t st);
cudaError_t launch_gemv(const Plan& p, const void* X, int x_dtype, int64_t ldx, const void* packed,
                        const float* scale, const float* bias, float* Y, int64_t ldy,
                        void* workspace, const Epilogue& epi, cudaStream_t st);
cudaError_t launch_gemm_tc(const Plan& p, const void* Xb, int64_t ldxb, const void* packed,
                           const float* scale, const float* bias, float* Y, int64_t ldy,
                           void* workspace, const CUtensorMap& xmap, int a_from_tmem,
                           unsigned* status, const Epilogue& epi, cudaStream_t st);

cudaError_t launch_skinny_tc(const Plan& p, const float* scale, const float* bias, float* Y,
                             int64_t ldy, const void* packed, void* workspace,
                             const CUtensorMap& xmap, bool x_f32, const void* X, int64_t ldx,
                             int x_dtype, unsigned* status, const Epilogue& epi, cudaStream_t st);
// True when the stream-K kernel keeps the whole bf16 activation matrix in shared
// memory (it then reads X directly, at any stride, and needs no tensor map).
bool skinny_x_resident(int tile_m, int64_t k_pad);

// Builds the 2-D TMA descriptor for an [M, K] activation matrix with row stride
// ldx elements and box = 64 k x tile_m rows: bf16 with 128-byte swizzle
// (x_f32 = false), or fp32 without swizzle (x_f32 = true).
int make_x_tensor_map(CUtensorMap* map, const void* X, int64_t M, int64_t K, int64_t ldx,
                      int tile_m, bool x_f32 = false);

// GEMM tile sizes with a compiled kernel.
bool gemm_tile_supported(int tile_m);

}  // namespace mtrtq
