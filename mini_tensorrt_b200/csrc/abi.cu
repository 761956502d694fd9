// C ABI of the INT8 weight-only MatMul library (include/mtrtq.h).
//
// Argument checking mirrors the MTRT_ASSERT preconditions of the reference
// kernel (src/ops/kernels_matmul.cpp:43-60: ranks, inner dimensions, scale of
// length N) but reports a status instead of aborting. Planning (GEMV vs tcgen05
// GEMM, tile and split-K choice, workspace layout) is one pure function used by
// both mtrtq_workspace_bytes and mtrtq_matmul, so the two always agree.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>
#include <string>

#include "../../include/mtrtq.h"
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

// Device status word: a kernel whose bounded wait gives up stores
// MTRTQ_ERR_TIMEOUT here (kernels get its address as a parameter).
__device__ unsigned int g_device_status = 0;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MTRTQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Process-wide options (mtrtq_set_option).
int g_opt_gemm_a_source = 0;  // 0: automatic, 1: one tile per CTA, A in shared memory, 2: A in TMEM
int g_opt_force_path = 0;     // 0 auto, else the kernel (MTRTQ_OPT_FORCE_PATH)
int g_opt_overlap = 0;        // 1: programmatic dependent launch (MTRTQ_OPT_OVERLAP_LAUNCH)
int g_opt_producers = 1;      // grouped GEMV: bulk-copy issuing lanes (MTRTQ_OPT_PRODUCER_LANES)

std::mutex g_dev_mu;
DeviceInfo g_dev_cache[64];  // indexed by device ordinal; current_device() rejects >= 64

// Current device's properties; sm_count 148 when there is no device.
int current_device(DeviceInfo* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return fail(MTRTQ_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev_cache[dev];
  if (d.device != dev) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    d.device = dev;
    d.sm_count = prop.multiProcessorCount;
    d.major = prop.major;
    d.minor = prop.minor;
    d.smem_optin = prop.sharedMemPerBlockOptin;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_device_status);
    if (e != cudaSuccess) {
      d.device = -1;
      return cuda_fail(e, "device status address");
    }
  }
  *out = d;
  return MTRTQ_OK;
}

int sm_count_or_default() {
  DeviceInfo d;
  if (current_device(&d) == MTRTQ_OK) return d.sm_count;
  g_last_error.clear();
  return 148;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

constexpr int64_t kMaxDim = int64_t(1) << 30;
constexpr size_t kCounterBytes = 4096;                       // fixed ticket region
constexpr int64_t kMaxSplitTiles = kCounterBytes / sizeof(unsigned);
constexpr int64_t kDigitTcMinWeights = int64_t(24) << 20;  // K * N from which 8 < M <= 64 runs on it
// Weight bytes up to which bf16 calls with 8 < M <= 64 take the cluster GEMV.
constexpr int64_t kClusterWideMaxBytes = 8ll << 20;

int check_dims(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0)
    return fail(MTRTQ_ERR_INVALID_ARG, "sizes must be positive (M=%lld K=%lld N=%lld)",
                (long long)M, (long long)K, (long long)N);
  if (M > kMaxDim || K > kMaxDim || N > kMaxDim)
    return fail(MTRTQ_ERR_INVALID_ARG, "a size exceeds 2^30 (M=%lld K=%lld N=%lld)",
                (long long)M, (long long)K, (long long)N);
  const int64_t n_pad = round_up64(N, kTileN), k_pad = round_up64(K, kBlockK);
  if (n_pad > (int64_t(1) << 62) / k_pad) return fail(MTRTQ_ERR_INVALID_ARG, "K*N overflows");
  return MTRTQ_OK;
}

// Cluster GEMV geometry: one cluster of CS CTAs (CS <= 8) per 128-channel tile,
// each CTA streaming ceil(KB / CS) 64-k units through a ring of shared memory stages.
// All clusters should be resident at once (3 CTAs per SM for M <= 8, 2 up to 32, 1
// up to 64):
// CS is the largest split that keeps n_tiles * CS within that, at most KB; it
// grows, if needed, until a CTA's activation digits leave room for two stages;
// the ring then takes what the shared memory cap leaves (2 to 8 stages).
static bool gemv_cluster_plan(int64_t M, int sm_count, Plan* p) {
  if (M > kGemvClMaxM || p->n_tiles > 65535) return false;
  // One block of 8 tokens: 3 CTAs per SM; up to four: 2; up to eight: 1.
  const int tier = M <= 8 ? 0 : M <= 32 ? 1 : 2;
  const size_t cap = tier == 0 ? kGemvClSmemCap : tier == 1 ? kGemvClSmemCapWide : kGemvClSmemCapWide8;
  const int64_t KB = p->k_pad / kBlockK;
  const int64_t capacity =
      (int64_t)sm_count * (tier == 0 ? kGemvClCtasPerSm : tier == 1 ? kGemvClCtasPerSmWide : kGemvClCtasPerSmWide8);
  int64_t cs = capacity / p->n_tiles;
  if (cs > KB) cs = KB;
  if (cs > 8) cs = 8;
  if (cs < 1) cs = 1;
  while (cs < 8 && cs < KB && gemv_cluster_smem_bytes((int)M, KB, (int)cs, 2) > cap) ++cs;
  if (gemv_cluster_smem_bytes((int)M, KB, (int)cs, 2) > cap) return false;
  int stages = 2;
  while (stages < kGemvClMaxStages && stages < ceil_div64(KB, cs) &&
         gemv_cluster_smem_bytes((int)M, KB, (int)cs, stages + 1) <= cap)
    ++stages;
  p->kind = Plan::kGemvCluster;
  p->tile_m = (int)M;
  p->m_tiles = 1;
  p->kunits = (int)KB;
  p->splits = (int)cs;
  p->stages = stages;
  p->kunits_per_split = (int)ceil_div64(KB, cs);
  p->total = 0;  // no workspace
  return true;
}

// Whether M tokens in blocks of 8 over n_tiles channel tiles fit the grouped
// GEMV's tickets.
static bool stream_plan_fits(int64_t M, int64_t n_tiles) {
  return M <= 64 && ceil_div64(M, 8) * n_tiles <= kStreamMaxTiles;
}

// force_path: 0 chooses by shape and mode; 1 to 6 select a kernel (see
// MTRTQ_OPT_FORCE_PATH). Callers pass the process-wide option.
int plan_matmul(int64_t M, int64_t K, int64_t N, int x_dtype, int mode, int sm_count, Plan* out,
                int force_path) {
  if (int rc = check_dims(M, K, N)) return rc;
  if (x_dtype != MTRTQ_DTYPE_F32 && x_dtype != MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "x_dtype must be MTRTQ_DTYPE_F32 or MTRTQ_DTYPE_BF16");
  if (mode != MTRTQ_MODE_BF16 && mode != MTRTQ_MODE_FP32)
    return fail(MTRTQ_ERR_INVALID_ARG, "mode must be MTRTQ_MODE_BF16 or MTRTQ_MODE_FP32");
  if (mode == MTRTQ_MODE_FP32 && x_dtype == MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "MTRTQ_MODE_FP32 needs fp32 activations");
  Plan p;
  p.M = M;
  p.K = K;
  p.N = N;
  p.n_pad = round_up64(N, kTileN);
  p.k_pad = round_up64(K, kBlockK);
  p.n_tiles = (int)(p.n_pad / kTileN);

  // Path: M <= 64 -> the cluster GEMV when its shared memory allows (bf16 mode with
  // M > 8: small weights only);
  // otherwise bf16 mode -> stream-K tcgen05 kernel for M <= 32 (and at most
  // kMaxSplitTiles channel tiles), tile tcgen05 GEMM above; fp32 mode -> the
  // CUDA-core split-K GEMV.
  int path = 1;
  if (mode == MTRTQ_MODE_BF16) path = (M <= 32 && p.n_tiles <= kMaxSplitTiles) ? 3 : 2;
  {
    // For 8 < M <= 32 in bf16 mode the stream-K tcgen05 kernel is faster on large
    // weights (its MMAs do the 32 tokens in one pass), and the tile GEMM above; the
    // cluster GEMV stays ahead on small ones, where a call is latency-bound.
    Plan q = p;
    const bool small_w = K * N <= kClusterWideMaxBytes;
    if ((M <= 8 || mode == MTRTQ_MODE_FP32 || small_w) && gemv_cluster_plan(M, sm_count, &q)) path = 4;
    // 32 < M <= 64 on small weights: the grouped GEMV over blocks of 8 tokens
    // sharing the weights (the cluster GEMV's eight-block instance runs one CTA per
    // SM in two waves there: FFN-up 64 x 768 x 3072 + bias 15.3 us against 23.1 us).
    if (M > 32 && M <= 64 && small_w && stream_plan_fits(M, p.n_tiles)) path = 5;
    // 8 < M <= 64 (bf16 mode: <= 32) on large weights: the tensor-core digit GEMV,
    // one pass over the weights for all the tokens (B200, fp32 mode: 16 x 4096 x
    // 14336 21.5 us against 55.8 on the cluster GEMV, 32 x 768 x 50257 28.0
    // against 59.5, 64 x 14336 x 4096 61 against 304 on the CUDA-core GEMV; bf16
    // mode: 16 x 4096 x 14336 22.3 against 27.3 on the stream-K kernel). Below about
    // 25M weights the other kernels' lower fixed cost wins.
    const bool digit_tc_w = K * N >= kDigitTcMinWeights && p.n_tiles <= kStreamMaxTiles;
    if (M > 8 && digit_tc_w && M <= (mode == MTRTQ_MODE_FP32 ? kTcMaxTokens : 32)) path = 6;
  }
  if (force_path != 0) {
    if (force_path == 6 && (M > kTcMaxTokens || p.n_tiles > kStreamMaxTiles))
      return fail(MTRTQ_ERR_INVALID_ARG, "the tensor-core digit GEMV takes M <= %d and at most %d channel tiles",
                  kTcMaxTokens, kStreamMaxTiles);
    if ((force_path == 2 || force_path == 3) && mode != MTRTQ_MODE_BF16)
      return fail(MTRTQ_ERR_INVALID_ARG, "the tensor-core kernels compute in MTRTQ_MODE_BF16 only");
    if (force_path == 3 && (M > 32 || p.n_tiles > kMaxSplitTiles))
      return fail(MTRTQ_ERR_INVALID_ARG, "the stream-K kernel takes M <= 32 and N <= 131072");
    if (force_path == 5 && (M > 64 || !stream_plan_fits(M, p.n_tiles)))
      return fail(MTRTQ_ERR_INVALID_ARG, "the grouped GEMV takes M <= 64 and at most %d tiles x token blocks",
                  kStreamMaxTiles);
    if (force_path == 4) {
      Plan q = p;
      if (!gemv_cluster_plan(M, sm_count, &q))
        return fail(MTRTQ_ERR_INVALID_ARG,
                    "the cluster GEMV takes M <= 64 and at most 72 KiB (M <= 8), 110 KiB (M <= 32) "
                    "or 200 KiB (M <= 64) of shared memory per CTA");
    }
    path = force_path;
  }
  const bool gemm = path == 2;

  if (path == 4) {
    gemv_cluster_plan(M, sm_count, &p);
    p.round_x = (mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32);
    *out = p;
    return MTRTQ_OK;
  }
  if (path == 6) {
    p.kind = Plan::kGemvTC;
    p.tile_m = gemv_tc_tokens((int)M);
    p.m_tiles = 1;
    p.kunits = (int)(p.k_pad / kBlockK);
    p.kunits_per_split = p.kunits;
    const int64_t units = (int64_t)p.n_tiles * p.kunits;
    p.grid = gemv_tc_grid(units, sm_count, p.tile_m);
    p.round_x = (mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32);
    GroupProblem g;
    g.KB = p.kunits;
    p.total = gemv_tc_layout(&g, 1, p.grid, p.tile_m).total;
    *out = p;
    return MTRTQ_OK;
  }
  if (path == 5) {
    p.kind = Plan::kGemvStream;
    p.tile_m = 8;
    p.m_tiles = (int)ceil_div64(M, 8);
    p.kunits = (int)(p.k_pad / kBlockK);
    p.kunits_per_split = p.kunits;
    const int64_t units = (int64_t)p.n_tiles * p.kunits * p.m_tiles;
    const int64_t g = (int64_t)sm_count * kSCtasPerSm;
    p.grid = (int)(units < g ? units : g);
    p.round_x = (mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32);
    p.total = gemv_stream_workspace_bytes(p.grid);
    *out = p;
    return MTRTQ_OK;
  }

  if (path == 3) {
    p.kind = Plan::kSkinnyTC;
    p.tile_m = M <= 16 ? 16 : 32;
    p.m_tiles = 1;
    p.kunits = (int)(p.k_pad / kBlockK);
    p.kunits_per_split = p.kunits;
    const int64_t units = (int64_t)p.n_tiles * p.kunits;
    // One CTA per SM, but no tile shared by more than about 8 CTAs: every CTA
    // takes at least ceil(KB/8) units, which bounds the partials a tile's last
    // CTA has to sum.
    const int64_t min_units = ceil_div64(p.kunits, 8);
    int64_t g = units / min_units;
    if (g > sm_count) g = sm_count;
    if (g < 1) g = 1;
    p.grid = (int)g;
    p.splits = 1;
    p.ldxb = round_up64(K, 8);
    size_t off = kCounterBytes;
    p.off_counters = 0;
    p.off_partials = off;
    off += round256((size_t)p.grid * 2 * (size_t)M * kTileN * sizeof(float));
    p.off_xb = off;  // bf16 copy of X, used only when X's layout does not suit TMA
    off += round256((size_t)M * (size_t)p.ldxb * 2);
    p.total = off;
    *out = p;
    return MTRTQ_OK;
  }

  if (!gemm) {
    p.kind = Plan::kGemv;
    p.tile_m = 8;
    p.m_tiles = (int)ceil_div64(M, 8);
    if (p.m_tiles > 65535) return fail(MTRTQ_ERR_INVALID_ARG, "M too large for the GEMV path");
    p.kunits = (int)(p.k_pad / kSlabK);
    p.round_x = (mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32);
    const int64_t base = (int64_t)p.n_tiles * p.m_tiles;
    const int64_t target = (int64_t)sm_count * 6;
    int64_t splits = base < target ? ceil_div64(target, base) : 1;
    const int64_t max_by_len = p.kunits >= 4 ? p.kunits / 2 : 1;  // >= 2 slabs per split
    if (splits > max_by_len) splits = max_by_len;
    if (splits > 65535) splits = 65535;
    const int64_t sps = ceil_div64(p.kunits, splits);
    p.kunits_per_split = (int)sps;
    p.splits = (int)ceil_div64(p.kunits, sps);
    // Activations are staged in shared memory a chunk at a time: <= 32 KiB,
    // a multiple of the load unroll.
    const int mt = (int)(M < 8 ? M : 8);
    int64_t chunk = (32 * 1024) / (kSlabK * 4 * mt);
    chunk = chunk / kGemvUnroll * kGemvUnroll;
    const int64_t sps_r = round_up64(sps, kGemvUnroll);
    p.chunk_units = (int)(chunk < sps_r ? chunk : sps_r);
  } else {
    p.kind = Plan::kGemmTC;
    int tm = 256;
    if (M <= 16) tm = 16;
    else if (M <= 32) tm = 32;
    else if (M <= 64) tm = 64;
    else if (M <= 128) tm = 128;
    p.tile_m = tm;
    p.m_tiles = (int)ceil_div64(M, tm);
    if (p.n_tiles > 65535) return fail(MTRTQ_ERR_INVALID_ARG, "N too large for the GEMM path");
    p.kunits = (int)(p.k_pad / kBlockK);
    const int64_t base = (int64_t)p.n_tiles * p.m_tiles;
    const int64_t target = (int64_t)sm_count * (tm >= 256 ? 1 : 2);
    int64_t splits = base < target ? ceil_div64(target, base) : 1;
    const int64_t max_by_len = p.kunits >= 4 ? p.kunits / 2 : 1;  // >= 2 blocks per split
    if (splits > max_by_len) splits = max_by_len;
    if (splits > 65535) splits = 65535;
    const int64_t kbps = ceil_div64(p.kunits, splits);
    p.kunits_per_split = (int)kbps;
    p.splits = (int)ceil_div64(p.kunits, kbps);
    p.x_to_bf16 = (x_dtype == MTRTQ_DTYPE_F32);
    p.ldxb = round_up64(K, 8);
    // At least three 256-token tiles per SM and no k split: the persistent kernel
    // (its epilogue overlaps the next tile's MMAs; B200, M = 2048: 4096 x 14336 973
    // TFLOP/s against 868, 4096 x 11008 995 against 914), unless
    // MTRTQ_OPT_GEMM_A_SOURCE asks for a one-tile-per-CTA kernel. With fewer tiles
    // per SM the one-tile-per-CTA kernel, whose dequantized weights sit in TMEM
    // rather than shared memory, stays ahead (14336 x 4096: 1053 against 984).
    const int64_t tiles = (int64_t)p.n_tiles * p.m_tiles;
    if (tm == 256 && p.splits == 1 && tiles >= 3 * (int64_t)sm_count && g_opt_gemm_a_source == 0) {
      p.persistent = true;
      p.grid = sm_count;
    }
    if (tm == 256 && p.splits == 1 && tiles >= sm_count && g_opt_gemm_a_source == 3) {
      p.persistent = true;
      p.stream_k = true;
      p.grid = sm_count;
    }
  }

  // Split-K tickets live in a fixed region at the start of every workspace (each
  // call leaves its counters at zero). Its size is fixed so that the scratch of
  // one call (partials) never overlaps the counters of another call that shares
  // the workspace; a plan whose tiles do not fit runs unsplit.
  if (p.splits > 1 && (int64_t)p.n_tiles * p.m_tiles > kMaxSplitTiles) {
    p.splits = 1;
    p.kunits_per_split = p.kunits;
  }
  size_t off = 0;
  p.off_counters = off;
  off += kCounterBytes;
  p.off_partials = off;
  if (p.splits > 1) off += round256((size_t)p.splits * (size_t)M * (size_t)p.n_pad * sizeof(float));
  p.off_xb = off;
  if (p.x_to_bf16) off += round256((size_t)M * (size_t)p.ldxb * 2);
  if (p.stream_k) {
    // stream-K GEMM: [grid][2][256 tokens][128 channels] fp32 parts of cut tiles,
    // then one part counter per tile (its own, left at zero by each call).
    p.off_partials = off;
    off += round256((size_t)p.grid * 2 * 256 * kTileN * sizeof(float));
    p.off_counters = off;
    off += round256((size_t)p.n_tiles * p.m_tiles * sizeof(unsigned));
  }
  // A single-split GEMV needs no workspace at all.
  p.total = (p.splits > 1 || p.x_to_bf16 || p.stream_k) ? off : 0;
  *out = p;
  return MTRTQ_OK;
}

// The one problem of a single call as a group of one (the digit GEMV's launch).
GroupProblem single_problem(const Plan& p, const void* X, int64_t ldx, const void* packed, const float* scale,
                            const float* bias, float* Y, int64_t ldy, const Epilogue& epi) {
  GroupProblem g;
  g.X = X;
  g.ldx = ldx;
  g.W = static_cast<const char*>(packed);
  g.scale = scale;
  g.bias = bias;
  g.Y = Y;
  g.ldy = ldy;
  g.epi = epi;
  g.M = (int)p.M;
  g.K = (int)p.K;
  g.N = (int)p.N;
  g.KB = p.kunits;
  g.n_tiles = p.n_tiles;
  g.tile_begin = 0;
  g.unit_begin = 0;
  return g;
}

int check_device_sm100(DeviceInfo* d) {
  if (int rc = current_device(d)) return rc;
  if (d->major != 10)
    return fail(MTRTQ_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                d->device, d->major, d->minor);
  return MTRTQ_OK;
}

}  // namespace

int report_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int report_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

unsigned* device_status_address(int* rc) {
  DeviceInfo d;
  *rc = check_device_sm100(&d);
  return *rc ? nullptr : d.status;
}

// (device, kernel) pairs whose shared memory limit has been raised.
static std::mutex g_smem_mu;
static std::set<std::pair<int, const void*>> g_smem_done;

bool overlap_launch_enabled() { return g_opt_overlap != 0; }

// (device, kernel) pairs whose preferred carveout is the largest shared memory.
static std::set<std::pair<int, const void*>> g_carveout_done;

cudaError_t ensure_max_carveout(const void* kernel) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  std::lock_guard<std::mutex> lk(g_smem_mu);
  if (g_carveout_done.count({dev, kernel})) return cudaSuccess;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) g_carveout_done.insert({dev, kernel});
  return e;
}

cudaError_t ensure_smem_limit(const void* kernel, int bytes) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  std::lock_guard<std::mutex> lk(g_smem_mu);
  if (g_smem_done.count({dev, kernel})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_smem_done.insert({dev, kernel});
  return e;
}

}  // namespace mtrtq

using namespace mtrtq;

extern "C" {

int mtrtq_version(void) { return MTRTQ_VERSION; }

const char* mtrtq_status_string(int status) {
  switch (status) {
    case MTRTQ_OK: return "ok";
    case MTRTQ_ERR_INVALID_ARG: return "invalid argument";
    case MTRTQ_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
    case MTRTQ_ERR_WORKSPACE: return "workspace too small";
    case MTRTQ_ERR_NO_DEVICE: return "no sm_100 CUDA device";
    case MTRTQ_ERR_CUDA: return "CUDA error";
    case MTRTQ_ERR_TIMEOUT: return "device wait timed out";
    case MTRTQ_ERR_ZERO_SCALE: return "all-zero weight column";
    default: return "unknown status";
  }
}

const char* mtrtq_last_error(void) { return g_last_error.c_str(); }

int mtrtq_set_option(int option, int64_t value) {
  switch (option) {
    case MTRTQ_OPT_GEMM_A_SOURCE:
      if (value < 0 || value > 3) return fail(MTRTQ_ERR_INVALID_ARG, "GEMM A source is 0 to 3");
      g_opt_gemm_a_source = (int)value;
      return MTRTQ_OK;
    case MTRTQ_OPT_FORCE_PATH:
      if (value < 0 || value > 6) return fail(MTRTQ_ERR_INVALID_ARG, "path is 0 to 6");
      g_opt_force_path = (int)value;
      return MTRTQ_OK;
    case MTRTQ_OPT_OVERLAP_LAUNCH:
      if (value != 0 && value != 1) return fail(MTRTQ_ERR_INVALID_ARG, "overlap is 0 or 1");
      g_opt_overlap = (int)value;
      return MTRTQ_OK;
    case MTRTQ_OPT_PRODUCER_LANES:
      if (value != 1 && value != 2 && value != 3 && value != 6)
        return fail(MTRTQ_ERR_INVALID_ARG, "producer lanes are 1, 2, 3 or 6");
      g_opt_producers = (int)value;
      return MTRTQ_OK;
    default:
      return fail(MTRTQ_ERR_INVALID_ARG, "unknown option %d", option);
  }
}

int mtrtq_quantize_per_channel(const float* W, int64_t K, int64_t N, int8_t* q, float* scale,
                               int zero_column_policy) {
  if (!W || !q || !scale) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  if (K <= 0 || N <= 0) return fail(MTRTQ_ERR_INVALID_ARG, "K and N must be positive");
  if (zero_column_policy != MTRTQ_ZERO_COLUMN_REJECT && zero_column_policy != MTRTQ_ZERO_COLUMN_ZERO)
    return fail(MTRTQ_ERR_INVALID_ARG, "unknown zero-column policy");
  // Reference packer, tests/golden_kernel_test.cpp:163-170. The reference walks
  // column by column; this walks rows (cache-friendly for [K,N] row-major). The
  // bytes are identical: max is exact and order-free, and the division and
  // lround are per element.
  for (int64_t j = 0; j < N; ++j) scale[j] = 0.0f;  // running amax
  for (int64_t k = 0; k < K; ++k) {
    const float* row = W + k * N;
    for (int64_t j = 0; j < N; ++j) {
      const float a = std::fabs(row[j]);
      scale[j] = scale[j] < a ? a : scale[j];
    }
  }
  for (int64_t j = 0; j < N; ++j) {
    if (scale[j] == 0.0f && zero_column_policy == MTRTQ_ZERO_COLUMN_REJECT)
      return fail(MTRTQ_ERR_ZERO_SCALE, "weight column %lld is all zero", (long long)j);
  }
  for (int64_t j = 0; j < N; ++j) scale[j] = scale[j] / 127.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float* row = W + k * N;
    int8_t* qrow = q + k * N;
    for (int64_t j = 0; j < N; ++j)
      qrow[j] = scale[j] == 0.0f ? int8_t(0) : static_cast<int8_t>(std::lround(row[j] / scale[j]));
  }
  return MTRTQ_OK;
}

int64_t mtrtq_packed_bytes(int64_t K, int64_t N) {
  if (K <= 0 || N <= 0 || K > kMaxDim || N > kMaxDim) return -1;
  return round_up64(N, kTileN) * round_up64(K, kBlockK);
}

int mtrtq_prepack_host(const int8_t* q_KN, int64_t K, int64_t N, void* packed, size_t packed_bytes) {
  if (!q_KN || !packed) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  const int64_t need = mtrtq_packed_bytes(K, N);
  if (need < 0) return fail(MTRTQ_ERR_INVALID_ARG, "invalid K=%lld N=%lld", (long long)K, (long long)N);
  if ((int64_t)packed_bytes < need)
    return fail(MTRTQ_ERR_INVALID_ARG, "packed buffer %zu bytes < %lld", packed_bytes, (long long)need);
  const int64_t KS = round_up64(K, kBlockK) / kSlabK;
  const int64_t n_tiles = round_up64(N, kTileN) / kTileN;
  uint8_t* out = static_cast<uint8_t*>(packed);
  for (int64_t t = 0; t < n_tiles; ++t)
    for (int64_t s = 0; s < KS; ++s)
      for (int64_t r = 0; r < kTileN; ++r) {
        uint8_t* dst = out + ((t * KS + s) * kTileN + r) * kSlabK;
        const int64_t n = t * kTileN + r;
        for (int b = 0; b < kSlabK; ++b) {
          const int64_t k = s * kSlabK + b;
          dst[b] = (n < N && k < K) ? static_cast<uint8_t>(q_KN[k * N + n]) : 0;
        }
      }
  return MTRTQ_OK;
}

int mtrtq_prepack(const int8_t* q_KN, int64_t K, int64_t N, void* packed, size_t packed_bytes,
                  void* stream) {
  if (!q_KN || !packed) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  const int64_t need = mtrtq_packed_bytes(K, N);
  if (need < 0) return fail(MTRTQ_ERR_INVALID_ARG, "invalid K=%lld N=%lld", (long long)K, (long long)N);
  if ((int64_t)packed_bytes < need)
    return fail(MTRTQ_ERR_INVALID_ARG, "packed buffer %zu bytes < %lld", packed_bytes, (long long)need);
  if (!aligned(packed, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "packed weights must be 256-byte aligned");
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  cudaError_t e = launch_prepack(q_KN, K, N, packed, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prepack launch");
  return MTRTQ_OK;
}

int64_t mtrtq_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int mode) {
  Plan p;
  if (plan_matmul(M, K, N, x_dtype, mode, sm_count_or_default(), &p, g_opt_force_path) != MTRTQ_OK)
    return -1;
  return (int64_t)p.total;
}

int mtrtq_matmul(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                 const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N, int mode,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return mtrtq_matmul_ex(X, x_dtype, ldx, packed, scale, bias, Y, ldy, M, K, N, mode, workspace,
                         workspace_bytes, MTRTQ_EPILOGUE_NONE, nullptr, 0, stream);
}

int mtrtq_matmul_ex(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                    const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N, int mode,
                    void* workspace, size_t workspace_bytes, int epilogue, const float* residual,
                    int64_t ldr, void* stream) {
  if (!X || !packed || !scale || !Y) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  if (epilogue != MTRTQ_EPILOGUE_NONE && epilogue != MTRTQ_EPILOGUE_GELU_TANH &&
      epilogue != MTRTQ_EPILOGUE_ADD_RESIDUAL)
    return fail(MTRTQ_ERR_INVALID_ARG, "unknown epilogue %d", epilogue);
  Epilogue epi;
  epi.kind = epilogue;
  if (epilogue == MTRTQ_EPILOGUE_ADD_RESIDUAL) {
    if (!residual) return fail(MTRTQ_ERR_INVALID_ARG, "the residual epilogue needs a residual");
    if (ldr < N) return fail(MTRTQ_ERR_INVALID_ARG, "ldr (%lld) < N (%lld)", (long long)ldr, (long long)N);
    if (!aligned(residual, 4)) return fail(MTRTQ_ERR_ALIGNMENT, "residual must be 4-byte aligned");
    epi.residual = residual;
    epi.ldr = ldr;
  }
  if (ldx < K) return fail(MTRTQ_ERR_INVALID_ARG, "ldx (%lld) < K (%lld)", (long long)ldx, (long long)K);
  if (ldy < N) return fail(MTRTQ_ERR_INVALID_ARG, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  Plan p;
  if (int rc = plan_matmul(M, K, N, x_dtype, mode, d.sm_count, &p, g_opt_force_path)) return rc;
  if (!aligned(packed, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "packed weights must be 256-byte aligned");
  if (!aligned(scale, 4) || (bias && !aligned(bias, 4)) || !aligned(Y, 4))
    return fail(MTRTQ_ERR_ALIGNMENT, "scale, bias and Y must be 4-byte aligned");
  if (!aligned(X, 16)) return fail(MTRTQ_ERR_ALIGNMENT, "X must be 16-byte aligned");
  if (p.total > 0) {
    if (!workspace || workspace_bytes < p.total)
      return fail(MTRTQ_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, p.total);
    if (!aligned(workspace, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (p.kind == Plan::kGemv) {
    e = launch_gemv(p, X, x_dtype, ldx, packed, scale, bias, Y, ldy, workspace, epi, st);
    if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
    return MTRTQ_OK;
  }
  unsigned* status = d.status;
  if (p.kind == Plan::kGemvStream) {
    // blocks of 8 tokens, each a problem of the group, all reading the same weights
    GroupProblem gp[kGroupMax];
    const size_t esz = x_dtype == MTRTQ_DTYPE_BF16 ? 2 : 4;
    int64_t units = 0;
    for (int i = 0; i < p.m_tiles; ++i) {
      GroupProblem& g = gp[i];
      const int64_t m0 = 8 * (int64_t)i;
      g.X = static_cast<const char*>(X) + m0 * ldx * esz;
      g.ldx = ldx;
      g.W = static_cast<const char*>(packed);
      g.scale = scale;
      g.bias = bias;
      g.Y = Y + m0 * ldy;
      g.ldy = ldy;
      g.epi = epi;
      if (epi.kind == MTRTQ_EPILOGUE_ADD_RESIDUAL) g.epi.residual = epi.residual + m0 * epi.ldr;
      g.M = (int)(M - m0 < 8 ? M - m0 : 8);
      g.K = (int)K;
      g.N = (int)N;
      g.KB = p.kunits;
      g.n_tiles = p.n_tiles;
      g.tile_begin = i * p.n_tiles;
      g.unit_begin = units;
      units += (int64_t)p.n_tiles * p.kunits;
    }
    e = launch_gemv_stream(gp, p.m_tiles, units, p.grid, x_dtype, p.round_x, workspace, status, g_opt_overlap != 0,
                           g_opt_producers, st);
    if (e != cudaSuccess) return cuda_fail(e, "grouped GEMV launch");
    return MTRTQ_OK;
  }
  if (p.kind == Plan::kGemvTC) {
    const GroupProblem g = single_problem(p, X, ldx, packed, scale, bias, Y, ldy, epi);
    e = launch_gemv_tc(&g, 1, (int64_t)p.n_tiles * p.kunits, p.grid, p.tile_m, x_dtype, p.round_x, workspace,
                       status, g_opt_overlap != 0, st);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMV launch");
    return MTRTQ_OK;
  }
  if (p.kind == Plan::kGemvCluster) {
    e = launch_gemv_cluster(p, X, x_dtype, ldx, packed, scale, bias, Y, ldy, status,
                            g_opt_overlap != 0, epi, st);
    if (e != cudaSuccess) return cuda_fail(e, "cluster GEMV launch");
    return MTRTQ_OK;
  }
  if (p.kind == Plan::kSkinnyTC && skinny_x_resident(p.tile_m, p.k_pad)) {
    CUtensorMap unused;
    std::memset(&unused, 0, sizeof(unused));
    e = launch_skinny_tc(p, scale, bias, Y, ldy, packed, workspace, unused, true, X, ldx, x_dtype,
                         status, epi, st);
    if (e != cudaSuccess) return cuda_fail(e, "stream-K kernel launch");
    return MTRTQ_OK;
  }
  if (p.kind == Plan::kSkinnyTC) {
    // TMA reads X directly when its row stride is a multiple of 16 bytes; fp32 X
    // is rounded to bf16 inside the kernel. Otherwise stage a bf16 copy first.
    const int esz = x_dtype == MTRTQ_DTYPE_F32 ? 4 : 2;
    const void* xsrc = X;
    int64_t ldxs = ldx;
    bool x_f32 = x_dtype == MTRTQ_DTYPE_F32;
    if ((ldx * esz) % 16 != 0) {
      void* xb = static_cast<char*>(workspace) + p.off_xb;
      e = launch_x_to_bf16(X, x_dtype, ldx, M, K, xb, p.ldxb, st);
      if (e != cudaSuccess) return cuda_fail(e, "activation staging launch");
      xsrc = xb;
      ldxs = p.ldxb;
      x_f32 = false;
    }
    CUtensorMap xmap;
    const int rc = make_x_tensor_map(&xmap, xsrc, M, K, ldxs, p.tile_m, x_f32);
    if (rc != 0) return fail(MTRTQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", rc);
    e = launch_skinny_tc(p, scale, bias, Y, ldy, packed, workspace, xmap, x_f32, xsrc, ldxs,
                         x_f32 ? MTRTQ_DTYPE_F32 : MTRTQ_DTYPE_BF16, status, epi, st);
    if (e != cudaSuccess) return cuda_fail(e, "stream-K kernel launch");
    return MTRTQ_OK;
  }
  const void* xb = X;
  int64_t ldxb = ldx;
  if (p.x_to_bf16) {
    xb = static_cast<char*>(workspace) + p.off_xb;
    ldxb = p.ldxb;
    e = launch_x_to_bf16(X, x_dtype, ldx, M, K, const_cast<void*>(xb), ldxb, st);
    if (e != cudaSuccess) return cuda_fail(e, "activation staging launch");
  } else if ((ldx * 2) % 16 != 0) {
    return fail(MTRTQ_ERR_ALIGNMENT, "bf16 X on the GEMM path needs ldx %% 8 == 0 (ldx=%lld)",
                (long long)ldx);
  }
  CUtensorMap xmap;
  const int rc = make_x_tensor_map(&xmap, xb, M, K, ldxb, p.tile_m);
  if (rc != 0) return fail(MTRTQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", rc);
  e = launch_gemm_tc(p, xb, ldxb, packed, scale, bias, Y, ldy, workspace, xmap,
                     g_opt_gemm_a_source == 1 ? 0 : 1, status, epi, st);
  if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
  return MTRTQ_OK;
}

int mtrtq_matmul_ln_ex(const float* X, int64_t ldx, const float* ln_gamma, const float* ln_beta,
                       float ln_eps, const void* packed, const float* scale, const float* bias, float* Y,
                       int64_t ldy, int64_t M, int64_t K, int64_t N, int mode, void* workspace,
                       size_t workspace_bytes, int epilogue, const float* residual, int64_t ldr,
                       void* stream) {
  if (!X || !ln_gamma || !ln_beta || !packed || !scale || !Y)
    return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  if (epilogue != MTRTQ_EPILOGUE_NONE && epilogue != MTRTQ_EPILOGUE_GELU_TANH &&
      epilogue != MTRTQ_EPILOGUE_ADD_RESIDUAL)
    return fail(MTRTQ_ERR_INVALID_ARG, "unknown epilogue %d", epilogue);
  Epilogue epi;
  epi.kind = epilogue;
  if (epilogue == MTRTQ_EPILOGUE_ADD_RESIDUAL) {
    if (!residual) return fail(MTRTQ_ERR_INVALID_ARG, "the residual epilogue needs a residual");
    if (ldr < N) return fail(MTRTQ_ERR_INVALID_ARG, "ldr (%lld) < N (%lld)", (long long)ldr, (long long)N);
    if (!aligned(residual, 4)) return fail(MTRTQ_ERR_ALIGNMENT, "residual must be 4-byte aligned");
    epi.residual = residual;
    epi.ldr = ldr;
  }
  if (ldx < K) return fail(MTRTQ_ERR_INVALID_ARG, "ldx (%lld) < K (%lld)", (long long)ldx, (long long)K);
  if (ldy < N) return fail(MTRTQ_ERR_INVALID_ARG, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  Plan p;
  if (int rc = plan_matmul(M, K, N, MTRTQ_DTYPE_F32, mode, d.sm_count, &p, g_opt_force_path)) return rc;
  if (p.kind != Plan::kGemvCluster && p.kind != Plan::kGemvTC)
    return fail(MTRTQ_ERR_INVALID_ARG,
                "the LayerNorm prologue runs on the decode GEMVs only (M <= 64); this call plans another "
                "kernel (M=%lld K=%lld N=%lld): run mtrtq_layernorm, then mtrtq_matmul_ex",
                (long long)M, (long long)K, (long long)N);
  if (!aligned(packed, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "packed weights must be 256-byte aligned");
  if (!aligned(scale, 4) || (bias && !aligned(bias, 4)) || !aligned(Y, 4) || !aligned(ln_gamma, 4) ||
      !aligned(ln_beta, 4))
    return fail(MTRTQ_ERR_ALIGNMENT, "scale, bias, Y, gamma and beta must be 4-byte aligned");
  if (!aligned(X, 16)) return fail(MTRTQ_ERR_ALIGNMENT, "X must be 16-byte aligned");
  if (p.kind == Plan::kGemvTC) {
    if (!workspace || workspace_bytes < p.total)
      return fail(MTRTQ_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, p.total);
    if (!aligned(workspace, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
    const GroupProblem g = single_problem(p, X, ldx, packed, scale, bias, Y, ldy, epi);
    cudaError_t e = launch_gemv_tc(&g, 1, (int64_t)p.n_tiles * p.kunits, p.grid, p.tile_m, MTRTQ_DTYPE_F32,
                                   p.round_x, workspace, d.status, g_opt_overlap != 0,
                                   static_cast<cudaStream_t>(stream), ln_gamma, ln_beta, ln_eps);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMV launch");
    return MTRTQ_OK;
  }
  cudaError_t e = launch_gemv_cluster(p, X, MTRTQ_DTYPE_F32, ldx, packed, scale, bias, Y, ldy, d.status,
                                      g_opt_overlap != 0, epi, static_cast<cudaStream_t>(stream), ln_gamma,
                                      ln_beta, ln_eps);
  if (e != cudaSuccess) return cuda_fail(e, "cluster GEMV launch");
  return MTRTQ_OK;
}

// Host staging sits after the kernel scratch: X [M, K] then Y [M, N], fp32, each
// 256-byte aligned. It never starts inside the ticket-counter region, even for a
// plan without scratch: a workspace shared with other calls keeps its counters
// there, and they must stay zero.
static int host_layout(int64_t M, int64_t K, int64_t N, int mode, size_t* scratch, size_t* xbytes,
                       size_t* total) {
  Plan p;
  if (int rc = plan_matmul(M, K, N, MTRTQ_DTYPE_F32, mode, sm_count_or_default(), &p, g_opt_force_path))
    return rc;
  *scratch = std::max(round256(p.total), kCounterBytes);
  *xbytes = round256((size_t)(M * K) * sizeof(float));
  *total = *scratch + *xbytes + round256((size_t)(M * N) * sizeof(float));
  return MTRTQ_OK;
}

int64_t mtrtq_host_workspace_bytes(int64_t M, int64_t K, int64_t N, int mode) {
  size_t scratch, xbytes, total;
  if (host_layout(M, K, N, mode, &scratch, &xbytes, &total) != MTRTQ_OK) return -1;
  return (int64_t)total;
}

int mtrtq_matmul_host(const float* X, const void* packed, const float* scale, const float* bias,
                      float* Y, int64_t M, int64_t K, int64_t N, int mode, void* workspace,
                      size_t workspace_bytes, int blocking, void* stream) {
  if (!X || !Y || !workspace) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  size_t scratch, xbytes, total;
  if (int rc = host_layout(M, K, N, mode, &scratch, &xbytes, &total)) return rc;
  if (workspace_bytes < total)
    return fail(MTRTQ_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, total);
  if (!aligned(workspace, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  float* xd = reinterpret_cast<float*>(ws + scratch);
  float* yd = reinterpret_cast<float*>(ws + scratch + xbytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(xd, X, (size_t)(M * K) * sizeof(float), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return cuda_fail(e, "copy of X to the device");
  if (int rc = mtrtq_matmul_ex(xd, MTRTQ_DTYPE_F32, K, packed, scale, bias, yd, N, M, K, N, mode,
                               workspace, scratch, MTRTQ_EPILOGUE_NONE, nullptr, 0, stream))
    return rc;
  e = cudaMemcpyAsync(Y, yd, (size_t)(M * N) * sizeof(float), cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return cuda_fail(e, "copy of Y to the host");
  if (blocking) {
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
  }
  return MTRTQ_OK;
}

}  // extern "C"

namespace mtrtq {
namespace {

// Scratch of mtrtq_matmul_gemv_noalloc: split counters (first 4 KiB, zero at load)
// then split partials. Host code may not use this name as a device address; the
// address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MTRTQ_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// This device's address of g_noalloc_scratch (looked up on its first use here,
// with the device current).
int noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MTRTQ_ERR_NO_DEVICE, "device ordinal %d is outside 0..%d", dev, kMaxDevices - 1);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return MTRTQ_OK;
}

}  // namespace
}  // namespace mtrtq

extern "C" {

int mtrtq_matmul_gemv_noalloc(const void* X, int x_dtype, int64_t ldx, const void* packed,
                              const float* scale, const float* bias, float* Y, int64_t ldy,
                              int64_t M, int64_t K, int64_t N, int mode, void* stream) {
  if (!X || !packed || !scale || !Y) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  if (ldx < K) return fail(MTRTQ_ERR_INVALID_ARG, "ldx (%lld) < K (%lld)", (long long)ldx, (long long)K);
  if (ldy < N) return fail(MTRTQ_ERR_INVALID_ARG, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)N);
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  Plan p;
  if (int rc = plan_matmul(M, K, N, x_dtype, mode, d.sm_count, &p, /*force_path=*/1)) return rc;
  if (p.total > (size_t)MTRTQ_NOALLOC_SCRATCH_BYTES)
    return fail(MTRTQ_ERR_WORKSPACE,
                "problem needs %zu bytes of scratch; the no-allocation entry point holds %d",
                p.total, MTRTQ_NOALLOC_SCRATCH_BYTES);
  if (!aligned(packed, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "packed weights must be 256-byte aligned");
  if (!aligned(scale, 4) || (bias && !aligned(bias, 4)) || !aligned(Y, 4))
    return fail(MTRTQ_ERR_ALIGNMENT, "scale, bias and Y must be 4-byte aligned");
  if (!aligned(X, 16)) return fail(MTRTQ_ERR_ALIGNMENT, "X must be 16-byte aligned");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(d.device, &scratch)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Split counters must start at zero; a previous call leaves them at zero, but one
  // that gave up on a timeout may not, so clear them (memset: no allocation). A plan
  // with one split touches neither counters nor partials.
  cudaError_t e = cudaSuccess;
  if (p.splits > 1) {
    e = cudaMemsetAsync(static_cast<char*>(scratch) + p.off_counters, 0, kCounterBytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "clear no-allocation counters");
  }
  e = launch_gemv(p, X, x_dtype, ldx, packed, scale, bias, Y, ldy, scratch, Epilogue(), st);
  if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
  return MTRTQ_OK;
}

}  // extern "C"

namespace mtrtq {
namespace {

// Validates a group and lays its problems out in one unit list; *units and *tiles
// receive the totals. Device pointers are checked only when check_ptrs is set.
int group_layout(const mtrtq_gemv_problem* probs, int count, bool check_ptrs, GroupProblem* out,
                 int64_t* units, int* tiles, int max_m) {
  if (!probs) return fail(MTRTQ_ERR_INVALID_ARG, "null problem list");
  if (count < 1 || count > kGroupMax)
    return fail(MTRTQ_ERR_INVALID_ARG, "a group holds 1 to %d problems (got %d)", kGroupMax, count);
  int64_t u = 0;
  int t = 0;
  for (int i = 0; i < count; ++i) {
    const mtrtq_gemv_problem& q = probs[i];
    if (int rc = check_dims(q.M, q.K, q.N)) return rc;
    if (q.M > max_m)
      return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: a group takes M <= %d (M=%lld)", i, max_m, (long long)q.M);
    if (q.epilogue != MTRTQ_EPILOGUE_NONE && q.epilogue != MTRTQ_EPILOGUE_GELU_TANH &&
        q.epilogue != MTRTQ_EPILOGUE_ADD_RESIDUAL)
      return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: unknown epilogue %d", i, q.epilogue);
    if (check_ptrs) {
      if (!q.X || !q.packed || !q.scale || !q.Y) return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: null pointer", i);
      if (q.ldx < q.K || q.ldy < q.N)
        return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: ldx < K or ldy < N", i);
      if (!aligned(q.packed, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "problem %d: packed weights must be 256-byte aligned", i);
      if (!aligned(q.X, 16)) return fail(MTRTQ_ERR_ALIGNMENT, "problem %d: X must be 16-byte aligned", i);
      if (!aligned(q.scale, 4) || (q.bias && !aligned(q.bias, 4)) || !aligned(q.Y, 4))
        return fail(MTRTQ_ERR_ALIGNMENT, "problem %d: scale, bias and Y must be 4-byte aligned", i);
      if (q.epilogue == MTRTQ_EPILOGUE_ADD_RESIDUAL && (!q.residual || q.ldr < q.N || !aligned(q.residual, 4)))
        return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: the residual epilogue needs a residual with ldr >= N", i);
    }
    GroupProblem& g = out[i];
    g.X = q.X;
    g.ldx = q.ldx;
    g.W = static_cast<const char*>(q.packed);
    g.scale = q.scale;
    g.bias = q.bias;
    g.Y = q.Y;
    g.ldy = q.ldy;
    g.epi.kind = q.epilogue;
    g.epi.residual = q.epilogue == MTRTQ_EPILOGUE_ADD_RESIDUAL ? q.residual : nullptr;
    g.epi.ldr = q.ldr;
    g.M = (int)q.M;
    g.K = (int)q.K;
    g.N = (int)q.N;
    g.KB = (int)(round_up64(q.K, kBlockK) / kBlockK);
    g.n_tiles = (int)(round_up64(q.N, kTileN) / kTileN);
    g.tile_begin = t;
    g.unit_begin = u;
    t += g.n_tiles;
    u += (int64_t)g.n_tiles * g.KB;
    if (t > kStreamMaxTiles)
      return fail(MTRTQ_ERR_INVALID_ARG, "a group holds at most %d channel tiles of 128", kStreamMaxTiles);
  }
  *units = u;
  *tiles = t;
  return MTRTQ_OK;
}

int group_grid(int64_t units, int sm_count) {
  const int64_t g = (int64_t)sm_count * kSCtasPerSm;
  return (int)(units < g ? units : g);
}

// Groups run on the tensor-core digit GEMV (M <= 64), or on the mma.sync
// grouped GEMV (M <= 8) when MTRTQ_OPT_FORCE_PATH is 5.
bool group_on_stream_kernel() { return g_opt_force_path == 5; }
int group_max_m() { return group_on_stream_kernel() ? 8 : kTcMaxTokens; }

int group_max_tokens(const GroupProblem* gp, int count) {
  int m = 1;
  for (int i = 0; i < count; ++i) m = gp[i].M > m ? gp[i].M : m;
  return m;
}

}  // namespace
}  // namespace mtrtq

extern "C" {

int64_t mtrtq_gemv_group_workspace_bytes(const mtrtq_gemv_problem* problems, int count) {
  GroupProblem gp[kGroupMax];
  int64_t units = 0;
  int tiles = 0;
  if (group_layout(problems, count, false, gp, &units, &tiles, kTcMaxTokens) != MTRTQ_OK) return -1;
  // Enough for either kernel, so that the option may change between calls.
  const int sm = sm_count_or_default();
  const size_t a = gemv_stream_workspace_bytes(group_grid(units, sm));
  const int nt = gemv_tc_tokens(group_max_tokens(gp, count));
  const size_t b = gemv_tc_layout(gp, count, gemv_tc_grid(units, sm, nt), nt).total;
  return (int64_t)(a > b ? a : b);
}

int mtrtq_gemv_group(const mtrtq_gemv_problem* problems, int count, int x_dtype, int mode, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (x_dtype != MTRTQ_DTYPE_F32 && x_dtype != MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "x_dtype must be MTRTQ_DTYPE_F32 or MTRTQ_DTYPE_BF16");
  if (mode != MTRTQ_MODE_BF16 && mode != MTRTQ_MODE_FP32)
    return fail(MTRTQ_ERR_INVALID_ARG, "mode must be MTRTQ_MODE_BF16 or MTRTQ_MODE_FP32");
  if (mode == MTRTQ_MODE_FP32 && x_dtype == MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "MTRTQ_MODE_FP32 needs fp32 activations");
  GroupProblem gp[kGroupMax];
  int64_t units = 0;
  int tiles = 0;
  if (int rc = group_layout(problems, count, true, gp, &units, &tiles, group_max_m())) return rc;
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  const bool on_stream = group_on_stream_kernel();
  const int nt = gemv_tc_tokens(group_max_tokens(gp, count));
  const int grid = on_stream ? group_grid(units, d.sm_count) : gemv_tc_grid(units, d.sm_count, nt);
  const size_t need =
      on_stream ? gemv_stream_workspace_bytes(grid) : gemv_tc_layout(gp, count, grid, nt).total;
  if (!workspace || workspace_bytes < need)
    return fail(MTRTQ_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  const bool round_x = mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32;
  cudaError_t e =
      on_stream ? launch_gemv_stream(gp, count, units, grid, x_dtype, round_x, workspace, d.status,
                                     g_opt_overlap != 0, g_opt_producers, static_cast<cudaStream_t>(stream))
                : launch_gemv_tc(gp, count, units, grid, nt, x_dtype, round_x, workspace, d.status,
                                 g_opt_overlap != 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "grouped GEMV launch");
  return MTRTQ_OK;
}

int mtrtq_gemv_group_allgather(const mtrtq_gemv_problem* problems, int count, int x_dtype, int mode,
                               void* workspace, size_t workspace_bytes, const mtrtq_shard_comm* comm,
                               unsigned epoch, void* stream) {
  if (!comm) return fail(MTRTQ_ERR_INVALID_ARG, "null communicator");
  if (comm->world < 1 || comm->world > MTRTQ_MAX_WORLD || comm->rank < 0 || comm->rank >= comm->world)
    return fail(MTRTQ_ERR_INVALID_ARG, "rank %d / world %d out of range", comm->rank, comm->world);
  if (comm->world == 1) return mtrtq_gemv_group(problems, count, x_dtype, mode, workspace, workspace_bytes, stream);
  if (!comm->alternating)
    return fail(MTRTQ_ERR_INVALID_ARG,
                "the fused all-gather needs alternating output buffers (comm->alternating = 1): it has no entry "
                "barrier; run mtrtq_gemv_group, then mtrtq_shard_allgather");
  if (group_on_stream_kernel())
    return fail(MTRTQ_ERR_INVALID_ARG, "the fused all-gather runs on the digit GEMV (MTRTQ_OPT_FORCE_PATH 5 is set)");
  for (int r = 0; r < comm->world; ++r)
    if (!comm->y[r] || !comm->flags[r]) return fail(MTRTQ_ERR_INVALID_ARG, "rank %d: null output or flag buffer", r);
  if (x_dtype != MTRTQ_DTYPE_F32 && x_dtype != MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "x_dtype must be MTRTQ_DTYPE_F32 or MTRTQ_DTYPE_BF16");
  if (mode != MTRTQ_MODE_BF16 && mode != MTRTQ_MODE_FP32)
    return fail(MTRTQ_ERR_INVALID_ARG, "mode must be MTRTQ_MODE_BF16 or MTRTQ_MODE_FP32");
  if (mode == MTRTQ_MODE_FP32 && x_dtype == MTRTQ_DTYPE_BF16)
    return fail(MTRTQ_ERR_INVALID_ARG, "MTRTQ_MODE_FP32 needs fp32 activations");
  GroupProblem gp[kGroupMax];
  int64_t units = 0;
  int tiles = 0;
  if (int rc = group_layout(problems, count, true, gp, &units, &tiles, kTcMaxTokens)) return rc;
  for (int i = 0; i < count; ++i)
    if (reinterpret_cast<const char*>(gp[i].Y) < reinterpret_cast<const char*>(comm->y[comm->rank]))
      return fail(MTRTQ_ERR_INVALID_ARG, "problem %d: Y lies below this rank's output buffer", i);
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  const int nt = gemv_tc_tokens(group_max_tokens(gp, count));
  const int grid = gemv_tc_grid(units, d.sm_count, nt);
  const size_t need = gemv_tc_layout(gp, count, grid, nt).total;
  if (!workspace || workspace_bytes < need)
    return fail(MTRTQ_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(MTRTQ_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  TcExchange xc;
  xc.world = comm->world;
  xc.rank = comm->rank;
  xc.own_base = reinterpret_cast<const char*>(comm->y[comm->rank]);
  for (int r = 0; r < comm->world; ++r) {
    xc.peer_base[r] = reinterpret_cast<char*>(comm->y[r]);
    xc.flags[r] = comm->flags[r];
  }
  xc.epoch = epoch;
  const bool round_x = mode == MTRTQ_MODE_BF16 && x_dtype == MTRTQ_DTYPE_F32;
  cudaError_t e = launch_gemv_tc(gp, count, units, grid, nt, x_dtype, round_x, workspace, d.status,
                                 g_opt_overlap != 0, static_cast<cudaStream_t>(stream), nullptr, nullptr, 0.0f, &xc);
  if (e != cudaSuccess) return cuda_fail(e, "grouped GEMV launch (fused all-gather)");
  return MTRTQ_OK;
}

int mtrtq_plan_info(int64_t M, int64_t K, int64_t N, int x_dtype, int mode, int64_t* info, int n_info) {
  if (!info || n_info < 6) return fail(MTRTQ_ERR_INVALID_ARG, "info needs 6 slots");
  Plan p;
  if (int rc = plan_matmul(M, K, N, x_dtype, mode, sm_count_or_default(), &p, g_opt_force_path))
    return rc;
  info[0] = p.kind;  // 0 GEMV, 1 tile GEMM, 2 stream-K tcgen05, 3 cluster GEMV, 4 grouped GEMV, 5 digit tcgen05 GEMV
  info[1] = p.tile_m;
  info[2] = p.m_tiles;
  info[3] = p.n_tiles;
  info[4] = (p.kind == Plan::kSkinnyTC || p.kind == Plan::kGemvStream || p.kind == Plan::kGemvTC) ? p.grid : p.splits;
  info[5] = p.kunits_per_split * (p.kind == Plan::kGemv ? kSlabK : kBlockK);
  return MTRTQ_OK;
}

int mtrtq_read_status(int* device_status) {
  if (!device_status) return fail(MTRTQ_ERR_INVALID_ARG, "null pointer");
  DeviceInfo d;
  if (int rc = check_device_sm100(&d)) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  const unsigned zero = 0;
  e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clear device status");
  *device_status = (int)v;
  return MTRTQ_OK;
}

}  // extern "C"
