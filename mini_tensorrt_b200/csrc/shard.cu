// MatMulQ split across the GPUs of one node, with the exchange done by this
// library's own kernels over peer memory (NVLink P2P loads, stores and atomics;
// no NCCL, no multicast).
//
// The op shards without changing its result: output columns are independent
// (split N) and k partial sums add (split K). Rank r computes its shard with the
// single-GPU kernels (the planner's choice for the shard's shape), then:
//   * entry: it tells every peer it has entered call `epoch` and waits until every
//     peer has too -- a peer's kernels that read the previous call's result ran
//     before its entry signal on its stream, so no buffer a peer still reads is
//     overwritten;
//   * push: one kernel stores this rank's result into every peer's buffer (split
//     N: the shard's columns of the peer's Y; split K: this rank's slot of the
//     peer's slot buffer); its last block releases one arrival on every peer's
//     data flag (gpu-scope acq_rel tickets among the blocks, then one
//     system-scope fence and a relaxed add on each peer's flag);
//   * finish: split N -- the push kernel's last block, after signalling, waits for
//     every peer's arrival, so the kernel ends when the rank holds every segment;
//     split K -- a reduce kernel waits, then sums the ranks' slots in rank order
//     (fixed, so every rank gets identical bits) and adds the bias once.
// Where the caller's destinations alternate between two buffers (comm.alternating)
// the entry barrier is skipped: a peer's data for the previous exchange already
// shows it has finished reading the buffer this one writes.
// Every wait spins on the rank's own flag with an acquire load, bounded by about
// a second of SM clock; a wait that gives up stores MTRTQ_ERR_TIMEOUT in the
// device status word and returns.
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>

#include "../../include/mtrtq.h"
#include "q8_common.cuh"
#include "q8_internal.h"

namespace mtrtq {

// abi.cu: the thread's last-error text and the current device's status word.
int report_error(int code, const char* fmt, ...);
int report_cuda_error(cudaError_t e, const char* what);
unsigned* device_status_address(int* rc);

namespace {

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void red_add_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spins until *flag >= target (bounded). Returns false (and records a timeout)
// when it gives up.
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spins (relaxed loads) until *flag >= target, then one acquire fence orders the
// caller's later reads after the arrivals it saw. Bounded: returns false (and
// records a timeout) when it gives up.
__device__ bool wait_flag(const unsigned* flag, unsigned target, unsigned* status) {
  const long long t0 = clock64();
  while ((int)(ld_relaxed_sys(flag) - target) < 0) {
    if (clock64() - t0 > kSpinLimitCycles) {
      atomicExch(status, 6u /* MTRTQ_ERR_TIMEOUT */);
      return false;
    }
  }
  fence_acq_rel_sys();
  return true;
}

// A rank's flag words: arrivals at the entry barrier and of peers' data, the push
// kernel's block tickets, and the epoch of a call whose entry wait gave up (its
// push is then skipped: no store goes to a peer that may not be there).
constexpr int kFlagEntry = kShardFlagEntry, kFlagData = kShardFlagData, kFlagTicket = kShardFlagTicket,
              kFlagAbort = kShardFlagAbort, kFlagEpoch = kShardFlagEpoch;

// The call's epoch: the caller's, or -- epoch 0 -- the rank's device-side count,
// which the entry kernel advances (so that a captured graph replays correctly).
__device__ __forceinline__ unsigned call_epoch(unsigned* own_flags, unsigned epoch) {
  return epoch != 0 ? epoch : *reinterpret_cast<volatile unsigned*>(own_flags + kFlagEpoch);
}

struct ShardPeers {
  unsigned* flags[MTRTQ_MAX_WORLD];
  float* dst[MTRTQ_MAX_WORLD];  // each rank's destination base (null: not pushed to)
};

// Pieces of a rank's result to push: segment k is the rows x cols block at
// float offset off[k] (row stride ld[k]) from the source base, and goes to the same
// offset from every peer's destination base.
constexpr int kMaxSegs = 16;
struct SegList {
  int count;
  int64_t off[kMaxSegs], rows[kMaxSegs], cols[kMaxSegs], ld[kMaxSegs];
  int64_t first[kMaxSegs + 1];  // prefix of the segments' work items
  bool vec[kMaxSegs];           // 16-byte items (off, cols, ld multiples of 4)
};

// Entry barrier: one thread signals every peer, then waits for all of them.
__global__ void shard_entry_kernel(ShardPeers peers, int rank, int world, unsigned epoch, unsigned* status) {
  if (threadIdx.x != 0) return;
  if (epoch == 0) {
    epoch = peers.flags[rank][kFlagEpoch] + 1;
    peers.flags[rank][kFlagEpoch] = epoch;
  }
  const unsigned target = epoch * (unsigned)(world - 1);
  fence_acq_rel_sys();
  for (int p = 0; p < world; ++p)
    if (p != rank) red_add_relaxed_sys(peers.flags[p] + kFlagEntry, 1u);
  if (!wait_flag(peers.flags[rank] + kFlagEntry, target, status)) peers.flags[rank][kFlagAbort] = epoch;
}

// Advances the device-side epoch where no entry barrier runs.
__global__ void shard_epoch_kernel(unsigned* own_flags) {
  if (threadIdx.x == 0) own_flags[kFlagEpoch] = own_flags[kFlagEpoch] + 1;
}

// Stores every segment of src into every peer's destination, then the last block
// to finish releases one arrival on every peer's data flag.
__global__ void shard_push_kernel(const float* src, SegList segs, ShardPeers peers, int rank, int world,
                                  unsigned epoch, bool wait_after, unsigned* status) {
  __shared__ unsigned s_ticket;
  epoch = call_epoch(peers.flags[rank], epoch);
  if (*reinterpret_cast<volatile unsigned*>(peers.flags[rank] + kFlagAbort) == epoch) return;
  const int64_t total = segs.first[segs.count];
  int k = 0;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    while (e >= segs.first[k + 1]) ++k;  // items ascend within a thread
    const int64_t i = e - segs.first[k];
    if (segs.vec[k]) {
      const int64_t c4 = segs.cols[k] / 4, r = i / c4, o = segs.off[k] + r * segs.ld[k] + (i - r * c4) * 4;
      const float4 v = *reinterpret_cast<const float4*>(src + o);
      for (int p = 0; p < world; ++p)
        if (p != rank && peers.dst[p]) *reinterpret_cast<float4*>(peers.dst[p] + o) = v;
    } else {
      const int64_t r = i / segs.cols[k], o = segs.off[k] + r * segs.ld[k] + (i - r * segs.cols[k]);
      const float v = src[o];
      for (int p = 0; p < world; ++p)
        if (p != rank && peers.dst[p]) peers.dst[p][o] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // This block's stores (observed through the barrier) are released to this
    // GPU with the ticket (gpu scope: every block runs here); the last block
    // acquires them all and releases them to the peers with one system-scope
    // fence before it signals (causality carries over from one scope to the next).
    s_ticket = ticket_acq_rel(peers.flags[rank] + kFlagTicket);
  }
  __syncthreads();
  if (threadIdx.x == 0 && s_ticket == gridDim.x - 1) {
    fence_acq_rel_sys();
    peers.flags[rank][kFlagTicket] = 0u;
    for (int p = 0; p < world; ++p)
      if (p != rank) red_add_relaxed_sys(peers.flags[p] + kFlagData, 1u);
    // All-gather: the same block then waits for every peer's data (it signalled
    // its own first, so no rank waits on one that has not signalled); the kernel
    // ends when this rank holds every segment.
    if (wait_after) wait_flag(peers.flags[rank] + kFlagData, epoch * (unsigned)(world - 1), status);
  }
}

// Split K: waits for every peer's slot, then y[m, n] = sum over ranks in rank
// order of slots[r][m][n] (+ bias[n]) (+ residual[m, n], which may be Y).
__global__ void shard_reduce_kernel(const float* slots, int64_t M, int64_t N, int world, const float* bias,
                                    const float* residual, int64_t ldr, float* Y, int64_t ldy, unsigned* own_flags,
                                    unsigned epoch, unsigned* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0)
    s_ok = world == 1 || wait_flag(own_flags + kFlagData, call_epoch(own_flags, epoch) * (unsigned)(world - 1), status)
               ? 1 : 0;
  __syncthreads();
  if (!s_ok) return;
  const int64_t total = M * N;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = e / N, n = e - m * N;
    float s = 0.0f;
    for (int r = 0; r < world; ++r) s += __ldcg(slots + (int64_t)r * total + e);
    if (bias) s = __fadd_rn(s, bias[n]);
    if (residual) s = __fadd_rn(residual[m * ldr + n], s);
    Y[m * ldy + n] = s;
  }
}

int grid_for(int64_t work, int sm_count);

// Entry barrier (unless the caller's buffers alternate), then the push of `segs`
// from src to every peer's dst base.
cudaError_t launch_exchange(const float* src, const SegList& segs, ShardPeers peers, int rank, int world,
                            unsigned epoch, unsigned* status, int sm_count, bool entry, bool wait_after,
                            cudaStream_t st) {
  if (entry) {
    shard_entry_kernel<<<1, 32, 0, st>>>(peers, rank, world, epoch, status);
  } else if (epoch == 0) {
    shard_epoch_kernel<<<1, 32, 0, st>>>(peers.flags[rank]);
  }
  // one block per SM at most: few blocks take the (same-address) tickets
  int64_t items = segs.first[segs.count];
  int grid = grid_for(items > 0 ? items : 1, sm_count);
  if (grid > sm_count) grid = sm_count;
  shard_push_kernel<<<grid, 256, 0, st>>>(src, segs, peers, rank, world, epoch, wait_after, status);
  return cudaGetLastError();
}

// Whether src and every destination base allow 16-byte accesses.
bool bases_aligned(const float* src, const float* const* bases, int world) {
  if ((uintptr_t)src % 16) return false;
  for (int p = 0; p < world; ++p)
    if (bases[p] && (uintptr_t)bases[p] % 16) return false;
  return true;
}

void seg_add(SegList& s, int64_t off, int64_t rows, int64_t cols, int64_t ld, bool base_aligned) {
  const int k = s.count++;
  s.off[k] = off;
  s.rows[k] = rows;
  s.cols[k] = cols;
  s.ld[k] = ld;
  s.vec[k] = base_aligned && off % 4 == 0 && cols % 4 == 0 && ld % 4 == 0;
  s.first[k + 1] = s.first[k] + rows * (s.vec[k] ? cols / 4 : cols);
}

int grid_for(int64_t work, int sm_count) {
  const int64_t g = (work + 255) / 256;
  const int64_t cap = (int64_t)sm_count * 4;
  return (int)(g < 1 ? 1 : g > cap ? cap : g);
}

// Imported peer allocations: the pointer handed out -> the base to close.
std::mutex g_ipc_mu;
std::map<void*, void*> g_ipc_bases;

struct IpcHandle {
  cudaIpcMemHandle_t h;
  uint64_t offset;
};
static_assert(sizeof(IpcHandle) <= MTRTQ_IPC_HANDLE_BYTES, "handle size");

}  // namespace

}  // namespace mtrtq

using namespace mtrtq;

extern "C" {

int mtrtq_shard_range(int64_t extent, int split, int rank, int world, int64_t* begin, int64_t* end) {
  if (!begin || !end || extent <= 0 || world < 1 || world > MTRTQ_MAX_WORLD || rank < 0 || rank >= world ||
      (split != MTRTQ_SPLIT_N && split != MTRTQ_SPLIT_K))
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_range: extent > 0, 1 <= world <= 8, 0 <= rank < world, split N or K");
  const int64_t q = split == MTRTQ_SPLIT_N ? kTileN : kBlockK;
  const int64_t blocks = (extent + q - 1) / q;
  const int64_t b0 = (int64_t)rank * blocks / world, b1 = (int64_t)(rank + 1) * blocks / world;
  *begin = b0 * q < extent ? b0 * q : extent;
  *end = b1 * q < extent ? b1 * q : extent;
  return MTRTQ_OK;
}

int mtrtq_ipc_export(const void* device_ptr, void* handle) {
  if (!device_ptr || !handle) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_ipc_export: null pointer");
  void* base = nullptr;
  // The allocation that holds device_ptr (a caching allocator may hand out an
  // offset into a larger block): the handle names the block, plus the offset.
  // cuMemGetAddressRange through the runtime's driver entry point (no libcuda link).
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return report_error(MTRTQ_ERR_CUDA, "mtrtq_ipc_export: cuMemGetAddressRange unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  if (get_range(&b, &sz, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_ipc_export: not a device allocation");
  base = reinterpret_cast<void*>(b);
  IpcHandle h;
  if (cudaError_t e = cudaIpcGetMemHandle(&h.h, base)) return report_cuda_error(e, "cudaIpcGetMemHandle");
  h.offset = static_cast<uint64_t>(static_cast<const char*>(device_ptr) - static_cast<const char*>(base));
  *static_cast<IpcHandle*>(handle) = h;
  return MTRTQ_OK;
}

int mtrtq_ipc_import(const void* handle, void** device_ptr) {
  if (!handle || !device_ptr) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_ipc_import: null pointer");
  IpcHandle h = *static_cast<const IpcHandle*>(handle);
  void* base = nullptr;
  if (cudaError_t e = cudaIpcOpenMemHandle(&base, h.h, cudaIpcMemLazyEnablePeerAccess))
    return report_cuda_error(e, "cudaIpcOpenMemHandle");
  void* p = static_cast<char*>(base) + h.offset;
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  g_ipc_bases[p] = base;
  *device_ptr = p;
  return MTRTQ_OK;
}

int mtrtq_ipc_close(void* device_ptr) {
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    auto it = g_ipc_bases.find(device_ptr);
    if (it == g_ipc_bases.end()) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_ipc_close: not an imported pointer");
    base = it->second;
    g_ipc_bases.erase(it);
  }
  if (cudaError_t e = cudaIpcCloseMemHandle(base)) return report_cuda_error(e, "cudaIpcCloseMemHandle");
  return MTRTQ_OK;
}

int64_t mtrtq_shard_slot_bytes(int64_t M, int64_t N, int world) {
  if (M <= 0 || N <= 0 || world < 1 || world > MTRTQ_MAX_WORLD) return -1;
  return M * N * world * (int64_t)sizeof(float);
}

int64_t mtrtq_shard_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int mode, int split, int rank,
                                    int world) {
  int64_t b = 0, e = 0;
  if (mtrtq_shard_range(split == MTRTQ_SPLIT_N ? N : K, split, rank, world, &b, &e) != MTRTQ_OK) return -1;
  if (e <= b) return 0;
  return split == MTRTQ_SPLIT_N ? mtrtq_workspace_bytes(M, K, e - b, x_dtype, mode)
                                : mtrtq_workspace_bytes(M, e - b, N, x_dtype, mode);
}

// Checks a comm; *sm_count and *status receive the device's SM count and status word.
static int check_comm(const mtrtq_shard_comm* comm, unsigned epoch, int* sm_count, unsigned** status) {
  if (!comm) return report_error(MTRTQ_ERR_INVALID_ARG, "null comm");
  if (comm->world < 1 || comm->world > MTRTQ_MAX_WORLD || comm->rank < 0 || comm->rank >= comm->world)
    return report_error(MTRTQ_ERR_INVALID_ARG, "1 <= world <= 8 and 0 <= rank < world");
  for (int p = 0; p < comm->world; ++p)
    if (!comm->flags[p]) return report_error(MTRTQ_ERR_INVALID_ARG, "every rank's flags are needed");
  int rc = 0;
  *status = device_status_address(&rc);
  if (rc) return rc;
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return report_cuda_error(e, "cudaGetDevice");
  if (cudaError_t e = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, dev))
    return report_cuda_error(e, "cudaDeviceGetAttribute");
  return MTRTQ_OK;
}

static ShardPeers peers_of(const mtrtq_shard_comm* comm, float* const* bases, int64_t base_offset) {
  ShardPeers peers;
  for (int p = 0; p < MTRTQ_MAX_WORLD; ++p) {
    peers.flags[p] = p < comm->world ? comm->flags[p] : nullptr;
    peers.dst[p] = (p < comm->world && p != comm->rank && bases[p]) ? bases[p] + base_offset : nullptr;
  }
  return peers;
}

// Split K's second half: every rank's slot r of `slots` holds rank r's partial
// [M, N]; this rank's is pushed to every peer, then Y = sum in rank order
// (+ bias) (+ residual).
static int exchange_reduce(const mtrtq_shard_comm* comm, unsigned epoch, int64_t M, int64_t N, const float* bias,
                           const float* residual, int64_t ldr, float* Y, int64_t ldy, int sm_count, unsigned* status,
                           cudaStream_t st) {
  const int rank = comm->rank, world = comm->world;
  if (world > 1) {
    SegList segs = {};
    seg_add(segs, (int64_t)rank * M * N, 1, M * N, M * N, bases_aligned(comm->slots[rank], comm->slots, world));
    if (cudaError_t er = launch_exchange(comm->slots[rank], segs, peers_of(comm, comm->slots, 0), rank, world, epoch,
                                         status, sm_count, !comm->alternating, false, st))
      return report_cuda_error(er, "shard exchange launch");
  }
  shard_reduce_kernel<<<grid_for(M * N, sm_count), 256, 0, st>>>(comm->slots[rank], M, N, world, bias, residual, ldr,
                                                                 Y, ldy, comm->flags[rank], epoch, status);
  if (cudaError_t er = cudaGetLastError()) return report_cuda_error(er, "shard reduce launch");
  return MTRTQ_OK;
}

int mtrtq_matmul_sharded(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                         const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N, int mode,
                         int split, const mtrtq_shard_comm* comm, unsigned epoch, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!X || !Y) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: null pointer");
  if (split != MTRTQ_SPLIT_N && split != MTRTQ_SPLIT_K)
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: split is MTRTQ_SPLIT_N or MTRTQ_SPLIT_K");
  if (M <= 0 || K <= 0 || N <= 0 || ldx < K || ldy < N)
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: positive sizes, ldx >= K, ldy >= N");
  int sm_count = 0;
  unsigned* status = nullptr;
  if (!comm) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: null comm");
  const int rank = comm->rank, world = comm->world;
  if (world >= 1 && world <= MTRTQ_MAX_WORLD && rank >= 0 && rank < world) {
    if (split == MTRTQ_SPLIT_N) {
      for (int p = 0; p < world; ++p)
        if (p != rank && !comm->y[p])
          return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: split N needs every peer's Y");
    } else {
      for (int p = 0; p < world; ++p)
        if (!comm->slots[p])
          return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: split K needs every rank's slots");
      if (comm->slot_elems < M * N * world)
        return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: slot buffers hold %lld floats < M*N*world",
                            (long long)comm->slot_elems);
    }
  }
  if (int rc = check_comm(comm, epoch, &sm_count, &status)) return rc;
  int64_t b = 0, e = 0;
  mtrtq_shard_range(split == MTRTQ_SPLIT_N ? N : K, split, rank, world, &b, &e);
  if (!packed && e > b) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_matmul_sharded: this rank's shard is not empty");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t esz = x_dtype == MTRTQ_DTYPE_BF16 ? 2 : 4;

  if (split == MTRTQ_SPLIT_N) {
    // the shard's columns of Y, then those columns to every peer's Y
    if (e > b) {
      if (int rc = mtrtq_matmul(X, x_dtype, ldx, packed, scale, bias ? bias + b : nullptr, Y + b, ldy, M, K, e - b,
                                mode, workspace, workspace_bytes, stream))
        return rc;
    }
    if (world == 1) return MTRTQ_OK;
    SegList segs = {};
    seg_add(segs, b, e > b ? M : 0, e - b, ldy, bases_aligned(Y, comm->y, world));
    if (cudaError_t er = launch_exchange(Y, segs, peers_of(comm, comm->y, 0), rank, world, epoch, status, sm_count,
                                         !comm->alternating, true, st))
      return report_cuda_error(er, "shard exchange launch");
    return MTRTQ_OK;
  }
  // split K: the scaled partial over this rank's k range into its own slot
  float* local = comm->slots[rank] + (int64_t)rank * M * N;
  if (e > b) {
    if (int rc = mtrtq_matmul(static_cast<const char*>(X) + b * esz, x_dtype, ldx, packed, scale, nullptr, local, N,
                              M, e - b, N, mode, workspace, workspace_bytes, stream))
      return rc;
  } else if (cudaError_t er = cudaMemsetAsync(local, 0, (size_t)(M * N) * sizeof(float), st)) {
    return report_cuda_error(er, "clear an empty shard's partial");
  }
  return exchange_reduce(comm, epoch, M, N, bias, nullptr, 0, Y, ldy, sm_count, status, st);
}

int mtrtq_shard_allgather(const mtrtq_shard_segment* segments, int count, const mtrtq_shard_comm* comm,
                          unsigned epoch, void* stream) {
  if (!segments || count < 0 || count > kMaxSegs)
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allgather: 0 to %d segments", kMaxSegs);
  int sm_count = 0;
  unsigned* status = nullptr;
  if (int rc = check_comm(comm, epoch, &sm_count, &status)) return rc;
  for (int p = 0; p < comm->world; ++p)
    if (!comm->y[p]) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allgather: every rank's buffer is needed");
  SegList segs = {};
  for (int k = 0; k < count; ++k) {
    const mtrtq_shard_segment& g = segments[k];
    if (g.offset < 0 || g.rows < 0 || g.cols < 0 || (g.rows > 1 && g.ld < g.cols))
      return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allgather: segment %d: offset, rows, cols >= 0, ld >= cols", k);
    seg_add(segs, g.offset, g.rows, g.cols, g.rows > 1 ? g.ld : g.cols,
            bases_aligned(comm->y[comm->rank], comm->y, comm->world));
  }
  if (comm->world == 1) return MTRTQ_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaError_t er = launch_exchange(comm->y[comm->rank], segs, peers_of(comm, comm->y, 0), comm->rank, comm->world,
                                       epoch, status, sm_count, !comm->alternating, true, st))
    return report_cuda_error(er, "shard exchange launch");
  return MTRTQ_OK;
}

int mtrtq_shard_allreduce(const float* partial, const float* bias, const float* residual, int64_t ldr, float* Y,
                          int64_t ldy, int64_t M, int64_t N, const mtrtq_shard_comm* comm, unsigned epoch,
                          void* stream) {
  if (!partial || !Y || M <= 0 || N <= 0 || ldy < N || (residual && ldr < N))
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allreduce: pointers, positive sizes, ldy, ldr >= N");
  int sm_count = 0;
  unsigned* status = nullptr;
  if (int rc = check_comm(comm, epoch, &sm_count, &status)) return rc;
  for (int p = 0; p < comm->world; ++p)
    if (!comm->slots[p]) return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allreduce: every rank's slots are needed");
  if (comm->slot_elems < M * N * comm->world)
    return report_error(MTRTQ_ERR_INVALID_ARG, "mtrtq_shard_allreduce: slot buffers hold %lld floats < M*N*world",
                        (long long)comm->slot_elems);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* local = comm->slots[comm->rank] + (int64_t)comm->rank * M * N;
  if (partial != local) {
    if (cudaError_t er = cudaMemcpyAsync(local, partial, (size_t)(M * N) * sizeof(float), cudaMemcpyDeviceToDevice, st))
      return report_cuda_error(er, "copy the partial into this rank's slot");
  }
  return exchange_reduce(comm, epoch, M, N, bias, residual, ldr, Y, ldy, sm_count, status, st);
}

int64_t mtrtq_shard_slot_offset(int rank, int64_t M, int64_t N) {
  if (rank < 0 || rank >= MTRTQ_MAX_WORLD || M <= 0 || N <= 0) return -1;
  return (int64_t)rank * M * N;
}

}  // extern "C"
