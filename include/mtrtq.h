/*
 * mtrtq -- B200 (sm_100a) INT8 weight-only MatMul, C ABI.
 *
 * Computes the reference's MatMulQ op, C[M,N] = A[M,K] x dequant(W_q8[K,N], scale[N]),
 * with C[i,j] = scale[j] * sum_k A[i,k] * W[k,j]  (src/ops/kernels_matmul.cpp:42-74),
 * optionally followed by the bias broadcast Add (src/ops/kernels_elementwise.cpp:31-35).
 *
 * The interface replaces, for this op, the reference's CPU kernel function
 *   void matmul_q8_f32(const OpContext&)  registered as ("MatMulQ", DType::kF32)
 *   (src/ops/kernels_matmul.cpp:78-81, include/mtrt/registry.h:19-22,
 *    include/mtrt/op_context.h:13-20)
 * and adds the device launcher the CUDA backend lacks (backends/cuda/kernels.h:11-76
 * declares raw-device-pointer launchers for every other op; the CUDA executor throws
 * on MatMulQ at backends/cuda/cuda_executor.cpp:152-154).
 *
 * Conventions
 *  - Every entry point returns an int status (MTRTQ_OK == 0). None aborts or traps;
 *    mtrtq_last_error() gives a message for the calling thread's last failure.
 *  - Device pointers are plain CUDA device addresses. `stream` is a cudaStream_t
 *    passed as void* (NULL = the legacy default stream), so the header needs no
 *    CUDA include and binds from any FFI.
 *  - Launch calls never allocate: scratch lives in a caller workspace sized by
 *    mtrtq_workspace_bytes(). The workspace must be zero-filled once after it is
 *    allocated: its first 4 KiB hold split-K ticket counters, which every call
 *    leaves at zero again; the rest is per-call scratch. One workspace may serve
 *    calls of any shapes, but calls that share it must be ordered (same stream).
 *  - Matrices are row-major and contiguous unless a leading dimension is given.
 *  - No CPU fallback: without an sm_100 device the launch calls fail with
 *    MTRTQ_ERR_NO_DEVICE.
 */
#ifndef MTRTQ_H_
#define MTRTQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTRTQ_VERSION 100 /* 1.0.0 */

/* Status codes. The reference validates with MTRT_ASSERT (Debug abort, Release
 * no-op, include/mtrt/support/assert.h:21-30) and aborts on CUDA errors
 * (backends/cuda/kernels.cu:13-21); this ABI reports instead. */
enum {
  MTRTQ_OK = 0,
  MTRTQ_ERR_INVALID_ARG = 1,  /* null pointer, non-positive or too-large size, bad enum */
  MTRTQ_ERR_ALIGNMENT = 2,    /* a pointer or leading dimension breaks a stated alignment */
  MTRTQ_ERR_WORKSPACE = 3,    /* workspace smaller than mtrtq_workspace_bytes() */
  MTRTQ_ERR_NO_DEVICE = 4,    /* no CUDA device of compute capability 10.x */
  MTRTQ_ERR_CUDA = 5,         /* a CUDA runtime call or launch failed */
  MTRTQ_ERR_TIMEOUT = 6,      /* a bounded device-side wait gave up (see mtrtq_read_status) */
  MTRTQ_ERR_ZERO_SCALE = 7    /* quantization met an all-zero column (see below) */
};

/* Activation element types accepted for A. */
enum { MTRTQ_DTYPE_F32 = 0, MTRTQ_DTYPE_BF16 = 1 };

/* Arithmetic modes. The mode fixes what A is before the product; the kernel then
 * depends on the shape (mtrtq_plan_info reports it).
 *  MTRTQ_MODE_BF16: fp32 A is rounded to bf16 (round-to-nearest-even) once.
 *  MTRTQ_MODE_FP32: A keeps its fp32 value (result within 1e-4 of the reference).
 * Kernels:
 *  - decode, M <= 8 in either mode, and fp32 mode up to M = 32 (bf16 mode too when
 *    the weights are at most 8 MiB): the cluster GEMV. The int8 weights are never
 *    converted; each activation is written as three int8 digits over its CTA's k
 *    range, x = (s/127)(d0 + d1/2^7 + d2/2^14) with s the range's max |x|, which
 *    represents it to within 2^-15 s/127 (about 2^-22 of that max); int8 x int8
 *    warp MMAs accumulate exactly in int32, and the digits are combined in fp32.
 *  - 32 < M <= 64 on weights of at most 8 MiB, either mode: the mma.sync grouped
 *    GEMV over blocks of 8 tokens that share the weights, with the cluster GEMV's
 *    arithmetic.
 *  - 8 < M <= 64 (bf16 mode: <= 32) on 24M weights or more: the tensor-core digit
 *    GEMV (also mtrtq_gemv_group's kernel). A digitize kernel writes each
 *    activation row as four int8 digits, x = (s/127)(d0 + d1/2^7 + d2/2^14 +
 *    d3/2^21) with s the row's max |x| (within 2^-22 s/127); tcgen05 kind::i8 MMAs
 *    multiply the int8 weights by the digits with exact int32 sums in TMEM, and
 *    the digit sums are combined in fp32. One pass over the weights for all tokens.
 *  - bf16 mode, M <= 32 otherwise: a stream-K tcgen05 kernel; above, a tiled
 *    tcgen05 GEMM (persistent, two TMEM accumulators, when it has a 256-token tile
 *    per SM). Weights are dequantized to bf16 exactly, products accumulate in fp32
 *    in TMEM.
 *  - fp32 mode above M = 32 otherwise: a CUDA-core split-K GEMV, every product and
 *    sum fp32.
 * In every kernel the per-channel scale multiplies the finished sum, then the bias
 * is added, as in the reference (src/ops/kernels_matmul.cpp:66-73). */
enum { MTRTQ_MODE_BF16 = 0, MTRTQ_MODE_FP32 = 1 };

/* Quantize-time policy for an all-zero weight column (the reference packer divides
 * 0/0 there, tests/golden_kernel_test.cpp:166-169; numpy's packer uses scale 1,
 * python/quantize_gpt2.py:32). */
enum {
  MTRTQ_ZERO_COLUMN_REJECT = 0, /* return MTRTQ_ERR_ZERO_SCALE */
  MTRTQ_ZERO_COLUMN_ZERO = 1    /* scale 0, q 0: the bytes the reference's x86-64 build stores */
};

/* Library version (MTRTQ_VERSION of the build). */
int mtrtq_version(void);

/* Text for a status code; never NULL. */
const char* mtrtq_status_string(int status);

/* Message for the calling thread's last failing call ("" if none). */
const char* mtrtq_last_error(void);

/* ---- quantization (host) ------------------------------------------------------ */

/* Host, single-threaded. W f32 [K,N] row-major -> q int8 [K,N] row-major and
 * scale f32 [N], bit-exact with the reference packer (tests/golden_kernel_test.cpp:
 * 163-170): amax = max_k |W|, s = amax / 127.0f, q = (int8) lround(W / s).
 * zero_column_policy: MTRTQ_ZERO_COLUMN_*. */
int mtrtq_quantize_per_channel(const float* W, int64_t K, int64_t N, int8_t* q, float* scale,
                               int zero_column_policy);

/* ---- weight pre-pack ------------------------------------------------------------ */

/* Bytes of the device weight layout for a [K,N] int8 matrix:
 * N_pad x K_pad with N_pad = ceil(N/128)*128 and K_pad = ceil(K/64)*64.
 * The layout ("channel tiles of 16-k slabs"): for channel tile t (128 channels) and
 * slab s (16 consecutive k), 2048 contiguous bytes hold, for each of the 128 channels
 * in order, its 16 int8 weights. Padding is zero. Returns -1 for invalid sizes. */
int64_t mtrtq_packed_bytes(int64_t K, int64_t N);

/* Device: q_KN int8 [K,N] row-major (device memory, as the CUDA executor uploads a
 * weight, backends/cuda/cuda_executor.cpp:61-72) -> packed (device, 256-byte
 * aligned, packed_bytes >= mtrtq_packed_bytes). The int8 values are unchanged. */
int mtrtq_prepack(const int8_t* q_KN, int64_t K, int64_t N, void* packed, size_t packed_bytes,
                  void* stream);

/* Host: the same layout transform on host memory (for upload with one copy). */
int mtrtq_prepack_host(const int8_t* q_KN, int64_t K, int64_t N, void* packed,
                       size_t packed_bytes);

/* ---- the op ---------------------------------------------------------------------- */

/* Workspace bytes mtrtq_matmul needs for this problem (0 is possible). */
int64_t mtrtq_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int mode);

/* Y[M,N] (+)= ... : Y[i*ldy + j] = scale[j] * sum_k X[i*ldx + k] * W[k,j] (+ bias[j]).
 *   X       device, x_dtype elements, row stride ldx >= K (elements), 16-byte aligned
 *   packed  device, from mtrtq_prepack for the same K, N, 256-byte aligned
 *   scale   device f32 [N];  bias device f32 [N] or NULL
 *   Y       device f32, row stride ldy >= N (elements), 4-byte aligned
 *   workspace device, >= mtrtq_workspace_bytes(M,K,N,x_dtype,mode) bytes, 256-byte
 *           aligned, zero-filled once after allocation (may be NULL if that size is 0)
 * Asynchronous on `stream`. */
int mtrtq_matmul(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                 const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N,
                 int mode, void* workspace, size_t workspace_bytes, void* stream);

/* Epilogues of mtrtq_matmul_ex: what happens to t = scale[j] * sum + bias[j]. */
enum {
  MTRTQ_EPILOGUE_NONE = 0,        /* Y = t (mtrtq_matmul) */
  MTRTQ_EPILOGUE_GELU_TANH = 1,   /* Y = gelu_new(t): the int8 form of the reference's
                                     FusedMatMulBiasGeluTanh (src/ops/kernels_fused.cpp:19-59) */
  MTRTQ_EPILOGUE_ADD_RESIDUAL = 2 /* Y = residual[i*ldr + j] + t: MatMulQ + Add + the
                                     residual Add of the decoder (tools/run_gpt2.cpp:174);
                                     residual may be Y itself (in place) */
};

/* mtrtq_matmul with an epilogue fused into the kernel's store. residual (device
 * f32, row stride ldr >= N, 4-byte aligned) is read only by
 * MTRTQ_EPILOGUE_ADD_RESIDUAL. */
int mtrtq_matmul_ex(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                    const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N, int mode,
                    void* workspace, size_t workspace_bytes, int epilogue, const float* residual,
                    int64_t ldr, void* stream);

/* LayerNorm then MatMulQ in one kernel: Y = epilogue(LN(X) x dequant(W) (+ bias)),
 * LN(X)[i,k] = (X[i,k] - mean_i) * inv_i * ln_gamma[k] + ln_beta[k] with the mean and
 * the biased variance of row i over its K values and inv_i = 1 / sqrt(var_i + ln_eps)
 * (the reference's LayerNorm, src/ops/kernels_transformer.cpp:19-54, followed by its
 * MatMulQ, as the decoder runs them: tools/run_gpt2.cpp:142-143, :176-177, :188-189).
 * X is fp32; ln_gamma and ln_beta are device f32 [K]; the rest as mtrtq_matmul_ex.
 * Runs on the cluster GEMV, which computes each row's statistics in every CTA that
 * reads the row; a call that plans another kernel (mtrtq_plan_info path != 3) fails
 * with MTRTQ_ERR_INVALID_ARG, and the caller runs mtrtq_layernorm and mtrtq_matmul_ex
 * instead. The workspace arguments are accepted for symmetry and not used. */
int mtrtq_matmul_ln_ex(const float* X, int64_t ldx, const float* ln_gamma, const float* ln_beta,
                       float ln_eps, const void* packed, const float* scale, const float* bias, float* Y,
                       int64_t ldy, int64_t M, int64_t K, int64_t N, int mode, void* workspace,
                       size_t workspace_bytes, int epilogue, const float* residual, int64_t ldr,
                       void* stream);

/* The reference's op on host tensors: X [M, K] and Y [M, N] are fp32 in HOST memory
 * (contiguous), the packed weights, scale and bias are resident on the device
 * (as for mtrtq_matmul). Enqueues on `stream` the copy of X into the workspace,
 * the product (mtrtq_matmul's plan for fp32 X) into the workspace, and the copy of
 * Y back to the host. With blocking != 0 it returns after Y has arrived, as the
 * reference's CPU kernel does (src/ops/kernels_matmul.cpp:42-74); with 0 it
 * returns at once and the caller synchronizes the stream before reading Y.
 * Pinned (page-locked) X and Y let the copies run asynchronously; pageable ones
 * work but copy synchronously.
 *   workspace  device, >= mtrtq_host_workspace_bytes(M,K,N,mode) bytes, 256-byte
 *              aligned, zero-filled once after allocation. Its first part is the
 *              kernel scratch of mtrtq_matmul (at least the 4 KiB counter region,
 *              so the workspace may also serve mtrtq_matmul calls); the X and Y
 *              staging follow.
 * Calls that share a workspace must be ordered on one stream. */
int64_t mtrtq_host_workspace_bytes(int64_t M, int64_t K, int64_t N, int mode);
int mtrtq_matmul_host(const float* X, const void* packed, const float* scale, const float* bias,
                      float* Y, int64_t M, int64_t K, int64_t N, int mode, void* workspace,
                      size_t workspace_bytes, int blocking, void* stream);

/* Y = X x dequant(W) (+ bias) through the decode GEMV (CUDA cores, split-K), with
 * the same arguments and results as mtrtq_matmul on its GEMV path, but without a
 * caller workspace and without allocating anything.
 *
 * No counterpart in the reference (its CPU kernel needs no scratch). It is for
 * callers that cannot allocate device memory at call time: a host runtime whose
 * run() contract forbids allocation and whose arena was planned without room for
 * this op's scratch, a plugin living inside a framework that owns every device
 * allocation, or a real-time decode loop that must not risk the device-wide
 * synchronization an allocation can cause.
 *
 * The scratch it uses instead is a fixed device array inside the library,
 * MTRTQ_NOALLOC_SCRATCH_BYTES (8 MiB) on every GPU that loads the library, held
 * until the process exits. Problems whose split-K scratch
 * (mtrtq_workspace_bytes with MTRTQ_OPT_FORCE_PATH = 1) exceeds it are rejected
 * with MTRTQ_ERR_WORKSPACE. The first call on a device looks up that device's
 * array address (cudaGetSymbolAddress, with the device current); make that first
 * call before any stream capture. A call whose plan splits K resets the array's
 * split counters on `stream` before its kernel. All calls share the one array, so
 * calls that overlap on the GPU (different streams, or other host threads) race:
 * keep them ordered. */
#define MTRTQ_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int mtrtq_matmul_gemv_noalloc(const void* X, int x_dtype, int64_t ldx, const void* packed,
                              const float* scale, const float* bias, float* Y, int64_t ldy,
                              int64_t M, int64_t K, int64_t N, int mode, void* stream);

/* ---- a group of independent decode products in one launch ------------------------ */

/* One problem of a group: Y = X x dequant(W) (+ bias), then the epilogue, with the
 * arguments of mtrtq_matmul_ex (M <= 64; M <= 8 under MTRTQ_OPT_FORCE_PATH 5). */
typedef struct mtrtq_gemv_problem {
  const void* X;          /* [M, ldx], 16-byte aligned, the group's x_dtype */
  int64_t ldx;
  const void* packed;     /* mtrtq_prepack layout, 256-byte aligned */
  const float* scale;     /* [N] */
  const float* bias;      /* [N] or NULL */
  float* Y;               /* [M, ldy] */
  int64_t ldy;
  int64_t M, K, N;        /* 1 <= M <= 64 */
  int epilogue;           /* MTRTQ_EPILOGUE_* */
  const float* residual;  /* MTRTQ_EPILOGUE_ADD_RESIDUAL: [M, ldr] (may be Y) */
  int64_t ldr;
} mtrtq_gemv_problem;

#define MTRTQ_GROUP_MAX 16

/* Computes `count` (1..MTRTQ_GROUP_MAX) independent decode products in one
 * persistent launch of the tensor-core digit GEMV (after its digitize kernel): the
 * problems' 64-k weight units are split into equal contiguous ranges over two CTAs
 * per SM (one when a problem has more than 32 tokens), so every SM streams the same
 * bytes whatever the shapes and the launch's fixed cost is paid once. Results are
 * those of mtrtq_matmul_ex on each problem within its tolerance (int8 weights times
 * four int8 digits of each activation row, exact int32 sums), deterministic (the
 * parts of a tile cut between CTAs are added in a fixed order). Under
 * MTRTQ_OPT_FORCE_PATH 5 the group runs on the mma.sync grouped GEMV instead (M <= 8,
 * three CTAs per SM, three digits per value).
 *
 * Replaces a run of independent MatMulQ calls of the reference
 * (src/ops/kernels_matmul.cpp:42-74), such as the Q, K and V projections its KV
 * decoder issues one after another (tools/run_gpt2.cpp:142-150).
 *
 * No Y may overlap another problem's X, Y or residual. At most 1024 channel tiles
 * of 128 in all. workspace: >= mtrtq_gemv_group_workspace_bytes (enough for either
 * kernel), 256-byte aligned, zero-filled once after allocation (calls leave its
 * counters at zero; after a MTRTQ_ERR_TIMEOUT fill it again); calls sharing it must
 * be stream-ordered. Honours MTRTQ_OPT_OVERLAP_LAUNCH. */
int64_t mtrtq_gemv_group_workspace_bytes(const mtrtq_gemv_problem* problems, int count);
int mtrtq_gemv_group(const mtrtq_gemv_problem* problems, int count, int x_dtype, int mode, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ---- one MatMulQ split across the GPUs of a node -------------------------------- */

/* The op shards without changing its result: output columns are independent and k
 * partial sums add (the split the reference's tensor-parallel decoder would use).
 * Rank r holds one shard of the weights and computes it with the single-GPU
 * kernels; the exchange is this library's own kernels over peer memory (NVLink
 * P2P stores and atomics, no NCCL, no multicast):
 *   MTRTQ_SPLIT_N: rank r holds W[:, n0:n1) and scale[n0:n1) (whole 128-channel
 *     tiles, mtrtq_shard_range) and stores Y[:, n0:n1) into every rank's Y: after
 *     the call every rank's Y holds the whole product (an all-gather);
 *   MTRTQ_SPLIT_K: rank r holds W[k0:k1, :] (whole 64-k units) and the full scale,
 *     computes the scaled partial over its k range and stores it into its slot of
 *     every rank's slot buffer; every rank then sums the slots in rank order and
 *     adds the bias once (an all-reduce; identical bits on every rank).
 * Each call starts with a barrier (every rank signals every peer and waits for
 * all), so no rank overwrites a buffer a peer's earlier kernels still read. Waits
 * are bounded (about a second); one that gives up stores MTRTQ_ERR_TIMEOUT in the
 * device status word (mtrtq_read_status) and the call's exchange is skipped.
 *
 * The peer pointers in mtrtq_shard_comm must be usable from this device: another
 * process's allocation opened with mtrtq_ipc_import (or the caller's own IPC), or
 * a peer device's memory in this process with peer access enabled. */
#define MTRTQ_MAX_WORLD 8
#define MTRTQ_SHARD_FLAG_BYTES 64   /* per rank, device memory, zero-filled once */
#define MTRTQ_IPC_HANDLE_BYTES 72
enum { MTRTQ_SPLIT_N = 0, MTRTQ_SPLIT_K = 1 };

typedef struct mtrtq_shard_comm {
  int rank, world;                   /* this process's rank, 1 <= world <= 8 */
  float* y[MTRTQ_MAX_WORLD];         /* split N: every rank's Y (same M, N, ldy) */
  float* slots[MTRTQ_MAX_WORLD];     /* split K: every rank's slot buffer */
  int64_t slot_elems;                /* floats in each slot buffer (>= M * N * world) */
  unsigned* flags[MTRTQ_MAX_WORLD];  /* every rank's flag words */
  int alternating;                   /* 1: the caller's exchanges alternate between two
                                        destination buffers (and every rank sends to
                                        every peer in each); the entry barrier is then
                                        skipped: a peer's data for the previous exchange
                                        already shows it has finished reading the buffer
                                        this one writes */
} mtrtq_shard_comm;

/* mtrtq_gemv_group with its all-gather fused in (split N across the ranks): each
 * problem's Y lies in this rank's comm->y[rank] buffer (its column shard of an
 * output every rank lays out the same way), and every output element is also stored
 * at the same offset in every peer's buffer by the kernel that computes it (stores
 * over NVLink); the launch's last CTA then signals every peer and waits, bounded,
 * for their shards, so the call ends when every rank holds every rank's outputs.
 * Needs comm->alternating = 1 (no entry barrier: successive calls must alternate
 * between two output buffers) and every rank making the same calls in the same
 * order; epoch as for mtrtq_shard_allgather (0: device-counted, for CUDA graphs).
 * world = 1: mtrtq_gemv_group. Replaces the split-N step's product and all-gather
 * pair (one MatMulQ, src/ops/kernels_matmul.cpp:42-74, per rank, then the gather). */
int mtrtq_gemv_group_allgather(const mtrtq_gemv_problem* problems, int count, int x_dtype, int mode,
                               void* workspace, size_t workspace_bytes, const mtrtq_shard_comm* comm,
                               unsigned epoch, void* stream);

/* [begin, end) of `rank`'s shard of an extent (N for MTRTQ_SPLIT_N, K for
 * MTRTQ_SPLIT_K): whole 128-channel tiles or 64-k units, split as evenly as possible
 * (rank r starts at unit floor(r * units / world): later ranks take the extra ones;
 * with fewer units than ranks some shards are empty). */
int mtrtq_shard_range(int64_t extent, int split, int rank, int world, int64_t* begin, int64_t* end);
/* Bytes of one rank's slot buffer for split K; workspace of the local product. */
int64_t mtrtq_shard_slot_bytes(int64_t M, int64_t N, int world);
int64_t mtrtq_shard_workspace_bytes(int64_t M, int64_t K, int64_t N, int x_dtype, int mode, int split, int rank,
                                    int world);
/* Y (every rank) = X x dequant(W) (+ bias). X: the full [M, K] on every rank;
 * packed/scale: this rank's shard (packed as an unsplit weight of the shard's
 * shape; NULL for an empty shard); bias: the full [N] or NULL. epoch: 1 for the
 * first exchange on these flags, then +1 per exchange (every rank the same); or 0
 * for every call, and the count is kept on the device (the calls can then be
 * captured in a CUDA graph and replayed); do not mix the two on the same flags.
 * Calls on the same comm must be ordered on one stream per rank. */
int mtrtq_matmul_sharded(const void* X, int x_dtype, int64_t ldx, const void* packed, const float* scale,
                         const float* bias, float* Y, int64_t ldy, int64_t M, int64_t K, int64_t N, int mode,
                         int split, const mtrtq_shard_comm* comm, unsigned epoch, void* workspace,
                         size_t workspace_bytes, void* stream);
/* The exchange steps on their own, for callers that compute their shards
 * themselves (a tensor-parallel layer keeps column-parallel outputs sharded and
 * reduces only after the row-parallel product). Each call has the entry barrier
 * and bounded waits described above, and counts as one epoch.
 * mtrtq_shard_allgather: for each segment (rows x cols floats at `offset` from
 * the buffer base, row stride ld), this rank's part of the buffers comm->y is
 * stored into the same place of every peer's buffer; each rank passes the
 * segments it owns (at most 16), and every rank's buffer then holds all of them.
 * mtrtq_shard_allreduce: `partial` [M, N] (row stride N; best placed at this
 * rank's slot, comm->slots[rank] + mtrtq_shard_slot_offset(rank, M, N), which
 * saves a copy) goes to this rank's slot of every rank's slot buffer; then
 * Y = sum of the slots in rank order (+ bias[N]) (+ residual, which may be Y),
 * the same bits on every rank. */
typedef struct mtrtq_shard_segment {
  int64_t offset, rows, cols, ld;
} mtrtq_shard_segment;
int mtrtq_shard_allgather(const mtrtq_shard_segment* segments, int count, const mtrtq_shard_comm* comm,
                          unsigned epoch, void* stream);
int mtrtq_shard_allreduce(const float* partial, const float* bias, const float* residual, int64_t ldr, float* Y,
                          int64_t ldy, int64_t M, int64_t N, const mtrtq_shard_comm* comm, unsigned epoch,
                          void* stream);
int64_t mtrtq_shard_slot_offset(int rank, int64_t M, int64_t N);

/* Peer pointers across processes: mtrtq_ipc_export writes MTRTQ_IPC_HANDLE_BYTES
 * naming the device allocation that holds device_ptr (and the offset into it);
 * another process's mtrtq_ipc_import opens it (peer access enabled) and returns
 * the same address in its own space; mtrtq_ipc_close releases it. Set-up calls. */
int mtrtq_ipc_export(const void* device_ptr, void* handle);
int mtrtq_ipc_import(const void* handle, void** device_ptr);
int mtrtq_ipc_close(void* device_ptr);

/* ---- options and diagnostics ----------------------------------------------------- */

/* Process-wide options. Both change how a call is carried out, never its result
 * beyond fp32 summation order; the workspace size depends on them, so set them
 * before querying mtrtq_workspace_bytes. */
enum {
  MTRTQ_OPT_GEMM_A_SOURCE = 1, /* tile tcgen05 GEMM. 0 (default): the persistent
                                  kernel (one CTA per SM, two TMEM accumulators,
                                  dequantized weights in 128-byte-swizzled shared
                                  memory) when the plan has at least one 256-token
                                  tile per SM and no k split, otherwise one tile
                                  per CTA with the weights staged in TMEM;
                                  1: one tile per CTA, weights in shared memory;
                                  2: one tile per CTA, weights in TMEM;
                                  3: the persistent kernel in stream-K form (equal
                                  runs of tile x k-block iterations per CTA, cut
                                  tiles added by their last CTA), from one tile per
                                  SM, no k split */
  MTRTQ_OPT_FORCE_PATH = 2,    /* 0 (default): chosen by shape and mode (see
                                  mtrtq_plan_info). Otherwise one kernel for every
                                  call: 1 CUDA-core split-K GEMV; 2 tile tcgen05 GEMM;
                                  3 stream-K tcgen05 kernel (M <= 32); 4 cluster
                                  GEMV (M <= 64); 5 mma.sync grouped GEMV over
                                  blocks of 8 tokens (M <= 64; also makes
                                  mtrtq_gemv_group use it, for M <= 8); 6 tensor-core
                                  digit GEMV (M <= 64, mtrtq_gemv_group's default
                                  kernel). 2 and 3 need MTRTQ_MODE_BF16. A call the forced
                                  kernel cannot take fails with
                                  MTRTQ_ERR_INVALID_ARG. */
  MTRTQ_OPT_OVERLAP_LAUNCH = 3 /* 0 (default) or 1: the cluster GEMV is launched with
                                  programmatic stream serialization, so it may start
                                  while the kernel ahead of it in the stream is still
                                  running. It reads the packed weights, scales and
                                  biases early and waits for that kernel before it
                                  reads X or writes Y: set it only where the kernel
                                  ahead never writes the weights, scales or biases
                                  (for example, not right after mtrtq_prepack on the
                                  same stream). The decode-loop helpers below
                                  (embedding, LayerNorm, attention, gelu, add,
                                  argmax, next token) are then launched the same
                                  way; each waits for the kernel ahead before it
                                  touches global memory. */,
  MTRTQ_OPT_PRODUCER_LANES = 4 /* 1 (default), 2, 3 or 6: threads of the grouped
                                  GEMV (mtrtq_gemv_group) that issue its weight
                                  copies; results do not depend on it. */
};
int mtrtq_set_option(int option, int64_t value);

/* The plan mtrtq_matmul would use: info[0] path (0 CUDA-core GEMV, 1 tile GEMM,
 * 2 stream-K tcgen05 kernel, 3 cluster GEMV), [1] token rows per tile, [2] token
 * tiles, [3] channel tiles, [4] k splits (stream-K: persistent CTAs; cluster GEMV:
 * CTAs per cluster), [5] k per split. n_info >= 6. */
int mtrtq_plan_info(int64_t M, int64_t K, int64_t N, int x_dtype, int mode, int64_t* info,
                    int n_info);

/* Reads and clears the device status word the kernels set when a bounded wait gives
 * up (MTRTQ_OK or MTRTQ_ERR_TIMEOUT). Synchronizes the current device. After a
 * timeout the workspace of the failed call must be zero-filled again. */
int mtrtq_read_status(int* device_status);

/* ---- KV-cache decode loop helpers --------------------------------------------
 * The steps of the reference's KVDecoder::step (tools/run_gpt2.cpp:135-191) around
 * its MatMulQ calls, as device launches on `stream`, so that a whole decode step
 * (embedding, 12 x {LayerNorm, QKV, attention, out-proj, residual, LayerNorm, FFN-up,
 * gelu_new, FFN-down, residual}, final LayerNorm, LM head, argmax) can be captured
 * once as a CUDA graph and replayed. All sequences of the batch sit at one position
 * `*pos` (device int32), which mtrtq_decode_advance increments. fp32 throughout.
 * They return MTRTQ_ERR_INVALID_ARG or MTRTQ_ERR_CUDA (launch failure). */

/* x[b, :] = wte[tok, :] + wpe[*pos, :] (tools/run_gpt2.cpp:138-140), tok =
 * prompt[b * prompt_len + *pos] while *pos < prompt_len, else next_tok[b]. wte
 * [V, D], wpe [n_pos, D]; a position past n_pos gives zeros. */
int mtrtq_decode_embed(const int32_t* prompt, int64_t prompt_len, const int32_t* next_tok,
                       const int32_t* pos, const float* wte, const float* wpe, int64_t n_pos, float* x,
                       int64_t B, int64_t D, int64_t V, void* stream);

/* Row-wise LayerNorm, biased variance (tools/run_gpt2.cpp:113-122,
 * src/ops/kernels_transformer.cpp:19-54): y = (x - mean) / sqrt(var + eps) * gamma + beta. */
int mtrtq_layernorm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                    int64_t D, float eps, void* stream);
/* The same with rows of x ldx >= D elements apart (y stays [rows, D]). */
int mtrtq_layernorm_strided(const float* x, int64_t ldx, const float* gamma, const float* beta, float* y,
                            int64_t rows, int64_t D, float eps, void* stream);

/* Attention of each sequence's new query over its cached keys (tools/run_gpt2.cpp:
 * 143-172): qkv [B, 3*H*head_dim] rows (q | k | v); appends k and v at *pos into
 * kcache / vcache [B, max_ctx, H*head_dim]; out [B, H*head_dim] =
 * softmax(q . K^T / sqrt(head_dim)) V over positions 0..*pos per head. */
int mtrtq_decode_attention(const float* qkv, float* kcache, float* vcache, const int32_t* pos,
                           float* out, int64_t B, int64_t H, int64_t head_dim, int64_t max_ctx,
                           void* stream);

/* Prefill of a whole prompt, so that every Linear of the prompt is one MatMulQ of
 * M = B * P rows (the reference consumes the prompt one position at a time,
 * tools/run_gpt2.cpp:198-214; rows are independent in its MatMulQ, so the
 * products are the same).
 * mtrtq_prefill_embed: x [B*P, D] row b*P + i = wte[ids[b, i]] + wpe[i] (ids [B, P]).
 * mtrtq_prefill_attention: qkv [B*P, 3*H*head_dim] rows (q | k | v); writes every
 * position's k and v into kcache / vcache [B, max_ctx, H*head_dim] and out [B*P,
 * H*head_dim] = causal softmax(q . K^T / sqrt(head_dim)) V, position i over 0..i
 * (P <= 1536). */
int mtrtq_prefill_embed(const int32_t* ids, int64_t B, int64_t P, const float* wte, const float* wpe,
                        int64_t n_pos, float* x, int64_t D, int64_t V, void* stream);
int mtrtq_prefill_attention(const float* qkv, float* kcache, float* vcache, float* out, int64_t B, int64_t P,
                            int64_t H, int64_t head_dim, int64_t max_ctx, void* stream);

/* GPT-2 gelu_new (tools/run_gpt2.cpp:178-181, src/ops/kernels_gpt.cpp:44-61):
 * y = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))). y may alias x. */
int mtrtq_gelu_tanh(const float* x, float* y, int64_t n, void* stream);

/* y += a (the residual adds, tools/run_gpt2.cpp:174, :183). */
int mtrtq_add_inplace(float* y, const float* a, int64_t n, void* stream);

/* Greedy next token (tools/run_gpt2.cpp:42-47), in two launches.
 * mtrtq_argmax_rows folds the maximum of logits[r, 0..V) (row stride ldl) into
 * best[r], a 64-bit key holding the value and, among equal values, the first
 * index; best[] (device, rows entries) must be zero before the first fold.
 * mtrtq_decode_next then sets tok[r] to that index and history[*pos * rows + r]
 * too (when *pos < history_len), zeroes best[] and advances *pos by one. */
int mtrtq_argmax_rows(const float* logits, int64_t rows, int64_t V, int64_t ldl,
                      unsigned long long* best, void* stream);
int mtrtq_decode_next(unsigned long long* best, int64_t rows, int32_t* tok, int32_t* history,
                      int64_t history_len, int32_t* pos, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MTRTQ_H_ */
