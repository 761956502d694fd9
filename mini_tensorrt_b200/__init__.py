"""mini_tensorrt_b200 -- the reference's INT8 weight-only MatMul (MatMulQ) on B200.

Hand-written sm_100a kernels behind a C ABI (include/mtrtq.h, libmtrtq.so):
  * decode (M <= 8, and fp32 mode to M = 32): a cluster GEMV that streams the
    int8 weights with bulk async copies and multiplies them, unconverted, by
    three int8 digits of each activation on int8 warp MMAs (exact int32 sums),
    reducing the k-split in distributed shared memory;
  * small batches (bf16 mode, M <= 32): a stream-K tcgen05 kernel;
  * prefill (bf16 mode, M > 32): TMA-staged int8 weight tiles dequantized to
    bf16 and fed to tcgen05.mma with fp32 accumulators in TMEM, scale and bias
    in the epilogue;
  * fp32 mode above M = 32: a CUDA-core split-K GEMV.
The Python layer here is plumbing (device memory, streams, the registry mirror);
the library raises if libmtrtq.so is missing -- there is no CPU fallback.
"""
from ._lib import MtrtqError, lib  # noqa: F401
from .matmulq import (PackedWeight, Workspace, matmul_q8, packed_bytes, plan_info,  # noqa: F401
                      prepack_host, quantize_per_channel, read_device_status, set_option,
                      workspace_bytes)
from .registry import (DType, GraphError, KernelRegistry, Node, OpContext,  # noqa: F401
                       register_cuda_kernels, run_kernel)

__version__ = "1.0.0"
