"""mini_tensorrt_b200 -- the reference's INT8 weight-only MatMul (MatMulQ) on B200.

Hand-written sm_100a kernels behind a C ABI (include/mtrtq.h, libmtrtq.so):
  * decode GEMV (M <= 8): coalesced 128-bit int8 loads, exact int8->fp32
    conversion, packed fp32x2 FMAs, deterministic split-K;
  * prefill GEMM (M > 8): TMA-staged int8 weight tiles dequantized to bf16 and
    fed to tcgen05.mma with fp32 accumulators in TMEM, scale and bias in the
    epilogue.
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
