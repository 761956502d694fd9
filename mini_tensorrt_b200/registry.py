"""Host mirror of the reference's kernel interface, with the device MatMulQ behind it.

The reference binds kernels as plain functions `void fn(const OpContext&)` in a
KernelRegistry keyed by (op_type, DType of output 0) (include/mtrt/registry.h:17-40,
include/mtrt/op_context.h:13-20, src/ops/registry.cpp:7-24); MatMulQ is keyed
("MatMulQ", kF32) with inputs {A f32 [M,K], W i8 [K,N], scale f32 [N]} and one f32
output (src/ops/kernels_matmul.cpp:42-81). This module keeps those names, argument
meanings and the setup-time lookup, so a caller (an executor's plan loop,
src/runtime/executor.cpp:105-142) finds the device kernel the same way it finds
the CPU one. A and C are torch CUDA tensors, or host tensors (copied in and out
around the device product, as the reference's CPU kernel is called); W may be a
PackedWeight (pre-packed at load time, as an executor would) or a raw int8 [K,N]
tensor (packed per call).
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field

import torch

from .matmulq import PackedWeight, matmul_q8, matmul_q8_host


class DType(enum.Enum):
    """include/mtrt/dtype.h:10-14."""
    kF32 = 0
    kI32 = 1
    kI8 = 2


class GraphError(RuntimeError):
    """Setup-time error, as the reference raises (include/mtrt/graph.h:15-17)."""


@dataclass
class Node:
    """IR node: op type, tensor ids and attributes (include/mtrt/node.h:31-45).
    MatMulQ reads attrs["mode"] ("bf16" default, or "fp32") on the device."""
    op_type: str
    inputs: list = field(default_factory=list)
    outputs: list = field(default_factory=list)
    attrs: dict = field(default_factory=dict)


@dataclass
class OpContext:
    """Borrowed inputs, preallocated outputs and the node (include/mtrt/op_context.h:13-18)."""
    inputs: list
    outputs: list
    node: Node


class KernelRegistry:
    """(op_type, DType) -> kernel function; lookups happen at setup, never per step."""

    def __init__(self):
        self._table = {}

    def register_kernel(self, op_type: str, dtype: DType, fn) -> None:
        self._table[(op_type, dtype)] = fn

    def lookup(self, op_type: str, dtype: DType):
        """The kernel, or None if nothing is registered (src/ops/registry.cpp:16-19)."""
        return self._table.get((op_type, dtype))


def _require(cond: bool, msg: str) -> None:
    # The reference's MTRT_ASSERT (include/mtrt/support/assert.h:21-30) aborts in Debug;
    # the device kernel raises instead so a Python caller can recover.
    if not cond:
        raise GraphError(msg)


def matmul_q8_f32_cuda(ctx: OpContext) -> None:
    """Device MatMulQ: C[M,N] = A[M,K] x dequant(W, scale). Same preconditions as
    src/ops/kernels_matmul.cpp:43-60, checked before the launch."""
    _require(len(ctx.inputs) == 3, "MatMulQ expects A, W_int8, scale")
    _require(len(ctx.outputs) == 1, "MatMulQ expects 1 output")
    A, W, scale = ctx.inputs
    C = ctx.outputs[0]
    _require(A.dtype in (torch.float32, torch.bfloat16), "MatMulQ: A must be f32 (or bf16)")
    _require(A.dim() == 2 and C.dim() == 2, "MatMulQ ranks")
    _require(A.is_contiguous() and C.is_contiguous(), "MatMulQ requires contiguous tensors")
    mode = ctx.node.attrs.get("mode", "bf16") if ctx.node is not None else "bf16"
    if isinstance(W, PackedWeight):
        pw = W
        _require(scale is None or scale.numel() == pw.N, "MatMulQ scale must be per-column [N]")
        if scale is not None and scale.data_ptr() != pw.scale.data_ptr():
            pw = PackedWeight(pw.packed, scale.to(device=pw.packed.device, dtype=torch.float32)
                              .contiguous(), pw.K, pw.N)
    else:
        _require(W.dtype == torch.int8, "MatMulQ: W must be i8")
        _require(W.dim() == 2 and W.is_contiguous(), "MatMulQ: W must be contiguous [K, N]")
        _require(scale.numel() == W.shape[1], "MatMulQ scale must be per-column [N]")
        pw = PackedWeight.from_int8(W, scale, device=A.device if A.is_cuda else "cuda")
    M, K = A.shape
    _require(pw.K == K, "MatMulQ inner dimensions disagree")
    _require(tuple(C.shape) == (M, pw.N), "MatMulQ output shape wrong")
    _require(C.dtype == torch.float32, "MatMulQ output must be f32")
    bias = ctx.node.attrs.get("bias") if ctx.node is not None else None
    if bias is not None:
        bias = bias.to(device=pw.packed.device, dtype=torch.float32)
    if A.device.type == "cpu":
        # Host tensors, as the reference's executor hands its CPU kernel: copies in
        # and out around the device product (mtrtq_matmul_host), blocking.
        _require(C.device.type == "cpu", "MatMulQ: a host A needs a host output")
        _require(A.dtype == torch.float32, "MatMulQ: a host A must be f32")
        matmul_q8_host(A, pw, bias=bias, out=C, mode=mode)
        return
    matmul_q8(A, pw, bias=bias, out=C, mode=mode)


def register_cuda_kernels(registry: KernelRegistry) -> None:
    """Registers the device kernels of this library (MatMulQ, keyed by its f32 output)."""
    registry.register_kernel("MatMulQ", DType.kF32, matmul_q8_f32_cuda)


def run_kernel(registry: KernelRegistry, op_type: str, inputs, output, attrs=None) -> None:
    """lookup + fn(OpContext), the path the reference's golden tests take
    (tests/golden_kernel_test.cpp:18-29)."""
    fn = registry.lookup(op_type, DType.kF32)
    if fn is None:
        raise GraphError(f"no kernel for op '{op_type}'")
    node = Node(op_type=op_type, attrs=dict(attrs or {}))
    fn(OpContext(list(inputs), [output], node))
