"""Torch-facing host API over the C ABI: device weight pre-pack and the MatMulQ launch.

PyTorch supplies device memory, streams and pointers here; the arithmetic is
the CUDA library's (libmtrtq.so). Nothing in this module computes on the CPU
except the host quantizer, which is the library's own C function.
"""
from __future__ import annotations

import contextlib

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

MODES = {"bf16": _lib.MODE_BF16, "fp32": _lib.MODE_FP32}


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def quantize_per_channel(W, zero_columns: str = "reject"):
    """Host quantization of W f32 [K,N] -> (q int8 [K,N], scale f32 [N]) with the
    reference packer's rule (tests/golden_kernel_test.cpp:163-170), computed by the
    library's C function. Accepts numpy arrays or CPU torch tensors; returns numpy."""
    if isinstance(W, torch.Tensor):
        W = W.detach().cpu().numpy()
    W = np.ascontiguousarray(W, dtype=np.float32)
    if W.ndim != 2:
        raise ValueError("W must be [K, N]")
    K, N = W.shape
    q = np.empty((K, N), dtype=np.int8)
    s = np.empty((N,), dtype=np.float32)
    policy = {"reject": _lib.ZERO_COLUMN_REJECT, "zero": _lib.ZERO_COLUMN_ZERO}[zero_columns]
    check(lib().mtrtq_quantize_per_channel(W.ctypes.data, K, N, q.ctypes.data, s.ctypes.data,
                                           policy), "mtrtq_quantize_per_channel")
    return q, s


def packed_bytes(K: int, N: int) -> int:
    n = lib().mtrtq_packed_bytes(K, N)
    if n < 0:
        raise ValueError(f"invalid weight shape K={K} N={N}")
    return n


def prepack_host(q: np.ndarray) -> np.ndarray:
    """Host layout transform int8 [K,N] -> packed bytes (uint8, 1-D)."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    K, N = q.shape
    out = np.empty(packed_bytes(K, N), dtype=np.uint8)
    check(lib().mtrtq_prepack_host(q.ctypes.data, K, N, out.ctypes.data, out.nbytes),
          "mtrtq_prepack_host")
    return out


@dataclass
class PackedWeight:
    """One MatMulQ weight on the device: packed int8 bytes + per-channel scale [N].

    Built once at load time (the CUDA executor's weight upload,
    backends/cuda/cuda_executor.cpp:61-72), reused by every launch."""

    packed: torch.Tensor  # uint8 [packed_bytes], 256-byte aligned
    scale: torch.Tensor   # float32 [N]
    K: int
    N: int

    @property
    def device(self) -> torch.device:
        return self.packed.device

    @classmethod
    def from_int8(cls, q, scale, device="cuda", stream=None) -> "PackedWeight":
        """Pre-pack int8 [K,N] (row-major, the reference's W layout) on the device."""
        q = torch.as_tensor(q)
        if q.dtype != torch.int8 or q.dim() != 2:
            raise ValueError("q must be int8 [K, N]")
        K, N = q.shape
        device = torch.device(device)
        q_dev = q.to(device).contiguous()
        scale = torch.as_tensor(scale, dtype=torch.float32).to(device).contiguous()
        if scale.numel() != N:
            raise ValueError("scale must be per-column [N]")
        nbytes = packed_bytes(K, N)
        packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
        with torch.cuda.device(device):
            check(lib().mtrtq_prepack(q_dev.data_ptr(), K, N, packed.data_ptr(), nbytes,
                                      _stream_ptr(stream)), "mtrtq_prepack")
        return cls(packed, scale, K, N)

    @classmethod
    def from_float(cls, W, device="cuda", zero_columns: str = "reject") -> "PackedWeight":
        """Quantize on the host with the reference rule, then pre-pack on the device."""
        q, s = quantize_per_channel(W, zero_columns)
        return cls.from_int8(torch.from_numpy(q), torch.from_numpy(s), device)


class Workspace:
    """Zero-filled device scratch grown on demand (only when a call needs more)."""

    def __init__(self, device="cuda"):
        self.device = torch.device(device)
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        return self.buf


_workspaces: dict = {}


def default_workspace(device) -> Workspace:
    device = torch.device(device)
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    if key not in _workspaces:
        _workspaces[key] = Workspace(torch.device(device.type, key[1]))
    return _workspaces[key]


def workspace_bytes(M: int, K: int, N: int, x_dtype: torch.dtype, mode: str) -> int:
    xd = _lib.DTYPE_BF16 if x_dtype == torch.bfloat16 else _lib.DTYPE_F32
    n = lib().mtrtq_workspace_bytes(M, K, N, xd, MODES[mode])
    if n < 0:
        raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_workspace_bytes", _lib.last_error())
    return n


def plan_info(M: int, K: int, N: int, x_dtype=torch.float32, mode: str = "bf16") -> dict:
    xd = _lib.DTYPE_BF16 if x_dtype == torch.bfloat16 else _lib.DTYPE_F32
    info = (ctypes.c_int64 * 6)()
    check(lib().mtrtq_plan_info(M, K, N, xd, MODES[mode], info, 6), "mtrtq_plan_info")
    path = {0: "gemv", 1: "gemm_tc", 2: "stream_k_tc", 3: "cluster_gemv", 4: "gemv_stream", 5: "gemv_tc"}[info[0]]
    out = {"path": path, "tile_m": info[1], "m_tiles": info[2], "n_tiles": info[3],
           "k_per_split": info[5]}
    out["ctas" if path in ("stream_k_tc", "gemv_stream", "gemv_tc") else "splits"] = info[4]
    return out


EPILOGUES = {"none": _lib.EPILOGUE_NONE, "gelu": _lib.EPILOGUE_GELU_TANH,
             "residual": _lib.EPILOGUE_ADD_RESIDUAL}


def matmul_q8(x: torch.Tensor, w: PackedWeight, bias: torch.Tensor | None = None,
              out: torch.Tensor | None = None, mode: str = "bf16",
              workspace: Workspace | torch.Tensor | None = None, stream=None,
              epilogue: str = "none", residual: torch.Tensor | None = None) -> torch.Tensor:
    """out[M,N] = x[M,K] @ dequant(w) (+ bias): the reference MatMulQ (+ Add) on the GPU.

    x: float32 or bfloat16 CUDA tensor [M, K] (row stride may exceed K).
    mode: "bf16" (x rounded to bf16 before the product) or "fp32".
    epilogue: "none"; "gelu" (gelu_new after the bias, the reference's fused
    MatMul+Bias+GeluTanh); "residual" (out = residual + result; residual may be out).
    """
    if x.dim() != 2 or x.shape[1] != w.K:
        raise ValueError(f"x must be [M, {w.K}], got {tuple(x.shape)}")
    if x.stride(1) != 1:
        raise ValueError("x must have unit stride along K")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("x must be float32 or bfloat16")
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.float32, device=x.device)
    if out.dtype != torch.float32 or out.shape != (M, w.N) or out.stride(1) != 1:
        raise ValueError("out must be float32 [M, N] with unit stride along N")
    xd = _lib.DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.DTYPE_F32
    need = lib().mtrtq_workspace_bytes(M, w.K, w.N, xd, MODES[mode])
    if need < 0:
        raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_workspace_bytes", _lib.last_error())
    if isinstance(workspace, torch.Tensor):
        ws = workspace
    else:
        ws = (workspace or default_workspace(x.device)).get(need)
    ws_ptr = ws.data_ptr() if ws is not None else None
    ws_bytes = ws.numel() * ws.element_size() if ws is not None else 0
    epi = EPILOGUES[epilogue]
    if epi == _lib.EPILOGUE_ADD_RESIDUAL:
        if residual is None or residual.dtype != torch.float32 or residual.shape != (M, w.N) \
                or residual.stride(1) != 1:
            raise ValueError("the residual epilogue needs residual float32 [M, N], unit stride")
    with torch.cuda.device(x.device):
        check(lib().mtrtq_matmul_ex(x.data_ptr(), xd, x.stride(0), w.packed.data_ptr(),
                                    w.scale.data_ptr(), _ptr(bias), out.data_ptr(), out.stride(0),
                                    M, w.K, w.N, MODES[mode], ws_ptr, ws_bytes, epi,
                                    _ptr(residual) if epi == _lib.EPILOGUE_ADD_RESIDUAL else None,
                                    residual.stride(0) if epi == _lib.EPILOGUE_ADD_RESIDUAL else 0,
                                    _stream_ptr(stream)),
              "mtrtq_matmul_ex")
    return out


def _group_problems(items):
    arr = (_lib.GemvProblem * len(items))()
    for i, it in enumerate(items):
        x, w, out = it["x"], it["w"], it["out"]
        bias, epi, res = it.get("bias"), EPILOGUES[it.get("epilogue", "none")], it.get("residual")
        if x.dim() != 2 or x.shape[1] != w.K or x.stride(1) != 1:
            raise ValueError(f"problem {i}: x must be [M, {w.K}] with unit stride along K")
        M = x.shape[0]
        if out.dtype != torch.float32 or out.shape != (M, w.N) or out.stride(1) != 1:
            raise ValueError(f"problem {i}: out must be float32 [M, N] with unit stride along N")
        if epi == _lib.EPILOGUE_ADD_RESIDUAL and (res is None or res.shape != (M, w.N) or res.stride(1) != 1):
            raise ValueError(f"problem {i}: the residual epilogue needs residual float32 [M, N]")
        arr[i] = _lib.GemvProblem(x.data_ptr(), x.stride(0), w.packed.data_ptr(), w.scale.data_ptr(), _ptr(bias),
                                  out.data_ptr(), out.stride(0), M, w.K, w.N, epi,
                                  _ptr(res) if epi == _lib.EPILOGUE_ADD_RESIDUAL else None,
                                  res.stride(0) if epi == _lib.EPILOGUE_ADD_RESIDUAL else 0)
    return arr


def group_workspace_bytes(items) -> int:
    """Bytes of workspace mtrtq_gemv_group needs for these problems."""
    arr = _group_problems(items)
    n = lib().mtrtq_gemv_group_workspace_bytes(arr, len(items))
    if n < 0:
        raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_gemv_group_workspace_bytes", _lib.last_error())
    return n


class GemvGroup:
    """A fixed group of independent decode products (M <= 8 each) run in one launch
    by mtrtq_gemv_group. items: dicts with x, w (PackedWeight), out, and optionally
    bias, epilogue ("none" | "gelu" | "residual") and residual. The tensors are bound
    once (their addresses are what the launch uses); the workspace is allocated and
    zero-filled here, at set-up."""

    def __init__(self, items, mode: str = "bf16"):
        if not items:
            raise ValueError("a group needs at least one problem")
        xd = {it["x"].dtype for it in items}
        if len(xd) != 1 or not xd <= {torch.float32, torch.bfloat16}:
            raise ValueError("every problem's x must have the same dtype, float32 or bfloat16")
        self.items = list(items)
        self.mode = mode
        self.x_dtype = _lib.DTYPE_BF16 if xd == {torch.bfloat16} else _lib.DTYPE_F32
        self.problems = _group_problems(self.items)
        dev = self.items[0]["x"].device
        n = lib().mtrtq_gemv_group_workspace_bytes(self.problems, len(self.items))
        if n < 0:
            raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_gemv_group_workspace_bytes", _lib.last_error())
        self.workspace = torch.zeros(max(n, 256), dtype=torch.uint8, device=dev)
        self.device = dev

    def __call__(self, stream=None):
        with torch.cuda.device(self.device):
            check(lib().mtrtq_gemv_group(self.problems, len(self.items), self.x_dtype, MODES[self.mode],
                                         self.workspace.data_ptr(), self.workspace.numel(), _stream_ptr(stream)),
                  "mtrtq_gemv_group")
        return [it["out"] for it in self.items]


def matmul_q8_ln(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float, w: PackedWeight,
                 bias: torch.Tensor | None = None, out: torch.Tensor | None = None, mode: str = "bf16",
                 stream=None, epilogue: str = "none", residual: torch.Tensor | None = None) -> torch.Tensor:
    """out = epilogue(LayerNorm(x; gamma, beta, eps) @ dequant(w) (+ bias)) in one
    launch sequence (mtrtq_matmul_ln_ex). x: float32 CUDA [M, K]; raises MtrtqError
    when the shape plans a kernel other than the decode GEMVs (check supports_ln
    first)."""
    if x.dim() != 2 or x.shape[1] != w.K or x.dtype != torch.float32 or x.stride(1) != 1:
        raise ValueError(f"x must be float32 [M, {w.K}] with unit stride along K")
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.float32, device=x.device)
    epi = EPILOGUES[epilogue]
    if epi == _lib.EPILOGUE_ADD_RESIDUAL and (residual is None or residual.shape != (M, w.N)):
        raise ValueError("the residual epilogue needs residual float32 [M, N]")
    need = lib().mtrtq_workspace_bytes(M, w.K, w.N, _lib.DTYPE_F32, MODES[mode])
    ws = default_workspace(x.device).get(need) if need > 0 else None
    with torch.cuda.device(x.device):
        check(lib().mtrtq_matmul_ln_ex(x.data_ptr(), x.stride(0), gamma.data_ptr(), beta.data_ptr(), float(eps),
                                       w.packed.data_ptr(), w.scale.data_ptr(), _ptr(bias), out.data_ptr(),
                                       out.stride(0), M, w.K, w.N, MODES[mode], _ptr(ws),
                                       ws.numel() if ws is not None else 0, epi,
                                       _ptr(residual) if epi == _lib.EPILOGUE_ADD_RESIDUAL else None,
                                       residual.stride(0) if epi == _lib.EPILOGUE_ADD_RESIDUAL else 0,
                                       _stream_ptr(stream)),
              "mtrtq_matmul_ln_ex")
    return out


def supports_ln(M: int, K: int, N: int, mode: str = "bf16") -> bool:
    """Whether mtrtq_matmul_ln_ex takes this shape (it plans a decode GEMV)."""
    return plan_info(M, K, N, torch.float32, mode)["path"] in ("cluster_gemv", "gemv_tc")


def host_workspace_bytes(M: int, K: int, N: int, mode: str = "bf16") -> int:
    n = lib().mtrtq_host_workspace_bytes(M, K, N, MODES[mode])
    if n < 0:
        raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_host_workspace_bytes", _lib.last_error())
    return n


def matmul_q8_host(x: torch.Tensor, w: PackedWeight, bias: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, mode: str = "bf16",
                   workspace: Workspace | torch.Tensor | None = None, stream=None,
                   blocking: bool = True) -> torch.Tensor:
    """The reference's MatMulQ (+ Add) on host tensors: x float32 [M, K] and the
    result in host memory, weights resident on w's device (mtrtq_matmul_host).
    Pinned x and out make the copies asynchronous; with blocking=False the caller
    synchronizes `stream` before reading out."""
    if x.device.type != "cpu" or x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != w.K:
        raise ValueError(f"x must be a float32 host tensor [M, {w.K}]")
    x = x.contiguous()
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.float32, pin_memory=x.is_pinned())
    if out.device.type != "cpu" or out.dtype != torch.float32 or out.shape != (M, w.N) \
            or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 host tensor [M, N]")
    dev = w.packed.device
    need = host_workspace_bytes(M, w.K, w.N, mode)
    ws = workspace if isinstance(workspace, torch.Tensor) else \
        (workspace or default_workspace(dev)).get(need)
    with torch.cuda.device(dev):
        check(lib().mtrtq_matmul_host(x.data_ptr(), w.packed.data_ptr(), w.scale.data_ptr(),
                                      _ptr(bias), out.data_ptr(), M, w.K, w.N, MODES[mode],
                                      ws.data_ptr(), ws.numel() * ws.element_size(),
                                      1 if blocking else 0, _stream_ptr(stream)),
              "mtrtq_matmul_host")
    return out


_options: dict = {}  # values set through set_option (the library starts with all at 0)


def set_option(option: int, value: int) -> None:
    check(lib().mtrtq_set_option(option, value), "mtrtq_set_option")
    _options[option] = value


def get_option(option: int) -> int:
    """The value last given to set_option in this process (0 if never set)."""
    return _options.get(option, 0)


@contextlib.contextmanager
def option(opt: int, value: int):
    """Runs the block with a process-wide option set, then restores its value."""
    old = get_option(opt)
    set_option(opt, value)
    try:
        yield
    finally:
        set_option(opt, old)


def read_device_status() -> int:
    v = ctypes.c_int(0)
    check(lib().mtrtq_read_status(ctypes.byref(v)), "mtrtq_read_status")
    return v.value
