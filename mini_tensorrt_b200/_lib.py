"""ctypes binding of libmtrtq.so (the C ABI in include/mtrtq.h).

The library is built in-tree (mini_tensorrt_b200/libmtrtq.so). There is no
fallback: if it is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmtrtq.so")

# Status codes (include/mtrtq.h)
OK = 0
ERR_INVALID_ARG = 1
ERR_ALIGNMENT = 2
ERR_WORKSPACE = 3
ERR_NO_DEVICE = 4
ERR_CUDA = 5
ERR_TIMEOUT = 6
ERR_ZERO_SCALE = 7

DTYPE_F32 = 0
DTYPE_BF16 = 1
MODE_BF16 = 0
MODE_FP32 = 1
ZERO_COLUMN_REJECT = 0
ZERO_COLUMN_ZERO = 1
OPT_GEMM_A_SOURCE = 1
OPT_FORCE_PATH = 2
OPT_OVERLAP_LAUNCH = 3
OPT_PRODUCER_LANES = 4
EPILOGUE_NONE, EPILOGUE_GELU_TANH, EPILOGUE_ADD_RESIDUAL = 0, 1, 2

# Every function the header declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
SIGNATURES = {
    "mtrtq_version": (_int, []),
    "mtrtq_status_string": (ctypes.c_char_p, [_int]),
    "mtrtq_last_error": (ctypes.c_char_p, []),
    "mtrtq_quantize_per_channel": (_int, [_vp, _i64, _i64, _vp, _vp, _int]),
    "mtrtq_packed_bytes": (_i64, [_i64, _i64]),
    "mtrtq_prepack": (_int, [_vp, _i64, _i64, _vp, _sz, _vp]),
    "mtrtq_prepack_host": (_int, [_vp, _i64, _i64, _vp, _sz]),
    "mtrtq_workspace_bytes": (_i64, [_i64, _i64, _i64, _int, _int]),
    "mtrtq_matmul": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int,
                            _vp, _sz, _vp]),
    "mtrtq_matmul_ex": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int,
                               _vp, _sz, _int, _vp, _i64, _vp]),
    "mtrtq_matmul_ln_ex": (_int, [_vp, _i64, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                  _i64, _int, _vp, _sz, _int, _vp, _i64, _vp]),
    "mtrtq_host_workspace_bytes": (_i64, [_i64, _i64, _i64, _int]),
    "mtrtq_matmul_host": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _int, _vp]),
    "mtrtq_set_option": (_int, [_int, _i64]),
    "mtrtq_plan_info": (_int, [_i64, _i64, _i64, _int, _int, _vp, _int]),
    "mtrtq_read_status": (_int, [_vp]),
    "mtrtq_matmul_gemv_noalloc": (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                         _int, _vp]),
    "mtrtq_decode_embed": (_int, [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "mtrtq_layernorm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "mtrtq_layernorm_strided": (_int, [_vp, _i64, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "mtrtq_decode_attention": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mtrtq_prefill_embed": (_int, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "mtrtq_prefill_attention": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mtrtq_gelu_tanh": (_int, [_vp, _vp, _i64, _vp]),
    "mtrtq_add_inplace": (_int, [_vp, _vp, _i64, _vp]),
    "mtrtq_argmax_rows": (_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "mtrtq_decode_next": (_int, [_vp, _i64, _vp, _vp, _i64, _vp, _vp]),
}
NOALLOC_SCRATCH_BYTES = 8 * 1024 * 1024
GROUP_MAX = 16


class GemvProblem(ctypes.Structure):
    """mtrtq_gemv_problem (include/mtrtq.h)."""
    _fields_ = [("X", _vp), ("ldx", _i64), ("packed", _vp), ("scale", _vp), ("bias", _vp), ("Y", _vp),
                ("ldy", _i64), ("M", _i64), ("K", _i64), ("N", _i64), ("epilogue", _int), ("residual", _vp),
                ("ldr", _i64)]


MAX_WORLD = 8
SPLIT_N, SPLIT_K = 0, 1
SHARD_FLAG_BYTES = 64
IPC_HANDLE_BYTES = 72


class ShardComm(ctypes.Structure):
    """mtrtq_shard_comm (include/mtrtq.h)."""
    _fields_ = [("rank", _int), ("world", _int), ("y", _vp * MAX_WORLD), ("slots", _vp * MAX_WORLD),
                ("slot_elems", _i64), ("flags", _vp * MAX_WORLD), ("alternating", _int)]


SIGNATURES["mtrtq_shard_range"] = (_int, [_i64, _int, _int, _int, _vp, _vp])
SIGNATURES["mtrtq_shard_slot_bytes"] = (_i64, [_i64, _i64, _int])
SIGNATURES["mtrtq_shard_workspace_bytes"] = (_i64, [_i64, _i64, _i64, _int, _int, _int, _int, _int])
SIGNATURES["mtrtq_matmul_sharded"] = (_int, [_vp, _int, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int,
                                             _int, _vp, ctypes.c_uint, _vp, _sz, _vp])
class ShardSegment(ctypes.Structure):
    """mtrtq_shard_segment (include/mtrtq.h)."""
    _fields_ = [("offset", _i64), ("rows", _i64), ("cols", _i64), ("ld", _i64)]


SIGNATURES["mtrtq_shard_allgather"] = (_int, [_vp, _int, _vp, ctypes.c_uint, _vp])
SIGNATURES["mtrtq_shard_allreduce"] = (_int, [_vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, ctypes.c_uint, _vp])
SIGNATURES["mtrtq_shard_slot_offset"] = (_i64, [_int, _i64, _i64])
SIGNATURES["mtrtq_ipc_export"] = (_int, [_vp, _vp])
SIGNATURES["mtrtq_ipc_import"] = (_int, [_vp, _vp])
SIGNATURES["mtrtq_ipc_close"] = (_int, [_vp])
SIGNATURES["mtrtq_gemv_group_workspace_bytes"] = (_i64, [_vp, _int])
SIGNATURES["mtrtq_gemv_group"] = (_int, [_vp, _int, _int, _int, _vp, _sz, _vp])
SIGNATURES["mtrtq_gemv_group_allgather"] = (_int, [_vp, _int, _int, _int, _vp, _sz, _vp, ctypes.c_uint, _vp])


class MtrtqError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, where: str, message: str):
        self.status = status
        super().__init__(f"{where}: status {status} ({status_string(status)}): {message}")


_lib = None


def lib() -> ctypes.CDLL:
    """Load libmtrtq.so once. Raises if it is missing: there is no CPU fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m mini_tensorrt_b200.build`")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def status_string(status: int) -> str:
    return lib().mtrtq_status_string(status).decode()


def last_error() -> str:
    return lib().mtrtq_last_error().decode()


def check(status: int, where: str) -> None:
    if status != OK:
        raise MtrtqError(status, where, last_error())
