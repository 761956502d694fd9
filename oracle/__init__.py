"""CPU oracle for the INT8 weight-only MatMul (MatMulQ) path.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
the cpu_baseline / --impl reference legs of bench.py, never by the product
package. It is the checker, not the thing measured or shipped.

Two libraries back it:
  * liboracle.so -- matmulq_oracle.c, a C restatement of the reference's
    MatMulQ kernel (src/ops/kernels_matmul.cpp:66-73), its test packer
    (tests/golden_kernel_test.cpp:163-170) and the bias Add
    (src/ops/kernels_elementwise.cpp:31-35).
  * _ref/libmtrt_ref.so -- the reference's own sources compiled by
    build_ref.sh, called through its KernelRegistry. Optional at run time:
    present where it was built (it travels with the repository snapshot).

Parity of the restatement is pinned against _ref (bit-exact) and against the
reference's Golden.MatMulQ fixture by tests/test_oracle.py.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_REF_PATH = os.path.join(_HERE, "_ref", "libmtrt_ref.so")

_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def lib():
    """The C restatement, loaded once. Raises if it was never built."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"oracle library missing: {_LIB_PATH} (run oracle/build_ref.sh)")
        l = ctypes.CDLL(_LIB_PATH)
        l.oracle_quantize_per_channel.argtypes = [_f32p, _i64, _i64, _i8p, _f32p]
        l.oracle_quantize_per_channel.restype = _i64
        l.oracle_matmul_q8_f32.argtypes = [_f32p, _i8p, _f32p, _f32p, _i64, _i64, _i64]
        l.oracle_matmul_q8_f32.restype = None
        l.oracle_matmul_q8_f32_rows.argtypes = [_f32p, _i8p, _f32p, _f32p, _i64p, _i64, _i64, _i64]
        l.oracle_matmul_q8_f32_rows.restype = None
        l.oracle_add_bias.argtypes = [_f32p, _f32p, _i64, _i64]
        l.oracle_add_bias.restype = None
        l.oracle_round_bf16.argtypes = [_f32p, _f32p, _i64]
        l.oracle_round_bf16.restype = None
        _lib = l
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


_PIN_PATH = os.path.join(_HERE, "_ref", "ref_packer_pin")


def ref_packer_available() -> bool:
    return os.path.exists(_PIN_PATH)


def ref_packer(W: np.ndarray, A: np.ndarray | None = None, expected: np.ndarray | None = None):
    """Packs W f32 [K,N] with the reference's own packer lines: the body of its
    TEST(Golden, MatMulQ) (tests/golden_kernel_test.cpp:155-175, packer at
    :163-170) compiled unmodified into oracle/_ref/ref_packer_pin. Returns
    (q int8 [K,N], scale f32 [N], C or None, checks_failed): C is the reference
    kernel's output on A when the test's fixed [2,5] output fits it, and
    checks_failed counts the test's own failed assertions (its 0.05 bar against
    `expected`, zeros when not given)."""
    import subprocess
    import tempfile
    if not ref_packer_available():
        raise RuntimeError(f"reference packer missing: {_PIN_PATH} (run oracle/build_ref.sh)")
    W = _f32(W)
    K, N = W.shape
    A = np.zeros((2, K), np.float32) if A is None else _f32(A)
    expected = np.zeros((2, 5), np.float32) if expected is None else _f32(expected)
    with tempfile.TemporaryDirectory() as d:
        np.save(os.path.join(d, "op_matmul_a.npy"), A)
        np.save(os.path.join(d, "op_matmul_b.npy"), W)
        np.save(os.path.join(d, "op_matmul_out.npy"), expected)
        out = os.path.join(d, "pin")
        r = subprocess.run([_PIN_PATH, d, out], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"ref_packer_pin failed ({r.returncode}): {r.stderr}")
        failed = int(r.stdout.strip().split("=")[1])
        q = np.fromfile(out + ".q", np.int8).reshape(K, N)
        s = np.fromfile(out + ".s", np.float32)
        C = np.fromfile(out + ".c", np.float32).reshape(A.shape[0], N) if os.path.exists(out + ".c") else None
    return q, s, C, failed


def ref():
    """The reference's own MatMulQ path (oracle/_ref). Raises if absent."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference library missing: {_REF_PATH} (run oracle/build_ref.sh)")
        r = ctypes.CDLL(_REF_PATH)
        r.ref_matmulq.argtypes = [_f32p, _i8p, _f32p, _f32p, _i64, _i64, _i64]
        r.ref_matmulq.restype = ctypes.c_int
        r.ref_add_bias.argtypes = [_f32p, _f32p, _i64, _i64]
        r.ref_add_bias.restype = ctypes.c_int
        r.ref_gemm_auto.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        r.ref_gemm_auto.restype = None
        r.ref_hardware_threads.argtypes = []
        r.ref_hardware_threads.restype = ctypes.c_int
        r.ref_matmulq_prepare.argtypes = [_f32p, _i8p, _f32p, _i64, _i64, _i64]
        r.ref_matmulq_prepare.restype = ctypes.c_void_p
        r.ref_matmulq_run.argtypes = [ctypes.c_void_p]
        r.ref_matmulq_run.restype = None
        r.ref_matmulq_output.argtypes = [ctypes.c_void_p, _f32p]
        r.ref_matmulq_output.restype = None
        r.ref_matmulq_free.argtypes = [ctypes.c_void_p]
        r.ref_matmulq_free.restype = None
        _ref = r
    return _ref


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def quantize_per_channel(W: np.ndarray):
    """(q int8 [K,N], scale f32 [N]) per tests/golden_kernel_test.cpp:163-170."""
    W = _f32(W)
    K, N = W.shape
    q = np.empty((K, N), dtype=np.int8)
    s = np.empty((N,), dtype=np.float32)
    lib().oracle_quantize_per_channel(_ptr(W, _f32p), K, N, _ptr(q, _i8p), _ptr(s, _f32p))
    return q, s


def matmul_q8(A: np.ndarray, q: np.ndarray, s: np.ndarray, bias: np.ndarray | None = None):
    """C = A x dequant(q, s) (+ bias), the reference's loop order, fp32."""
    A = _f32(A)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    M, K = A.shape
    K2, N = q.shape
    assert K == K2 and s.shape == (N,)
    C = np.empty((M, N), dtype=np.float32)
    lib().oracle_matmul_q8_f32(_ptr(A, _f32p), _ptr(q, _i8p), _ptr(s, _f32p), _ptr(C, _f32p), M, K, N)
    if bias is not None:
        b = _f32(bias)
        lib().oracle_add_bias(_ptr(C, _f32p), _ptr(b, _f32p), M, N)
    return C


def matmul_q8_rows(A, q, s, rows, bias=None):
    """Rows `rows` of matmul_q8(A, q, s, bias), computed alone (rows are independent)."""
    A = _f32(A)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    K, N = q.shape
    C = np.empty((rows.size, N), dtype=np.float32)
    lib().oracle_matmul_q8_f32_rows(_ptr(A, _f32p), _ptr(q, _i8p), _ptr(s, _f32p), _ptr(C, _f32p),
                                    _ptr(rows, _i64p), rows.size, K, N)
    if bias is not None:
        b = _f32(bias)
        lib().oracle_add_bias(_ptr(C, _f32p), _ptr(b, _f32p), rows.size, N)
    return C


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().oracle_round_bf16(_ptr(x, _f32p), _ptr(y, _f32p), x.size)
    return y


def ref_matmul_q8(A, q, s, bias=None):
    """The reference's registry MatMulQ (+ its Add kernel for the bias)."""
    A = _f32(A)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    M, K = A.shape
    N = q.shape[1]
    C = np.empty((M, N), dtype=np.float32)
    rc = ref().ref_matmulq(_ptr(A, _f32p), _ptr(q, _i8p), _ptr(s, _f32p), _ptr(C, _f32p), M, K, N)
    if rc != 0:
        raise RuntimeError("reference registry has no MatMulQ kernel")
    if bias is not None:
        b = _f32(bias)
        if ref().ref_add_bias(_ptr(C, _f32p), _ptr(b, _f32p), M, N) != 0:
            raise RuntimeError("reference registry has no Add kernel")
    return C


class RefMatmulqCall:
    """One reference MatMulQ call prepared once (Tensors built, kernel looked up);
    run() is the kernel call alone, as the reference executor's run loop makes it."""

    def __init__(self, A, q, s):
        A = _f32(A)
        q = np.ascontiguousarray(q, dtype=np.int8)
        s = _f32(s)
        self.M, K = A.shape
        self.N = q.shape[1]
        self._h = ref().ref_matmulq_prepare(_ptr(A, _f32p), _ptr(q, _i8p), _ptr(s, _f32p), self.M, K, self.N)
        if not self._h:
            raise RuntimeError("reference registry has no MatMulQ kernel")
        self._run = ref().ref_matmulq_run

    def run(self):
        self._run(self._h)

    def output(self):
        C = np.empty((self.M, self.N), np.float32)
        ref().ref_matmulq_output(self._h, _ptr(C, _f32p))
        return C

    def __del__(self):
        if getattr(self, "_h", None):
            ref().ref_matmulq_free(self._h)
            self._h = None


def ref_gemm_auto(A, B):
    """The reference's fp32 gemm_auto (threaded above its size threshold)."""
    A = _f32(A)
    B = _f32(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.zeros((M, N), dtype=np.float32)
    ref().ref_gemm_auto(_ptr(A, _f32p), _ptr(B, _f32p), _ptr(C, _f32p), M, N, K)
    return C
