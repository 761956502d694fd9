"""The no-allocation GEMV entry point (mtrtq_matmul_gemv_noalloc), through the C ABI.

Some callers cannot allocate device memory when they run the op -- a runtime whose
run() must not allocate, a plugin inside a framework that owns every device
allocation, a latency-critical decode loop -- so this entry point takes no
workspace and uses a fixed scratch array inside the library instead. Its results
must match the regular entry point's (mtrtq_matmul, whatever kernel it picks for
the shape), call after call, with the tolerances of the parity tests: 1e-4
normwise in fp32 mode, 1e-3 in bf16 mode (both sides round the activations to
bf16 there, so only the summation differs).

This file is collected last so that a run stopping at its first failure has run
every other test first; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from mini_tensorrt_b200 import _lib, matmulq, workloads as wl
from mini_tensorrt_b200.matmulq import MODES, PackedWeight
from tests.conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-4, "bf16": 1e-3}


def _noalloc(x, pw, bias, y, mode):
    rc = _lib.lib().mtrtq_matmul_gemv_noalloc(
        x.data_ptr(), _lib.DTYPE_F32, x.stride(0), pw.packed.data_ptr(), pw.scale.data_ptr(),
        bias.data_ptr() if bias is not None else None, y.data_ptr(), y.stride(0),
        x.shape[0], pw.K, pw.N, MODES[mode], torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.OK, _lib.last_error()


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_no_alloc_entry_point_matches_matmul_twice_in_a_row(cuda_device, mode):
    # Two consecutive calls of different shapes share the library's scratch: a
    # split-K decode shape (partials + counters) and the LM head.
    cases = [(8, 3072, 768, True), (1, 768, 50257, False)]
    for rep in range(2):
        for i, (M, K, N, with_bias) in enumerate(cases):
            W = wl.weights(K, N, 300 + i)
            q, s = matmulq.quantize_per_channel(W)
            pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
            x = torch.from_numpy(wl.activations(M, K, 400 + 10 * rep + i)).to(cuda_device)
            b = torch.from_numpy(wl.bias(N, 500 + i)).to(cuda_device) if with_bias else None
            ref = matmulq.matmul_q8(x, pw, bias=b, mode=mode)
            y = torch.full((M, N), float("nan"), device=cuda_device)
            _noalloc(x, pw, b, y, mode)
            torch.cuda.synchronize()
            got, want = y.cpu().numpy(), ref.cpu().numpy()
            assert np.all(np.isfinite(got))
            err = rel_err(got, want)
            assert err <= TOL[mode], f"rep {rep} case {i}: rel err {err:.3e}"
    assert matmulq.read_device_status() == 0


def test_no_alloc_entry_point_rejects_bad_arguments(cuda_device):
    lib = _lib.lib()
    x = torch.zeros(4, 64, device=cuda_device)
    y = torch.zeros(4, 64, device=cuda_device)
    assert lib.mtrtq_matmul_gemv_noalloc(None, 0, 64, None, None, None, y.data_ptr(), 64, 4, 64, 64,
                                         0, None) == _lib.ERR_INVALID_ARG
    pw = PackedWeight.from_float(wl.weights(64, 64, 1), cuda_device)
    rc = lib.mtrtq_matmul_gemv_noalloc(x.data_ptr(), 0, 64, pw.packed.data_ptr() + 16,
                                       pw.scale.data_ptr(), None, y.data_ptr(), 64, 4, 64, 64, 0, None)
    assert rc == _lib.ERR_ALIGNMENT
