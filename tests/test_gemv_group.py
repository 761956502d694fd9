"""The grouped decode GEMV (mtrtq_gemv_group): independent MatMulQ problems of
M <= 8 in one persistent launch, against the CPU oracle (the reference's MatMulQ
restated) and against the one-call-per-problem path."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from mini_tensorrt_b200 import _lib, matmulq, workloads as wl
from mini_tensorrt_b200.matmulq import GemvGroup, PackedWeight
from tests.conftest import rel_err

FP32_TOL, BF16_TOL, BF16_SAME_INPUT_TOL = 1e-4, 2e-2, 1e-4


def _gelu_new(u):
    u = u.astype(np.float64)
    return (0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))).astype(np.float32)


def make_items(shapes, dev, seed=0, x_dtype=torch.float32, epilogues=None, bias=True):
    """shapes: (M, K, N) per problem. Returns (items, host copies for the oracle)."""
    items, host = [], []
    for i, (M, K, N) in enumerate(shapes):
        W = wl.weights(K, N, seed * 100 + i)
        q, s = oracle.quantize_per_channel(W)
        X = wl.activations(M, K, seed * 100 + 50 + i)
        if x_dtype == torch.bfloat16:
            X = oracle.round_bf16(X)
        b = wl.bias(N, seed * 100 + 70 + i) if bias else None
        epi = epilogues[i] if epilogues else "none"
        R = wl.activations(M, N, seed * 100 + 90 + i) if epi == "residual" else None
        out = torch.from_numpy(R).to(dev).clone() if R is not None else torch.full((M, N), float("nan"), device=dev)
        it = {"x": torch.from_numpy(X).to(dev).to(x_dtype), "w": PackedWeight.from_int8(
            torch.from_numpy(q), torch.from_numpy(s), dev), "out": out, "epilogue": epi}
        if b is not None:
            it["bias"] = torch.from_numpy(b).to(dev)
        if epi == "residual":
            it["residual"] = out
        items.append(it)
        host.append((X, q, s, b, epi, R))
    return items, host


def want(h, round_x=False):
    X, q, s, b, epi, R = h
    t = oracle.matmul_q8(oracle.round_bf16(X) if round_x else X, q, s, b)
    if epi == "gelu":
        return _gelu_new(t)
    if epi == "residual":
        return (R + t).astype(np.float32)
    return t


def check_group(items, host, mode):
    for i, (it, h) in enumerate(zip(items, host)):
        got = it["out"].cpu().numpy()
        assert np.all(np.isfinite(got)), f"problem {i}"
        err = rel_err(got, want(h))
        assert err <= (FP32_TOL if mode == "fp32" else BF16_TOL), f"problem {i}: rel err {err:.3e}"
        if mode == "bf16":
            errb = rel_err(got, want(h, round_x=True))
            assert errb <= BF16_SAME_INPUT_TOL, f"problem {i}: rel err vs rounded inputs {errb:.3e}"


DECODE = [(M, K, N) for M in wl.DECODE_M for _, K, N in wl.DECODE_SHAPES]


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_decode_set_in_one_launch(cuda_device, mode):
    items, host = make_items(DECODE, cuda_device, seed=1, bias=False)
    g = GemvGroup(items, mode=mode)
    g()
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    check_group(items, host, mode)
    first = [it["out"].clone() for it in items]
    g()  # again: tickets were left at zero, and results do not depend on timing
    torch.cuda.synchronize()
    for a, it in zip(first, items):
        assert torch.equal(a, it["out"])


MIXED = [(3, 100, 300), (8, 77, 129), (1, 4096, 1000), (5, 64, 128), (2, 768, 50257), (7, 3000, 200),
         (1, 12345, 77), (4, 64 * 13, 128 * 3)]


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_ragged_mixed_group_with_epilogues(cuda_device, mode):
    epis = ["gelu", "residual", "none", "gelu", "none", "residual", "none", "gelu"]
    items, host = make_items(MIXED, cuda_device, seed=2, epilogues=epis)
    GemvGroup(items, mode=mode)()
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    check_group(items, host, mode)


@pytest.mark.gpu
def test_bf16_activations(cuda_device):
    items, host = make_items(MIXED[:5], cuda_device, seed=3, x_dtype=torch.bfloat16)
    GemvGroup(items, mode="bf16")()
    torch.cuda.synchronize()
    check_group(items, host, "bf16")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 768, 50257), (8, 768, 50257), (1, 64, 128), (8, 128, 256),
                                   (3, 14336, 4096)])
def test_single_problem_matches_per_call_path(cuda_device, shape):
    """A group of one (fewer units than CTAs for the small shapes) against the oracle
    and against mtrtq_matmul on the same problem."""
    items, host = make_items([shape], cuda_device, seed=4)
    GemvGroup(items, mode="fp32")()
    torch.cuda.synchronize()
    check_group(items, host, "fp32")
    it = items[0]
    ref = matmulq.matmul_q8(it["x"], it["w"], bias=it["bias"], mode="fp32")
    assert rel_err(it["out"].cpu().numpy(), ref.cpu().numpy()) <= FP32_TOL


@pytest.mark.gpu
def test_nan_activation_poisons_its_row_only(cuda_device):
    items, host = make_items([(4, 300, 700), (3, 768, 2304)], cuda_device, seed=5)
    x = items[1]["x"]
    x[2, 17] = float("nan")
    X = host[1][0].copy()
    X[2, 17] = np.nan
    host[1] = (X,) + host[1][1:]
    GemvGroup(items, mode="fp32")()
    torch.cuda.synchronize()
    got = items[1]["out"].cpu().numpy()
    assert np.all(np.isnan(got[2]))
    keep = [0, 1]
    assert rel_err(got[keep], want(host[1])[keep]) <= FP32_TOL
    assert rel_err(items[0]["out"].cpu().numpy(), want(host[0])) <= FP32_TOL


@pytest.mark.gpu
def test_argument_errors_on_device(cuda_device):
    items, _ = make_items([(2, 64, 128)], cuda_device, seed=6)
    g = GemvGroup(items, mode="fp32")
    lib = _lib.lib()
    bad = (_lib.GemvProblem * 1)()
    ctypes.memmove(bad, g.problems, ctypes.sizeof(bad))
    bad[0].Y = bad[0].Y + 2  # not 4-byte aligned
    rc = lib.mtrtq_gemv_group(bad, 1, _lib.DTYPE_F32, _lib.MODE_FP32, g.workspace.data_ptr(),
                              g.workspace.numel(), None)
    assert rc == _lib.ERR_ALIGNMENT
    rc = lib.mtrtq_gemv_group(g.problems, 1, _lib.DTYPE_F32, _lib.MODE_FP32, g.workspace.data_ptr(), 16, None)
    assert rc == _lib.ERR_WORKSPACE
    rc = lib.mtrtq_gemv_group(g.problems, 1, _lib.DTYPE_BF16, _lib.MODE_FP32, g.workspace.data_ptr(),
                              g.workspace.numel(), None)
    assert rc == _lib.ERR_INVALID_ARG
