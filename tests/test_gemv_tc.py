"""The tensor-core digit GEMV (gemv_tc.cu, MTRTQ_OPT_FORCE_PATH 6 and the default
kernel of mtrtq_gemv_group): tcgen05 kind::i8 products of the packed int8 weights
with four int8 digits of each activation row, against the CPU oracle (the
reference's MatMulQ restated).

Tolerances (tests/conftest.py rel_err: the larger of the normwise and the
element-wise measure):
  * fp32 mode against the oracle on the same inputs: <= 1e-4;
  * bf16 mode against the oracle on the same inputs: <= 2e-2, and against the
    oracle fed the bf16-rounded activations: <= 1e-4 (the digits hold a bf16 value
    exactly, so only the fp32 combination of the four digit sums differs)."""
import contextlib

import numpy as np
import pytest
import torch

import oracle
from mini_tensorrt_b200 import _lib, matmulq, workloads as wl
from mini_tensorrt_b200.matmulq import GemvGroup, PackedWeight, matmul_q8
from tests.conftest import rel_err
from tests.test_gemv_group import check_group, make_items

pytestmark = pytest.mark.gpu

FP32_TOL, BF16_TOL, BF16_SAME_INPUT_TOL = 1e-4, 2e-2, 1e-4


@contextlib.contextmanager
def forced(path):
    matmulq.set_option(_lib.OPT_FORCE_PATH, path)
    try:
        yield
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)


def _gelu_new(u):
    u = u.astype(np.float64)
    return (0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))).astype(np.float32)


SHAPES = [(1, 768, 2304), (8, 768, 50257), (1, 64, 128), (3, 100, 300), (8, 77, 129), (9, 768, 768),
          (16, 3072, 768), (17, 1000, 520), (32, 768, 3072), (33, 4096, 1000), (64, 768, 3072), (57, 77, 129),
          (64, 14336, 4096), (5, 12345, 77)]


@pytest.mark.parametrize("M,K,N", SHAPES, ids=[f"{M}x{K}x{N}" for M, K, N in SHAPES])
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_single_call_matches_oracle(cuda_device, M, K, N, mode):
    W = wl.weights(K, N, 900 + M)
    q, s = oracle.quantize_per_channel(W)
    X = wl.activations(M, K, 901 + M)
    b = wl.bias(N, 902)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    with forced(6):
        assert matmulq.plan_info(M, K, N, torch.float32, mode)["path"] == "gemv_tc"
        y = matmul_q8(torch.from_numpy(X).to(cuda_device), pw, bias=torch.from_numpy(b).to(cuda_device), mode=mode)
        torch.cuda.synchronize()
        y2 = matmul_q8(torch.from_numpy(X).to(cuda_device), pw, bias=torch.from_numpy(b).to(cuda_device), mode=mode)
        torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert torch.equal(y, y2), "results must not depend on timing"
    err = rel_err(got, oracle.matmul_q8(X, q, s, b))
    if mode == "fp32":
        assert err <= FP32_TOL, f"fp32 rel err {err:.3e}"
    else:
        assert err <= BF16_TOL, f"bf16 rel err {err:.3e}"
        errb = rel_err(got, oracle.matmul_q8(oracle.round_bf16(X), q, s, b))
        assert errb <= BF16_SAME_INPUT_TOL, f"bf16 rel err vs rounded inputs {errb:.3e}"


@pytest.mark.parametrize("epilogue", ["gelu", "residual"])
def test_epilogues(cuda_device, epilogue):
    M, K, N = 12, 768, 3072
    q, s = oracle.quantize_per_channel(wl.weights(K, N, 910))
    X, b, R = wl.activations(M, K, 911), wl.bias(N, 912), wl.activations(M, N, 913)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    T = lambda a: torch.from_numpy(a).to(cuda_device)
    y = T(R).clone()
    with forced(6):
        matmul_q8(T(X), pw, bias=T(b), out=y, mode="fp32", epilogue=epilogue,
                  residual=y if epilogue == "residual" else None)
        torch.cuda.synchronize()
    t = oracle.matmul_q8(X, q, s, b)
    want = _gelu_new(t) if epilogue == "gelu" else (R + t).astype(np.float32)
    assert rel_err(y.cpu().numpy(), want) <= FP32_TOL


def test_strided_and_bf16_activations(cuda_device):
    M, K, N = 7, 1000, 700
    q, s = oracle.quantize_per_channel(wl.weights(K, N, 920))
    X = wl.activations(M, K, 921)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    xb = torch.zeros((M, K + 3), device=cuda_device)  # a row stride that is not a multiple of 4
    xb[:, :K] = torch.from_numpy(X).to(cuda_device)
    with forced(6):
        y = matmul_q8(xb[:, :K], pw, mode="fp32")
        yb = matmul_q8(torch.from_numpy(X).to(cuda_device).to(torch.bfloat16), pw, mode="bf16")
        torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matmul_q8(X, q, s)) <= FP32_TOL
    assert rel_err(yb.cpu().numpy(), oracle.matmul_q8(oracle.round_bf16(X), q, s)) <= BF16_SAME_INPUT_TOL


def test_nan_and_zero_rows(cuda_device):
    M, K, N = 6, 768, 2304
    q, s = oracle.quantize_per_channel(wl.weights(K, N, 930))
    X = wl.activations(M, K, 931)
    X[1] = 0.0
    X[4, 100] = np.inf
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    with forced(6):
        y = matmul_q8(torch.from_numpy(X).to(cuda_device), pw, mode="fp32")
        torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.all(got[1] == 0.0)
    assert np.all(np.isnan(got[4]))
    keep = [0, 2, 3, 5]
    assert rel_err(got[keep], oracle.matmul_q8(X[keep], q, s)) <= FP32_TOL


@pytest.mark.parametrize("M,K,N", [(1, 768, 2304), (8, 768, 3072), (3, 100, 300), (16, 768, 768),
                                   (64, 768, 3072), (41, 768, 768), (8, 768, 50257)])
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_layernorm_prologue(cuda_device, M, K, N, mode):
    W = wl.weights(K, N, 940 + M)
    q, s = oracle.quantize_per_channel(W)
    rng = np.random.default_rng(941 + M)
    X = (rng.standard_normal((M, K)) * 3 + 0.5).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    be = (0.1 * rng.standard_normal(K)).astype(np.float32)
    b = wl.bias(N, 942)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    T = lambda a: torch.from_numpy(a).to(cuda_device)
    with forced(6):
        assert matmulq.supports_ln(M, K, N, mode)
        y = matmulq.matmul_q8_ln(T(X), T(g), T(be), 1e-5, pw, bias=T(b), mode=mode, epilogue="gelu")
        torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    c = X - X.mean(axis=1, keepdims=True, dtype=np.float32)
    var = (c * c).mean(axis=1, keepdims=True, dtype=np.float32)
    H = (c * (np.float32(1.0) / np.sqrt(var + np.float32(1e-5))) * g + be).astype(np.float32)
    got = y.cpu().numpy()
    err = rel_err(got, _gelu_new(oracle.matmul_q8(H, q, s, b)))
    assert err <= (FP32_TOL if mode == "fp32" else BF16_TOL), f"rel err {err:.3e}"
    if mode == "bf16":
        assert rel_err(got, _gelu_new(oracle.matmul_q8(oracle.round_bf16(H), q, s, b))) <= 2e-3


DECODE = [(M, K, N) for M in wl.DECODE_M for _, K, N in wl.DECODE_SHAPES]


@pytest.mark.parametrize("kernel", [6, 5])
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_group_kernels_agree_with_oracle(cuda_device, kernel, mode):
    """The decode set as one group on the digit GEMV (the default) and on the mma.sync
    grouped GEMV (force path 5)."""
    items, host = make_items(DECODE, cuda_device, seed=11, bias=False)
    with forced(kernel):
        g = GemvGroup(items, mode=mode)
        g()
        torch.cuda.synchronize()
        first = [it["out"].clone() for it in items]
        g()
        torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    check_group(items, host, mode)
    for a, it in zip(first, items):
        assert torch.equal(a, it["out"])


def test_group_of_wide_problems(cuda_device):
    """Problems of up to 64 tokens in one group (the digit GEMV's N = 4 x 64)."""
    shapes = [(64, 768, 3072), (17, 3072, 768), (40, 768, 2304), (1, 768, 50257), (33, 100, 300)]
    epis = ["gelu", "residual", "none", "none", "gelu"]
    items, host = make_items(shapes, cuda_device, seed=12, epilogues=epis)
    GemvGroup(items, mode="fp32")()
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    check_group(items, host, "fp32")


def test_single_and_group_agree(cuda_device):
    items, host = make_items([(8, 768, 2304)], cuda_device, seed=13)
    GemvGroup(items, mode="fp32")()
    it = items[0]
    with forced(6):
        y = matmul_q8(it["x"], it["w"], bias=it["bias"], mode="fp32")
    torch.cuda.synchronize()
    assert torch.equal(y, it["out"])
