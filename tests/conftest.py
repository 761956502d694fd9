import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; parity tests of the CUDA path")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device in this process")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "the CUDA path is built for sm_100a"
    return torch.device("cuda", 0)


def normwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| over the whole output."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref))
    if denom == 0.0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got - ref)) / denom)


def elementwise_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max over elements of |got - ref| / (|ref| + rms(ref)).

    `elementwise_rel_err <= tol` is the element-wise bound |d| <= tol*|ref| + atol
    with the floor atol = tol * rms(ref). Why a floor at all: an output is a dot
    product of K terms, and its rounding error (bf16 activations: each term off by
    up to 2^-9 of itself; fp32: summation order) scales with the magnitude of the
    terms, not with their sum. An output that cancels to near zero therefore carries
    the absolute error of a typical output, and a pure |d| <= tol*|ref| would fail
    on it for any tol. The output's root mean square is that typical magnitude."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(ref * ref)))
    if rms == 0.0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got - ref) / (np.abs(ref) + rms)))


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """The relative-error measure behind every floating-point tolerance in these
    tests: the larger of the normwise error (max |d| / max |ref|) and the
    element-wise one (|d| <= tol*|ref| + tol*rms(ref), see elementwise_rel_err),
    so a test's `rel_err(...) <= tol` holds both bounds."""
    return max(normwise_rel_err(got, ref), elementwise_rel_err(got, ref))
