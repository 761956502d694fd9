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
    """max |got - ref| / max |ref| over the whole output (the relative-error measure
    used for every floating-point tolerance in these tests)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref))
    if denom == 0.0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got - ref)) / denom)
