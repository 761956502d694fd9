"""The CPU oracle, pinned before it is trusted (no GPU needed).

* against the reference's own Golden.MatMulQ fixture (tests/golden_kernel_test.cpp:155-175);
* against the reference library's outputs for seeded inputs at every GPT-2 and
  large-model shape (hashes in tests/golden/seeded.json, made by gen_golden.py);
* live against oracle/_ref on ragged shapes when that library is present;
* the packer's rounding rule (lround: ties away from zero) and zero columns;
* the packing itself against the reference's own packer lines, run unmodified
  (its Golden.MatMulQ test body, oracle/_ref/ref_packer_pin), when built here.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
from tests.golden.gen_golden import SEEDED_CASES, case_inputs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_reference_golden_matmulq():
    g = np.load(os.path.join(GOLDEN, "matmulq_op.npz"))
    q, s = oracle.quantize_per_channel(g["b"])
    assert np.array_equal(q, g["q"]) and np.array_equal(s.view(np.uint32), g["s"].view(np.uint32))
    C = oracle.matmul_q8(g["a"], q, s)
    # Bit-exact with the reference kernel's output on the same packed weights.
    assert np.array_equal(C.view(np.uint32), g["c_ref"].view(np.uint32))
    # The reference test's own bar: within rtol = atol = 0.05 of fp32 A @ B
    # (tests/golden_kernel_test.cpp:174, numpy-style allclose of tests/support/golden.h:40-57).
    assert np.allclose(C, g["out"], rtol=0.05, atol=0.05)


with open(os.path.join(GOLDEN, "seeded.json")) as _f:
    _SEEDED = json.load(_f)["cases"]


@pytest.mark.parametrize("case", SEEDED_CASES, ids=[c[0] for c in SEEDED_CASES])
def test_seeded_cases_match_reference_bytes(case):
    exp = _SEEDED[case[0]]
    X, W, b = case_inputs(case)
    q, s = oracle.quantize_per_channel(W)
    assert _sha(q) == exp["q_sha256"], "int8 packing differs from the reference packer"
    assert _sha(s) == exp["scale_sha256"], "scales differ from the reference packer"
    C = oracle.matmul_q8(X, q, s, b)
    for i, v in exp["c_samples"].items():
        assert C.ravel()[int(i)] == np.float32(v)
    assert _sha(C) == exp["c_sha256"], "oracle output differs from the reference kernel"


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (1, 16, 17), (3, 48, 5), (2, 100, 129), (7, 33, 64),
                                   (16, 64, 128), (5, 1000, 7)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_oracle_equals_reference_library(M, K, N, with_bias):
    rng = np.random.default_rng(M * 1000 + K * 10 + N)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(0.02)
    X = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((N,), dtype=np.float32) if with_bias else None
    q, s = oracle.quantize_per_channel(W)
    a = oracle.matmul_q8(X, q, s, b)
    r = oracle.ref_matmul_q8(X, q, s, b)
    assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


def test_packer_ties_round_away_from_zero():
    # Column amax 127 -> scale exactly 1.0, so w/s = w and .5 ties are exact.
    W = np.array([[127.0, 2.5], [2.5, -2.5], [-3.5, 127.0], [0.5, -0.5]], dtype=np.float32)
    q, s = oracle.quantize_per_channel(W)
    assert s.tolist() == [1.0, 1.0]
    assert q[:, 0].tolist() == [127, 3, -4, 1]      # np.round would give 2, -4, 0
    assert q[:, 1].tolist() == [3, -3, 127, -1]


def test_packer_zero_column():
    W = np.zeros((4, 3), dtype=np.float32)
    W[:, 1] = [1.0, -2.0, 0.5, 0.0]
    q, s = oracle.quantize_per_channel(W)
    assert s[0] == 0.0 and s[2] == 0.0 and np.all(q[:, 0] == 0) and np.all(q[:, 2] == 0)
    C = oracle.matmul_q8(np.ones((2, 4), np.float32), q, s)
    assert np.all(C[:, 0] == 0.0) and np.all(C[:, 2] == 0.0)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_zero_column_output_matches_reference():
    # The reference packer divides 0/0 for an all-zero column; the bytes it stores
    # on x86-64 are q = 0, and its kernel then outputs 0 * 0. The oracle's explicit
    # zero policy gives the same output.
    W = np.zeros((8, 4), dtype=np.float32)
    W[:, 2] = np.arange(8, dtype=np.float32) - 3.5
    q, s = oracle.quantize_per_channel(W)
    X = np.arange(16, dtype=np.float32).reshape(2, 8)
    assert np.array_equal(oracle.matmul_q8(X, q, s), oracle.ref_matmul_q8(X, q, s))


def test_round_bf16_matches_torch():
    import torch
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 100,
                        np.array([0.0, -0.0, 1.0, 65504.0, 3.0e38, -3.0e38, 1e-40, np.inf, -np.inf],
                                 dtype=np.float32)])
    a = oracle.round_bf16(x)
    t = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(a.view(np.uint32), t.view(np.uint32))


_needs_pin = pytest.mark.skipif(not oracle.ref_packer_available(),
                                reason="oracle/_ref/ref_packer_pin not built here")


@_needs_pin
def test_reference_packer_runs_golden_matmulq():
    """The reference's TEST(Golden, MatMulQ), run as written on its own fixtures:
    its checks pass, and the packed bytes, scales and kernel output it produces are
    the committed ones (which the oracle matches above)."""
    g = np.load(os.path.join(GOLDEN, "matmulq_op.npz"))
    q, s, C, failed = oracle.ref_packer(g["b"], g["a"], g["out"])
    assert failed == 0
    assert np.array_equal(q, g["q"]) and np.array_equal(s.view(np.uint32), g["s"].view(np.uint32))
    assert np.array_equal(C.view(np.uint32), g["c_ref"].view(np.uint32))


def _unique_weight_cases():
    seen, out = set(), []
    for case in SEEDED_CASES:
        key = (case[2], case[3], case[5])
        if key not in seen:
            seen.add(key)
            out.append(case)
    return out


@_needs_pin
@pytest.mark.parametrize("case", _unique_weight_cases(), ids=lambda c: f"{c[5]}_{c[2]}x{c[3]}")
def test_reference_packer_pins_seeded_packing(case):
    """The reference's packer lines pack every seeded weight matrix into the bytes
    whose hashes are committed, and the oracle's restatement packs the same."""
    exp = _SEEDED[case[0]]
    _, W, _ = case_inputs(case)
    q, s, _, _ = oracle.ref_packer(W)
    assert _sha(q) == exp["q_sha256"] and _sha(s) == exp["scale_sha256"]
    qo, so = oracle.quantize_per_channel(W)
    assert np.array_equal(q, qo) and np.array_equal(s.view(np.uint32), so.view(np.uint32))


@_needs_pin
def test_reference_packer_ties_and_zero_column():
    """Exact .5 ties and an all-zero column through the reference's own lines: ties
    round away from zero (lround), and the zero column stores s = 0 with q = 0
    (0/0 through lround and the int8 cast on x86-64), as the oracle does."""
    W = np.array([[127.0, 2.5, 0.0], [2.5, -2.5, 0.0], [-3.5, 127.0, 0.0], [0.5, -0.5, 0.0]],
                 dtype=np.float32)
    q, s, _, _ = oracle.ref_packer(W)
    qo, so = oracle.quantize_per_channel(W)
    assert s.tolist() == [1.0, 1.0, 0.0] and np.array_equal(s.view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q, qo)
    assert q[:, 0].tolist() == [127, 3, -4, 1] and q[:, 2].tolist() == [0, 0, 0, 0]
