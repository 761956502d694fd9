"""Generates the committed golden fixtures for the MatMulQ parity tests.

Run in a checkout where the reference sources are available and the oracle
libraries are built (oracle/build_ref.sh):

    python tests/golden/gen_golden.py [REFERENCE_ROOT]

REFERENCE_ROOT: the argument, else $MTRTQ_REFERENCE_ROOT, else a checkout named
"reference" beside this repository.

Writes into tests/golden/:
  * matmulq_op.npz -- the reference's own Golden.MatMulQ case
    (tests/golden_kernel_test.cpp:155-175): its fixtures op_matmul_a [2,3],
    op_matmul_b [3,5], op_matmul_out [2,5] (PyTorch seed 123,
    python/gen_goldens.py:54-59), the per-column int8 packing of B and its scales
    as the reference's own test body packs them (oracle/_ref/ref_packer_pin), and
    MatMulQ's output computed by the reference's own kernel on them.
  * seeded.json -- for seeded inputs at the GPT-2 / large-model shapes
    (mini_tensorrt_b200/workloads.py): SHA-256 of the packed int8 weights and the
    scales (packed by the reference's own packer lines, oracle/_ref/ref_packer_pin)
    and of the reference kernel's fp32 output bytes, plus a few output values.
    The reference library computes the outputs, so a match of the oracle's bytes
    pins the oracle to the reference bit for bit without shipping megabytes.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from mini_tensorrt_b200 import workloads as wl  # noqa: E402

# (case id, M, K, N, with_bias, weight source)
SEEDED_CASES = [
    ("single_op_ffn_up_m64_bias", 64, 768, 3072, True, "ffn_up"),
    *[(f"decode_{name}_m{M}", M, K, N, False, name) for (name, K, N) in wl.DECODE_SHAPES
      for M in wl.DECODE_M],
    *[(f"large_{K}x{N}_m{M}", M, K, N, False, f"large_{K}x{N}") for (K, N) in wl.LARGE_SHAPES
      for M in (1, 16)],
]


def case_inputs(case):
    """Deterministic inputs of one seeded case: (X, W, bias or None)."""
    cid, M, K, N, with_bias, src = case
    if src.startswith("large_"):
        W = wl.weights(K, N, wl.shape_seed(src, K, N))
    else:
        W = wl.decode_weight(src, K, N)
    X = wl.activations(M, K, wl.shape_seed("x:" + cid, M, K))
    b = wl.bias(N, wl.shape_seed("b:" + cid, K, N)) if with_bias else None
    return X, W, b


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "MTRTQ_REFERENCE_ROOT", os.path.join(ROOT, "..", "reference"))
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/libmtrt_ref.so missing: run oracle/build_ref.sh first")

    g = os.path.join(ref_root, "models", "goldens")
    A = np.load(os.path.join(g, "op_matmul_a.npy")).astype(np.float32)
    B = np.load(os.path.join(g, "op_matmul_b.npy")).astype(np.float32)
    out = np.load(os.path.join(g, "op_matmul_out.npy")).astype(np.float32)
    if not oracle.ref_packer_available():
        raise SystemExit("oracle/_ref/ref_packer_pin missing: run oracle/build_ref.sh first")
    # Packing comes from the reference's own packer lines (its Golden.MatMulQ test
    # body, run by oracle/_ref/ref_packer_pin), not from the oracle's restatement.
    q, s, C, failed = oracle.ref_packer(B, A, out)
    assert failed == 0, "the reference's Golden.MatMulQ checks failed"
    np.savez(os.path.join(HERE, "matmulq_op.npz"), a=A, b=B, out=out, q=q, s=s, c_ref=C)

    cases = {}
    for case in SEEDED_CASES:
        cid, M, K, N, with_bias, _ = case
        X, W, b = case_inputs(case)
        q, s, _, _ = oracle.ref_packer(W)
        C = oracle.ref_matmul_q8(X, q, s, b)
        idx = np.linspace(0, C.size - 1, 8).astype(np.int64)
        cases[cid] = {
            "M": M, "K": K, "N": N, "bias": with_bias,
            "q_sha256": sha(q), "scale_sha256": sha(s), "c_sha256": sha(C),
            "c_samples": {str(int(i)): float(C.ravel()[i]) for i in idx},
        }
        print(cid, cases[cid]["c_sha256"][:16])
    with open(os.path.join(HERE, "seeded.json"), "w") as f:
        json.dump({"generator": "tests/golden/gen_golden.py",
                   "packing": "the reference's Golden.MatMulQ packer (oracle/_ref/ref_packer_pin)",
                   "outputs": "the reference's registry MatMulQ + Add (oracle/_ref/libmtrt_ref.so)",
                   "cases": cases}, f, indent=1)


if __name__ == "__main__":
    main()
