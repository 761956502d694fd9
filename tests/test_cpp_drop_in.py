"""The C++ drop-in (include/mtrtq_registry.hpp): the device MatMulQ registered into
the reference's own KernelRegistry and run through lookup -> fn(OpContext) by a
compiled C++ program (tests/cpp/registry_drop_in.cpp, built by oracle/build_ref.sh
against the reference's sources into oracle/_ref/registry_drop_in). The program
runs the reference's TEST(Golden, MatMulQ) body, unmodified, with the device kernel
bound in the registry, then seeded shapes against the reference's CPU kernel."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
BIN = os.path.join(ROOT, "oracle", "_ref", "registry_drop_in")
GOLDEN = os.path.join(ROOT, "tests", "golden", "matmulq_op.npz")


@pytest.mark.gpu
def test_reference_registry_runs_the_device_kernel(cuda_device, tmp_path):
    assert os.path.exists(BIN), "oracle/_ref/registry_drop_in was not built (oracle/build_ref.sh)"
    g = np.load(GOLDEN)
    for name, key in (("op_matmul_a", "a"), ("op_matmul_b", "b"), ("op_matmul_out", "out")):
        np.save(str(tmp_path / f"{name}.npy"), np.ascontiguousarray(g[key], dtype=np.float32))
    r = subprocess.run([BIN, str(tmp_path)], capture_output=True, text=True, timeout=300)
    lines = r.stdout.strip().splitlines()
    assert r.returncode == 0, r.stdout + r.stderr
    assert lines[0].startswith("Golden.MatMulQ") and lines[0].endswith("ok")
    assert len(lines) == 6 and all(l.endswith("ok") for l in lines), r.stdout
