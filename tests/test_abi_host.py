"""The C ABI without a GPU: the library loads, exports every declared symbol, validates
its arguments, and its host functions (quantizer, pre-pack layout, planner) are right.
No compute call reaches a device here."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

import oracle
from mini_tensorrt_b200 import _lib, matmulq, workloads as wl

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "mtrtq.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mtrtq_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 12
    lib = _lib.lib()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/mtrtq.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\b(mtrtq_\w+)\b", out))
    assert set(names) == exported, f"exports differ from the header: {exported ^ set(names)}"


def test_version_and_status_strings():
    lib = _lib.lib()
    assert lib.mtrtq_version() == 100
    for code in range(8):
        assert _lib.status_string(code)
    assert _lib.status_string(99) == "unknown status"


def test_header_compiles_as_c_and_cxx(tmp_path):
    src = tmp_path / "use.c"
    src.write_text('#include "mtrtq.h"\nint main(void){return mtrtq_version() == 100 ? 0 : 1;}\n')
    for compiler, name in (("gcc", "use.c"), ("g++", "use.cpp")):
        f = tmp_path / name
        f.write_text(src.read_text())
        exe = tmp_path / f"use_{compiler}"
        r = subprocess.run([compiler, "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(f),
                            "-o", str(exe), _lib.LIB_PATH, f"-Wl,-rpath,{os.path.dirname(_lib.LIB_PATH)}"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert subprocess.run([str(exe)]).returncode == 0


@pytest.mark.parametrize("K,N", [(1, 1), (3, 5), (48, 17), (768, 2304), (3072, 768), (100, 129)])
def test_library_quantizer_bit_exact_with_oracle(K, N):
    W = wl.weights(K, N, K * 7 + N)
    q, s = matmulq.quantize_per_channel(W)
    q2, s2 = oracle.quantize_per_channel(W)
    assert np.array_equal(q, q2)
    assert np.array_equal(s.view(np.uint32), s2.view(np.uint32))


def test_library_quantizer_zero_column_policies():
    W = np.zeros((4, 3), np.float32)
    W[:, 1] = [1, -2, 3, -4]
    with pytest.raises(_lib.MtrtqError) as e:
        matmulq.quantize_per_channel(W, "reject")
    assert e.value.status == _lib.ERR_ZERO_SCALE and "column 0" in str(e.value)
    q, s = matmulq.quantize_per_channel(W, "zero")
    q2, s2 = oracle.quantize_per_channel(W)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)


def reference_layout(q: np.ndarray) -> np.ndarray:
    """Packed layout restated in numpy: [tile][slab][row in tile][16 k]."""
    K, N = q.shape
    n_pad = -(-N // 128) * 128
    k_pad = -(-K // 64) * 64
    full = np.zeros((k_pad, n_pad), np.int8)
    full[:K, :N] = q
    t = full.reshape(k_pad // 16, 16, n_pad // 128, 128)  # [slab][b][tile][row]
    return np.ascontiguousarray(t.transpose(2, 0, 3, 1)).view(np.uint8).ravel()


@pytest.mark.parametrize("K,N", [(1, 1), (16, 128), (48, 17), (100, 300), (768, 2304), (768, 50257)])
def test_prepack_host_layout(K, N):
    q = np.random.default_rng(K + N).integers(-127, 128, size=(K, N), dtype=np.int8)
    p = matmulq.prepack_host(q)
    assert p.size == matmulq.packed_bytes(K, N)
    assert np.array_equal(p, reference_layout(q))


def test_invalid_arguments_are_rejected_without_a_device():
    lib = _lib.lib()
    assert lib.mtrtq_packed_bytes(0, 5) == -1 and lib.mtrtq_packed_bytes(5, -1) == -1
    assert lib.mtrtq_quantize_per_channel(None, 2, 2, None, None, 0) == _lib.ERR_INVALID_ARG
    buf = (ctypes.c_uint8 * 16)()
    assert lib.mtrtq_prepack_host(buf, 64, 128, buf, 16) == _lib.ERR_INVALID_ARG  # too small
    assert "packed buffer" in _lib.last_error()
    assert lib.mtrtq_workspace_bytes(1, 64, 64, 7, 0) == -1                       # bad dtype
    assert lib.mtrtq_workspace_bytes(1, 64, 64, _lib.DTYPE_BF16, _lib.MODE_FP32) == -1
    assert lib.mtrtq_workspace_bytes(0, 64, 64, 0, 0) == -1
    assert lib.mtrtq_workspace_bytes(1, 1 << 31, 64, 0, 0) == -1
    assert lib.mtrtq_set_option(99, 0) == _lib.ERR_INVALID_ARG
    assert lib.mtrtq_set_option(_lib.OPT_FORCE_PATH, 7) == _lib.ERR_INVALID_ARG
    assert lib.mtrtq_matmul(None, 0, 64, None, None, None, None, 64, 1, 64, 64, 0, None, 0,
                            None) == _lib.ERR_INVALID_ARG


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device status")
def test_launch_without_device_fails_loudly():
    lib = _lib.lib()
    x = (ctypes.c_float * 64)()
    rc = lib.mtrtq_matmul(x, 0, 64, x, x, None, x, 64, 1, 64, 64, 0, None, 0, None)
    assert rc == _lib.ERR_NO_DEVICE
    assert lib.mtrtq_prepack(x, 64, 64, x, 1 << 20, None) in (_lib.ERR_NO_DEVICE, _lib.ERR_ALIGNMENT)


@pytest.mark.parametrize("M,K,N,mode,path", [
    (1, 768, 50257, "bf16", "cluster_gemv"), (8, 768, 768, "fp32", "cluster_gemv"),
    (8, 3072, 768, "bf16", "cluster_gemv"), (9, 768, 768, "bf16", "cluster_gemv"),
    (32, 768, 3072, "bf16", "cluster_gemv"), (33, 768, 3072, "bf16", "gemv_stream"),
    (16, 768, 50257, "bf16", "gemv_tc"), (16, 768, 50257, "fp32", "gemv_tc"),
    (16, 4096, 4096, "bf16", "stream_k_tc"), (16, 4096, 4096, "fp32", "cluster_gemv"),
    (32, 4096, 14336, "bf16", "gemv_tc"), (64, 14336, 4096, "fp32", "gemv_tc"),
    (33, 4096, 14336, "bf16", "gemm_tc"), (8, 4096, 14336, "fp32", "cluster_gemv"),
    (64, 768, 3072, "bf16", "gemv_stream"), (65, 768, 3072, "bf16", "gemm_tc"),
    (64, 4096, 4096, "bf16", "gemm_tc"), (64, 4096, 14336, "fp32", "gemv_tc"),
    (2048, 4096, 14336, "bf16", "gemm_tc"), (64, 768, 3072, "fp32", "gemv_stream"),
    (40, 3072, 768, "fp32", "gemv_stream"),
    (65, 768, 3072, "fp32", "gemv"),
    (1, 768, 200000, "bf16", "cluster_gemv"), (33, 768, 200000, "bf16", "gemm_tc"),
    (8, 24576, 128, "bf16", "stream_k_tc"), (32, 65536, 128, "bf16", "stream_k_tc"),
    (32, 65536, 128, "fp32", "gemv"),
])
def test_planner(M, K, N, mode, path):
    info = matmulq.plan_info(M, K, N, torch.float32, mode)
    assert info["path"] == path
    assert info["n_tiles"] == -(-N // 128)
    if path == "stream_k_tc":
        units = info["n_tiles"] * (-(-K // 64))
        kb = -(-K // 64)
        assert info["ctas"] == max(1, min(148, units // -(-kb // 8)))
        assert matmulq.workspace_bytes(M, K, N, torch.float32, mode) >= 4096 + info["ctas"] * 2 * M * 512
        return
    if path == "gemv_stream":
        # blocks of 8 tokens sharing the weights, three persistent CTAs per SM at most
        units = info["n_tiles"] * (-(-K // 64)) * (-(-M // 8))
        assert info["ctas"] == min(148 * 3, units) and info["m_tiles"] == -(-M // 8)
        assert matmulq.workspace_bytes(M, K, N, torch.float32, mode) == 4096 + info["ctas"] * 8192
        return
    if path == "gemv_tc":
        nt = next(t for t in (8, 16, 32, 64) if M <= t)
        units = info["n_tiles"] * (-(-K // 64))
        assert info["tile_m"] == nt and info["ctas"] == _tc_grid(units, nt)
        assert matmulq.workspace_bytes(M, K, N, torch.float32, mode) == _tc_workspace([(M, K)], units)
        return
    if path == "cluster_gemv":
        # CS ranks take near-equal ranges of the 64-k units; no workspace
        kb = -(-K // 64)
        assert 1 <= info["splits"] <= min(8, kb)
        assert info["k_per_split"] == -(-kb // info["splits"]) * 64
        assert matmulq.workspace_bytes(M, K, N, torch.float32, mode) == 0
        return
    # every split has work, and the splits cover K
    unit = 16 if path == "gemv" else 64
    k_pad = -(-K // 64) * 64
    assert (info["splits"] - 1) * info["k_per_split"] < k_pad <= info["splits"] * info["k_per_split"]
    ws = matmulq.workspace_bytes(M, K, N, torch.float32, mode)
    if info["splits"] > 1:
        assert ws >= info["splits"] * M * (-(-N // 128) * 128) * 4
    assert ws % 256 == 0 and ws >= 0


def test_forced_paths_change_the_plan():
    try:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 2)
        assert matmulq.plan_info(4, 768, 768)["path"] == "gemm_tc"
        with pytest.raises(_lib.MtrtqError):
            matmulq.plan_info(4, 768, 768, mode="fp32")
        matmulq.set_option(_lib.OPT_FORCE_PATH, 1)
        assert matmulq.plan_info(64, 768, 768)["path"] == "gemv"
        matmulq.set_option(_lib.OPT_FORCE_PATH, 3)
        assert matmulq.plan_info(8, 768, 768)["path"] == "stream_k_tc"
        with pytest.raises(_lib.MtrtqError):
            matmulq.plan_info(65, 768, 768)
        matmulq.set_option(_lib.OPT_FORCE_PATH, 4)
        assert matmulq.plan_info(8, 768, 768, mode="fp32")["path"] == "cluster_gemv"
        assert matmulq.workspace_bytes(8, 768, 768, torch.float32, "fp32") == 0
        with pytest.raises(_lib.MtrtqError):
            matmulq.plan_info(65, 768, 768)
        matmulq.set_option(_lib.OPT_FORCE_PATH, 6)
        info = matmulq.plan_info(40, 768, 3072, mode="fp32")
        assert info["path"] == "gemv_tc" and info["tile_m"] == 64 and info["ctas"] == _tc_grid(24 * 12, 64) == 72
        assert matmulq.workspace_bytes(40, 768, 3072, torch.float32, "fp32") == _tc_workspace([(40, 768)], 24 * 12)
        assert matmulq.plan_info(8, 768, 50257)["ctas"] == 296
        assert matmulq.plan_info(1, 64, 128)["ctas"] == 1
        with pytest.raises(_lib.MtrtqError):
            matmulq.plan_info(65, 768, 768)
        with pytest.raises(_lib.MtrtqError):
            matmulq.set_option(_lib.OPT_FORCE_PATH, 7)
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)


@pytest.mark.parametrize("M,K,N,cs", [(1, 768, 768, 8), (1, 768, 50257, 1), (1, 4096, 14336, 3),
                                      (8, 14336, 4096, 8), (1, 64, 128, 1), (3, 768, 2304, 8),
                                      (8, 3072, 768, 8), (1, 768, 200000, 1), (8, 4096, 14336, 3),
                                      (8, 16384, 128, 8), (8, 24576, 128, None),
                                      (16, 768, 50257, 1), (32, 4096, 14336, 5), (32, 768, 768, 8),
                                      (32, 14336, 4096, None), (33, 768, 768, 8), (64, 768, 3072, 6),
                                      (64, 4096, 14336, 5), (65, 768, 768, None)])
def test_cluster_gemv_plan(M, K, N, cs):
    """One cluster per 128-channel tile, 1 to 8 CTAs splitting K into 64-k units,
    all clusters resident (3 CTAs per SM for M <= 8, 2 up to 32, 1 up to 64) where
    the tiles allow; refused when a CTA's activation digits (3 bytes per activation)
    and two 8 KiB ring stages exceed 72 KiB (M <= 8), 110 KiB (M <= 32) or 200 KiB,
    or when M > 64."""
    matmulq.set_option(_lib.OPT_FORCE_PATH, 4)
    try:
        if cs is None:
            with pytest.raises(_lib.MtrtqError):
                matmulq.plan_info(M, K, N)
            return
        info = matmulq.plan_info(M, K, N)
        assert info["path"] == "cluster_gemv" and info["splits"] == cs
        assert info["n_tiles"] == -(-N // 128)
        kb = -(-K // 64)
        assert info["k_per_split"] == -(-kb // cs) * 64
        cap = (72 if M <= 8 else 110 if M <= 32 else 200) * 1024
        assert 3 * M * -(-kb // cs) * 64 + 2 * 8192 <= cap
        assert matmulq.workspace_bytes(M, K, N, torch.float32, "bf16") == 0
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)


def _problem(M, K, N):
    p = _lib.GemvProblem()
    p.M, p.K, p.N, p.ldx, p.ldy, p.epilogue = M, K, N, K, N, 0
    return p


def _tc_grid(units, nt):
    """The digit GEMV's persistent CTAs: two per SM up to 32 tokens (one at 64), and
    none with fewer than four 64-k units."""
    return min(-(-units // 4), 148 * (1 if nt == 64 else 2))


def _tc_workspace(problems, units):
    """The digit GEMV's workspace: part counters (4 KiB), per-token scales (16 x 64
    fp32), [grid][2][nt][128] fp32 partials (256-byte rounded), and each problem's
    digits, 256 * nt bytes per 64-k unit; nt = 8, 16, 32 or 64 holds the largest M."""
    mmax = max(M for M, _ in problems)
    nt = next(t for t in (8, 16, 32, 64) if mmax <= t)
    part = -(-(_tc_grid(units, nt) * 2 * nt * 128 * 4) // 256) * 256
    return 4096 + 16 * 64 * 4 + part + sum(-(-K // 64) * 256 * nt for _, K in problems)


def test_group_workspace_and_limits():
    """mtrtq_gemv_group_workspace_bytes: enough for either group kernel -- the digit
    GEMV (one CTA per SM, at most one per 64-k unit) and the mma.sync grouped GEMV
    (tickets + 8 KiB of partials per CTA, three CTAs per SM); groups of 1..16
    problems of M <= 64 and at most 1024 channel tiles."""
    lib = _lib.lib()
    decode = [(M, K, N) for M in (1, 8) for K, N in ((768, 2304), (768, 768), (768, 3072), (3072, 768),
                                                       (768, 50257))]
    arr = (_lib.GemvProblem * 10)(*[_problem(*s) for s in decode])
    want = max(4096 + 148 * 3 * 8192, _tc_workspace([(M, K) for M, K, _ in decode], 11160))
    assert lib.mtrtq_gemv_group_workspace_bytes(arr, 10) == want
    one = (_lib.GemvProblem * 1)(_problem(1, 64, 128))
    assert lib.mtrtq_gemv_group_workspace_bytes(one, 1) == max(4096 + 1 * 8192, _tc_workspace([(1, 64)], 1))
    wide_m = (_lib.GemvProblem * 2)(_problem(64, 768, 3072), _problem(9, 100, 300))
    units = 24 * 12 + 3 * 2
    assert lib.mtrtq_gemv_group_workspace_bytes(wide_m, 2) == max(
        4096 + min(units, 444) * 8192, _tc_workspace([(64, 768), (9, 100)], units))
    assert lib.mtrtq_gemv_group_workspace_bytes(arr, 0) == -1
    many = (_lib.GemvProblem * 17)(*[_problem(1, 64, 128)] * 17)
    assert lib.mtrtq_gemv_group_workspace_bytes(many, 17) == -1
    assert lib.mtrtq_gemv_group_workspace_bytes((_lib.GemvProblem * 1)(_problem(65, 64, 128)), 1) == -1
    wide = (_lib.GemvProblem * 3)(*[_problem(1, 64, 50257)] * 3)  # 3 x 393 tiles > 1024
    assert lib.mtrtq_gemv_group_workspace_bytes(wide, 3) == -1
    assert "1024" in _lib.last_error()
