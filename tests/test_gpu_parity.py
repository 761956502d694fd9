"""Parity of the CUDA path with the CPU oracle, through the C ABI (GPU).

Tolerances (normwise relative error = max|y - ref| / max|ref|, tests/conftest.py):
  * MTRTQ_MODE_FP32 vs the oracle on the same fp32 inputs: <= 1e-4
    (the stated bar for fp32 CUDA-core mode);
  * MTRTQ_MODE_BF16 vs the oracle on the same inputs: <= 2e-2 (the stated bar
    after bf16 activation rounding), and vs the oracle fed the bf16-rounded
    activations: <= 1e-4 on CUDA cores, <= 1e-3 on tensor cores -- the products
    are then identical and only fp32 summation order differs.
Packing is checked bit for bit (device pre-pack vs the host layout transform).
"""
import contextlib

import numpy as np
import pytest
import torch

import oracle
from mini_tensorrt_b200 import _lib, matmulq, registry, workloads as wl
from mini_tensorrt_b200.matmulq import PackedWeight, matmul_q8
from tests.conftest import rel_err
from tests.golden.gen_golden import SEEDED_CASES, case_inputs

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_SPEC_TOL = 2e-2
BF16_SAME_INPUT_TOL_CORES = 1e-4
BF16_SAME_INPUT_TOL_TC = 1e-3


@contextlib.contextmanager
def forced(path):
    """Runs the block with MTRTQ_OPT_FORCE_PATH = path (0 restores the planner)."""
    matmulq.set_option(_lib.OPT_FORCE_PATH, path)
    try:
        yield
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)


def run(X, q, s, mode, bias=None, x_dtype=torch.float32, dev="cuda"):
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), dev)
    xt = torch.from_numpy(X).to(dev).to(x_dtype)
    bt = torch.from_numpy(bias).to(dev) if bias is not None else None
    y = torch.full((X.shape[0], q.shape[1]), float("nan"), device=dev)
    matmul_q8(xt, pw, bias=bt, out=y, mode=mode)
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    return y.cpu().numpy()


def check(Y, X, q, s, mode, bias=None, rows=None, tc=False):
    if rows is not None:
        ref = oracle.matmul_q8_rows(X, q, s, rows, bias)
        refb = oracle.matmul_q8_rows(oracle.round_bf16(X), q, s, rows, bias)
        Y = Y[rows]
    else:
        ref = oracle.matmul_q8(X, q, s, bias)
        refb = oracle.matmul_q8(oracle.round_bf16(X), q, s, bias)
    assert np.all(np.isfinite(Y))
    if mode == "fp32":
        err = rel_err(Y, ref)
        assert err <= FP32_TOL, f"fp32 mode rel err {err:.3e}"
    else:
        err = rel_err(Y, ref)
        assert err <= BF16_SPEC_TOL, f"bf16 mode rel err vs fp32 inputs {err:.3e}"
        errb = rel_err(Y, refb)
        tol = BF16_SAME_INPUT_TOL_TC if tc else BF16_SAME_INPUT_TOL_CORES
        assert errb <= tol, f"bf16 mode rel err vs rounded inputs {errb:.3e}"


def test_device_prepack_matches_host_layout(cuda_device):
    for K, N in [(48, 17), (768, 2304), (768, 50257), (100, 300)]:
        q = np.random.default_rng(K * N).integers(-128, 128, size=(K, N), dtype=np.int8)
        pw = PackedWeight.from_int8(torch.from_numpy(q), torch.ones(N), cuda_device)
        assert np.array_equal(pw.packed.cpu().numpy(), matmulq.prepack_host(q))


DECODE = [c for c in SEEDED_CASES if c[0].startswith("decode_")]


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("case", DECODE, ids=[c[0] for c in DECODE])
def test_decode_gemv_set(cuda_device, case, mode):
    X, W, b = case_inputs(case)
    q, s = oracle.quantize_per_channel(W)
    Y = run(X, q, s, mode)
    path = matmulq.plan_info(*X.shape, W.shape[1], mode=mode)["path"]
    assert path == "cluster_gemv"
    check(Y, X, q, s, mode)


@pytest.mark.parametrize("path,a_source", [(0, 0), (2, 2), (2, 1), (3, 0), (1, 0)],
                         ids=["auto", "tile_A_tmem", "tile_A_smem", "stream_k", "gemv"])
@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_single_op_with_bias(cuda_device, mode, path, a_source):
    if mode == "fp32" and path in (2, 3):
        pytest.skip("the tensor-core kernels compute in bf16 mode")
    if path == 3:
        # M = 64 exceeds the stream-K kernel's token tile: the library refuses it.
        matmulq.set_option(_lib.OPT_FORCE_PATH, 3)
        try:
            with pytest.raises(_lib.MtrtqError):
                matmulq.plan_info(64, 768, 3072)
        finally:
            matmulq.set_option(_lib.OPT_FORCE_PATH, 0)
        return
    case = SEEDED_CASES[0]
    X, W, b = case_inputs(case)
    q, s = oracle.quantize_per_channel(W)
    matmulq.set_option(_lib.OPT_GEMM_A_SOURCE, a_source)
    matmulq.set_option(_lib.OPT_FORCE_PATH, path)
    try:
        Y = run(X, q, s, mode, bias=b)
    finally:
        matmulq.set_option(_lib.OPT_GEMM_A_SOURCE, 0)
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)
    check(Y, X, q, s, mode, bias=b, tc=(mode == "bf16" and path != 1))


LARGE = [(K, N, M) for (K, N) in wl.LARGE_SHAPES for M in wl.LARGE_M]


@pytest.mark.parametrize("K,N,M", LARGE, ids=[f"{K}x{N}_m{M}" for K, N, M in LARGE])
def test_large_sweep_bf16_activations(cuda_device, K, N, M):
    W = wl.weights(K, N, wl.shape_seed(f"large_{K}x{N}", K, N))
    q, s = matmulq.quantize_per_channel(W)
    X = oracle.round_bf16(wl.activations(M, K, 1000 + M))
    Y = run(X, q, s, "bf16", x_dtype=torch.bfloat16)
    # Rows are independent in the reference loop: check a spread of rows exactly.
    rows = np.unique(np.linspace(0, M - 1, min(M, 12)).astype(np.int64))
    check(Y, X, q, s, "bf16", rows=rows, tc=M > 8)


RAGGED = [(1, 16, 1), (2, 48, 17), (3, 100, 129), (5, 64, 255), (8, 1000, 7), (9, 64, 128),
          (15, 48, 200), (17, 192, 130), (33, 80, 64), (100, 300, 500), (129, 64, 1), (257, 128, 384),
          (300, 200, 129)]


@pytest.mark.parametrize("M,K,N", RAGGED, ids=[f"{M}x{K}x{N}" for M, K, N in RAGGED])
@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_ragged_shapes(cuda_device, M, K, N, mode):
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(0.02)
    X = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((N,), dtype=np.float32) * np.float32(0.02)
    q, s = oracle.quantize_per_channel(W)
    Y = run(X, q, s, mode, bias=b)
    check(Y, X, q, s, mode, bias=b, tc=(mode == "bf16" and M > 8))


@pytest.mark.parametrize("M", [1, 4, 8, 16, 40, 64, 200])
def test_every_path_agrees(cuda_device, M):
    K, N = 768, 1000
    W = wl.weights(K, N, 5)
    q, s = oracle.quantize_per_channel(W)
    X = wl.activations(M, K, 6)
    outs = []
    for path in ((1, 2, 3, 4, 5) if M <= 32 else (1, 2, 4, 5) if M <= 64 else (1, 2)):
        matmulq.set_option(_lib.OPT_FORCE_PATH, path)
        try:
            outs.append(run(X, q, s, "bf16"))
        finally:
            matmulq.set_option(_lib.OPT_FORCE_PATH, 0)
    for Y in outs:
        check(Y, X, q, s, "bf16", tc=True)


@pytest.mark.parametrize("M", [3, 8, 20, 64])
@pytest.mark.parametrize("mode,path", [("fp32", 0), ("bf16", 0), ("fp32", 1), ("fp32", 4), ("bf16", 4)])
def test_nan_activation_poisons_its_row_only(cuda_device, M, mode, path):
    """A NaN activation makes its row's outputs NaN, as in the reference loop (every
    output of the row adds a NaN product), and leaves the other rows exact."""
    K, N = 300, 700
    q, s = oracle.quantize_per_channel(wl.weights(K, N, 81))
    X = wl.activations(M, K, 82)
    X[1, 5] = np.nan
    with forced(path):
        Y = run(X, q, s, mode)
    assert np.all(np.isnan(Y[1]))
    keep = np.arange(M) != 1
    check(Y[keep], X[keep], q, s, mode, tc=(mode == "bf16" and path != 4))


def test_strided_input_and_output(cuda_device):
    M, K, N = 24, 200, 300
    W = wl.weights(K, N, 11)
    q, s = oracle.quantize_per_channel(W)
    X = wl.activations(M, K, 12)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    for mode in ("bf16", "fp32"):
        xbig = torch.zeros((M, K + 56), device=cuda_device)
        xbig[:, :K] = torch.from_numpy(X).to(cuda_device)
        ybig = torch.full((M, N + 20), 7.0, device=cuda_device)
        lib = _lib.lib()
        ws = torch.zeros(max(256, matmulq.workspace_bytes(M, K, N, torch.float32, mode)),
                         dtype=torch.uint8, device=cuda_device)
        rc = lib.mtrtq_matmul(xbig.data_ptr(), 0, K + 56, pw.packed.data_ptr(), pw.scale.data_ptr(),
                              None, ybig.data_ptr(), N + 20, M, K, N, matmulq.MODES[mode],
                              ws.data_ptr(), ws.numel(), None)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        yb = ybig.cpu().numpy()
        assert np.all(yb[:, N:] == 7.0), "wrote outside the [M, N] window"
        check(yb[:, :N], X, q, s, mode, tc=(mode == "bf16"))


PERSISTENT = [(2048, 768, 7168), (300, 1000, 60000), (2048, 4096, 14336), (700, 64, 50257)]


@pytest.mark.parametrize("M,K,N", PERSISTENT, ids=[f"{M}x{K}x{N}" for M, K, N in PERSISTENT])
@pytest.mark.parametrize("epilogue", ["none", "gelu", "residual"])
def test_persistent_gemm(cuda_device, M, K, N, epilogue):
    """The persistent tile GEMM (one CTA per SM, two TMEM accumulators) and its
    stream-K form against the oracle, and against the one-tile-per-CTA kernel on the
    same inputs."""
    if epilogue != "none" and M * N > 2048 * 7168:
        pytest.skip("epilogues are covered on the smaller shapes")
    q, s = matmulq.quantize_per_channel(wl.weights(K, N, 1100 + K))
    X = oracle.round_bf16(wl.activations(M, K, 1101))
    b = wl.bias(N, 1102)
    R = wl.activations(M, N, 1103) if epilogue == "residual" else None
    info = matmulq.plan_info(M, K, N, torch.bfloat16, "bf16")
    assert info["path"] == "gemm_tc" and info["tile_m"] == 256
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    xt = torch.from_numpy(X).to(cuda_device).to(torch.bfloat16)
    bt = torch.from_numpy(b).to(cuda_device)
    outs = []
    # persistent (automatic: at least three tiles per SM), one tile per CTA, stream-K
    for a_source in (0, 2, 3):
        matmulq.set_option(_lib.OPT_GEMM_A_SOURCE, a_source)
        try:
            y = torch.from_numpy(R).to(cuda_device) if R is not None else torch.full((M, N), float("nan"),
                                                                                       device=cuda_device)
            matmul_q8(xt, pw, bias=bt, out=y, mode="bf16", epilogue=epilogue,
                      residual=y if epilogue == "residual" else None)
            torch.cuda.synchronize()
        finally:
            matmulq.set_option(_lib.OPT_GEMM_A_SOURCE, 0)
        assert matmulq.read_device_status() == 0
        outs.append(y.cpu().numpy())
    # the oracle on sampled rows (first and last token tiles included); the kernels
    # against each other on every element
    rows = np.unique(np.concatenate([np.arange(min(M, 8)), np.linspace(0, M - 1, 12).astype(np.int64),
                                     np.arange(max(0, M - 4), M)]))
    t = oracle.matmul_q8_rows(X, q, s, rows, b)
    if epilogue == "gelu":
        u = t.astype(np.float64)
        t = (0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))).astype(np.float32)
    elif epilogue == "residual":
        t = (R[rows] + t).astype(np.float32)
    assert np.all(np.isfinite(outs[0]))
    assert rel_err(outs[0][rows], t) <= BF16_SAME_INPUT_TOL_TC
    assert rel_err(outs[0], outs[1]) <= 1e-6
    # stream-K adds the fp32 parts of a cut tile (a different summation order)
    assert np.all(np.isfinite(outs[2])) and rel_err(outs[2][rows], t) <= BF16_SAME_INPUT_TOL_TC
    assert rel_err(outs[2], outs[1]) <= 1e-5


@pytest.mark.parametrize("M", [1, 8, 64, 2048])
def test_results_are_deterministic(cuda_device, M):
    K, N = 4096, 4096
    W = wl.weights(K, N, 21)
    q, s = matmulq.quantize_per_channel(W)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    x = torch.randn(M, K, device=cuda_device, generator=torch.Generator(cuda_device).manual_seed(3))
    a = matmul_q8(x, pw).clone()
    b = matmul_q8(x, pw).clone()
    assert torch.equal(a, b)


def test_registry_device_kernel_matches_golden(cuda_device):
    """Golden.MatMulQ (tests/golden_kernel_test.cpp:155-175) run through the device
    registry entry: lookup("MatMulQ", kF32) -> fn(OpContext)."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "matmulq_op.npz"))
    reg = registry.KernelRegistry()
    registry.register_cuda_kernels(reg)
    assert reg.lookup("MatMulQ", registry.DType.kF32) is not None
    assert reg.lookup("MatMulQ", registry.DType.kI8) is None
    A = torch.from_numpy(g["a"]).to(cuda_device)
    W = torch.from_numpy(g["q"]).to(cuda_device)
    s = torch.from_numpy(g["s"]).to(cuda_device)
    for mode in ("fp32", "bf16"):
        out = torch.empty((2, 5), device=cuda_device)
        registry.run_kernel(reg, "MatMulQ", [A, W, s], out, {"mode": mode})
        got = out.cpu().numpy()
        if mode == "fp32":
            assert rel_err(got, g["c_ref"]) <= FP32_TOL
        assert np.allclose(got, g["out"], rtol=0.05, atol=0.05)
    with pytest.raises(registry.GraphError):
        registry.run_kernel(reg, "MatMulQ", [A, W], torch.empty((2, 5), device=cuda_device))
    # host tensors, as the reference's executor passes them: copied in and out
    for mode in ("fp32", "bf16"):
        out = torch.full((2, 5), float("nan"))
        registry.run_kernel(reg, "MatMulQ", [A.cpu(), W.cpu(), s.cpu()], out, {"mode": mode})
        if mode == "fp32":
            assert rel_err(out.numpy(), g["c_ref"]) <= FP32_TOL
        assert np.allclose(out.numpy(), g["out"], rtol=0.05, atol=0.05)


def test_argument_errors_on_device(cuda_device):
    W = wl.weights(64, 64, 1)
    pw = PackedWeight.from_float(W, cuda_device)
    x = torch.randn(4, 64, device=cuda_device)
    with pytest.raises(ValueError):
        matmul_q8(torch.randn(4, 65, device=cuda_device), pw)
    lib = _lib.lib()
    y = torch.empty(4, 64, device=cuda_device)
    # misaligned packed weights
    rc = lib.mtrtq_matmul(x.data_ptr(), 0, 64, pw.packed.data_ptr() + 16, pw.scale.data_ptr(), None,
                          y.data_ptr(), 64, 4, 64, 64, 0, None, 0, None)
    assert rc == _lib.ERR_ALIGNMENT
    # workspace too small for a split plan
    need = matmulq.workspace_bytes(4, 64, 64, torch.float32, "bf16")
    if need > 0:
        rc = lib.mtrtq_matmul(x.data_ptr(), 0, 64, pw.packed.data_ptr(), pw.scale.data_ptr(), None,
                              y.data_ptr(), 64, 4, 64, 64, 0, None, 0, None)
        assert rc == _lib.ERR_WORKSPACE


def test_one_workspace_serves_every_shape(cuda_device):
    """Calls of different shapes share one workspace: split-K tickets of a call
    with many channel tiles must not meet another call's leftover partials."""
    ws = matmulq.Workspace(cuda_device)
    seq = [(8, 768, 768), (1, 768, 50257), (64, 768, 3072), (1, 4096, 11008), (16, 4096, 11008),
           (8, 3072, 768), (1, 768, 50257), (300, 200, 129), (2, 768, 50257)]
    for i, (M, K, N) in enumerate(seq):
        W = wl.weights(K, N, 100 + i)
        q, s = matmulq.quantize_per_channel(W)
        X = wl.activations(M, K, 200 + i)
        pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
        for mode in ("fp32", "bf16"):
            y = torch.full((M, N), float("nan"), device=cuda_device)
            matmul_q8(torch.from_numpy(X).to(cuda_device), pw, out=y, mode=mode, workspace=ws)
            check(y.cpu().numpy(), X, q, s, mode, tc=(mode == "bf16" and M > 8))


@pytest.mark.parametrize("M", [3, 8, 24])
def test_gemv_restages_activations_in_chunks(cuda_device, M):
    # fp32 mode, K = 14336: each CTA's k range spans several staged chunks.
    K, N = 14336, 512
    W = wl.weights(K, N, 31)
    q, s = matmulq.quantize_per_channel(W)
    X = wl.activations(M, K, 32)
    with forced(1):
        Y = run(X, q, s, "fp32")
    check(Y, X, q, s, "fp32")


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K", [100, 77])
def test_stream_k_with_unaligned_rows(cuda_device, x_dtype, K):
    # Row strides that are not a multiple of 16 bytes cannot be read by TMA: the
    # library stages a bf16 copy first. Same results either way.
    M, N = 5, 300
    W = wl.weights(K, N, 41)
    q, s = oracle.quantize_per_channel(W)
    X = oracle.round_bf16(wl.activations(M, K, 42))
    with forced(3):
        Y = run(X, q, s, "bf16", x_dtype=x_dtype)
    check(Y, X, q, s, "bf16", tc=True)


@pytest.mark.parametrize("M,K,N", [(1, 64, 128), (3, 64, 50257), (8, 12288, 256), (32, 4096, 640),
                                   (17, 192, 129), (16, 20000, 100), (5, 64 * 23, 128 * 7)])
def test_stream_k_partitions(cuda_device, M, K, N):
    """Tiles cut by CTA boundaries in every way: one unit per CTA, many tiles per
    CTA, tiles spread over many CTAs, ragged K and N."""
    W = wl.weights(K, N, 51)
    q, s = matmulq.quantize_per_channel(W)
    X = wl.activations(M, K, 52)
    b = wl.bias(N, 53)
    with forced(3):
        Y = run(X, q, s, "bf16", bias=b)
        assert matmulq.plan_info(M, K, N)["path"] == "stream_k_tc"
    check(Y, X, q, s, "bf16", bias=b, tc=True)


GSK_CASES = [(12, 768, 3072), (16, 768, 50257), (24, 4096, 1000), (32, 3072, 768), (9, 100, 300),
             (31, 77, 129), (64, 768, 3072), (40, 768, 3072), (40, 100, 300), (33, 4096, 1000), (64, 4096, 14336),
             (57, 77, 129),
             (1, 64, 128), (3, 64, 50257), (8, 12288, 256), (2, 4096, 14336), (1, 768, 50257),
             (5, 64 * 23, 128 * 7), (7, 12000, 100), (8, 4096, 1000), (4, 100, 300), (6, 77, 129)]


DECODE_PATHS = {4: "cluster_gemv", 5: "gemv_stream"}


@pytest.mark.parametrize("M,K,N", GSK_CASES, ids=[f"{M}x{K}x{N}" for M, K, N in GSK_CASES])
@pytest.mark.parametrize("mode", ["bf16", "fp32"])
@pytest.mark.parametrize("path", sorted(DECODE_PATHS), ids=list(DECODE_PATHS.values()))
def test_decode_gemv_partitions(cuda_device, M, K, N, mode, path):
    """The CUDA-core decode GEMVs: one unit per CTA, tiles spread over many CTAs,
    several tiles per CTA, ragged K and N, clusters of 1 to 8 CTAs."""
    W = wl.weights(K, N, 61)
    q, s = matmulq.quantize_per_channel(W)
    X = wl.activations(M, K, 62)
    b = wl.bias(N, 63)
    matmulq.set_option(_lib.OPT_FORCE_PATH, path)
    try:
        assert matmulq.plan_info(M, K, N, mode=mode)["path"] == DECODE_PATHS[path]
        Y = run(X, q, s, mode, bias=b)
        Y2 = run(X, q, s, mode, bias=b)
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)
    rows = np.arange(M)
    check(Y, X, q, s, mode, bias=b, rows=rows if N * K > 50_000_000 else None)
    assert np.array_equal(Y, Y2), "stream-K GEMV results must not depend on CTA timing"


@pytest.mark.parametrize("x_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("path", sorted(DECODE_PATHS), ids=list(DECODE_PATHS.values()))
def test_decode_gemv_strided(cuda_device, x_dtype, path):
    M, K, N = 6, 300, 700
    W = wl.weights(K, N, 71)
    q, s = matmulq.quantize_per_channel(W)
    X = oracle.round_bf16(wl.activations(M, K, 72))
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), "cuda")
    xbig = torch.zeros((M, K + 13), device="cuda", dtype=x_dtype)
    xbig[:, :K] = torch.from_numpy(X).to(x_dtype)
    ybig = torch.full((M, N + 5), float("nan"), device="cuda")
    matmulq.set_option(_lib.OPT_FORCE_PATH, path)
    try:
        matmul_q8(xbig[:, :K], pw, out=ybig[:, :N], mode="bf16")
    finally:
        matmulq.set_option(_lib.OPT_FORCE_PATH, 0)
    torch.cuda.synchronize()
    assert torch.isnan(ybig[:, N:]).all()
    check(ybig[:, :N].cpu().numpy(), X, q, s, "bf16")


@pytest.mark.parametrize("graph", [False, True], ids=["stream", "graph"])
def test_overlapped_launches_wait_for_their_inputs(cuda_device, graph):
    """With MTRTQ_OPT_OVERLAP_LAUNCH a cluster GEMV may start before the kernel ahead
    of it finishes. A chain where each call reads the previous call's output, whose
    buffer another kernel has just refilled with NaN, must still see every input
    complete."""
    K = N = 768
    M = 2
    qs = []
    for i in range(3):
        q, s = oracle.quantize_per_channel(wl.weights(K, N, 80 + i))
        qs.append((q, s, PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), "cuda")))
    x = torch.from_numpy(wl.activations(M, K, 90)).cuda()
    ys = [torch.empty((M, N), device="cuda") for _ in range(3)]

    def chain():
        for y in ys:
            y.fill_(float("nan"))
        inp = x
        for (_, _, pw), y in zip(qs, ys):
            matmul_q8(inp, pw, out=y, mode="fp32")
            inp = y

    matmulq.set_option(_lib.OPT_OVERLAP_LAUNCH, 1)
    try:
        with forced(4):
            chain()  # first calls (per-device setup) outside any capture
            torch.cuda.synchronize()
            if graph:
                g = torch.cuda.CUDAGraph()
                st = torch.cuda.Stream()
                with torch.cuda.stream(st):
                    with torch.cuda.graph(g, stream=st):
                        chain()
                for _ in range(3):
                    g.replay()
            else:
                for _ in range(3):
                    chain()
            torch.cuda.synchronize()
    finally:
        matmulq.set_option(_lib.OPT_OVERLAP_LAUNCH, 0)
    assert matmulq.read_device_status() == 0
    inp = x.cpu().numpy()
    for (q, s, _), y in zip(qs, ys):
        out = y.cpu().numpy()
        assert np.all(np.isfinite(out)), "a call read its input before it was written"
        err = rel_err(out, oracle.matmul_q8(inp, q, s))
        assert err <= FP32_TOL, f"fp32 mode rel err {err:.3e}"
        inp = out


EPI_PATHS = {1: "gemv", 2: "gemm_tc", 3: "stream_k_tc", 4: "cluster_gemv", 5: "gemv_stream"}
EPI_CASES = [(1, 768, 3072), (8, 3072, 768), (24, 768, 1000), (64, 768, 3072)]


def _gelu_new(u):
    u = u.astype(np.float64)
    return (0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))).astype(np.float32)


@pytest.mark.parametrize("M,K,N", EPI_CASES, ids=[f"{M}x{K}x{N}" for M, K, N in EPI_CASES])
@pytest.mark.parametrize("path", sorted(EPI_PATHS), ids=list(EPI_PATHS.values()))
@pytest.mark.parametrize("epilogue", ["gelu", "residual"])
def test_fused_epilogues(cuda_device, M, K, N, path, epilogue):
    """gelu_new after the bias (the reference's FusedMatMulBiasGeluTanh) and the
    residual add (in place: out is the residual), on every kernel that takes the shape."""
    mode = "fp32" if path == 1 else "bf16"
    if (path == 3 and M > 32) or (path in (4, 5) and M > 64):
        pytest.skip("the kernel does not take this M")
    W = wl.weights(K, N, 601)
    q, s = matmulq.quantize_per_channel(W)
    X = oracle.round_bf16(wl.activations(M, K, 602)) if mode == "bf16" else wl.activations(M, K, 602)
    b = wl.bias(N, 603)
    R = wl.activations(M, N, 604)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    x = torch.from_numpy(X).to(cuda_device)
    bt = torch.from_numpy(b).to(cuda_device)
    y = torch.from_numpy(R).to(cuda_device).clone()
    with forced(path):
        if epilogue == "gelu":
            matmul_q8(x, pw, bias=bt, out=y, mode=mode, epilogue="gelu")
        else:
            matmul_q8(x, pw, bias=bt, out=y, mode=mode, epilogue="residual", residual=y)
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    t = oracle.matmul_q8(X, q, s, b)
    want = _gelu_new(t) if epilogue == "gelu" else (R + t).astype(np.float32)
    err = rel_err(y.cpu().numpy(), want)
    assert err <= (1e-4 if path in (1, 4, 5) else 1e-3), f"rel err {err:.3e}"


@pytest.mark.parametrize("M,K,N", [(1, 768, 2304), (8, 768, 50257), (64, 768, 3072), (300, 1000, 520)])
@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
def test_host_buffers(cuda_device, M, K, N, pinned):
    """mtrtq_matmul_host: X and Y in host memory, copies and product on one stream."""
    W = wl.weights(K, N, 90 + M)
    q, s = oracle.quantize_per_channel(W)
    bias = wl.activations(1, N, 91)[0]
    X = wl.activations(M, K, 92 + M)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    bt = torch.from_numpy(bias).to(cuda_device)
    xh = torch.from_numpy(X)
    if pinned:
        xh = xh.pin_memory()
    for mode in ("bf16", "fp32"):
        Y = matmulq.matmul_q8_host(xh, pw, bias=bt, mode=mode)
        assert Y.device.type == "cpu"
        assert matmulq.read_device_status() == 0
        check(Y.numpy(), X, q, s, mode, bias=bias, tc=(mode == "bf16"))
    # non-blocking: results appear after the stream is synchronized
    st = torch.cuda.Stream(cuda_device)
    out = torch.full((M, N), float("nan"), pin_memory=pinned)
    matmulq.matmul_q8_host(xh, pw, bias=bt, out=out, mode="fp32", stream=st, blocking=False)
    st.synchronize()
    check(out.numpy(), X, q, s, "fp32", bias=bias)


def test_host_buffers_argument_errors(cuda_device):
    q, s = oracle.quantize_per_channel(wl.weights(64, 128, 93))
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    lib = _lib.lib()
    x = torch.zeros(2, 64)
    y = torch.zeros(2, 128)
    need = matmulq.host_workspace_bytes(2, 64, 128)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    args = lambda wsb: (x.data_ptr(), pw.packed.data_ptr(), pw.scale.data_ptr(), None, y.data_ptr(),
                        2, 64, 128, _lib.MODE_BF16, ws.data_ptr(), wsb, 1, None)
    assert lib.mtrtq_matmul_host(*args(need - 1)) == _lib.ERR_WORKSPACE
    assert lib.mtrtq_matmul_host(*args(need)) == 0
    bad = list(args(need))
    bad[0] = None
    assert lib.mtrtq_matmul_host(*bad) == _lib.ERR_INVALID_ARG


def test_host_call_leaves_shared_workspace_counters(cuda_device):
    """A host-buffer call whose plan needs no scratch still stages X and Y past the
    counter region, so a split-K call on the same workspace stays correct."""
    K, N = 768, 2304
    q, s = oracle.quantize_per_channel(wl.weights(K, N, 94))
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    ws = torch.zeros(max(matmulq.host_workspace_bytes(1, K, N),
                         matmulq.workspace_bytes(3, K, N, torch.float32, "fp32") + (1 << 20)),
                     dtype=torch.uint8, device=cuda_device)
    X = wl.activations(3, K, 95)
    matmulq.matmul_q8_host(torch.from_numpy(X[:1]), pw, mode="bf16", workspace=ws)
    with forced(1):
        y = torch.full((3, N), float("nan"), device=cuda_device)
        matmul_q8(torch.from_numpy(X).to(cuda_device), pw, out=y, mode="fp32", workspace=ws)
        torch.cuda.synchronize()
    check(y.cpu().numpy(), X, q, s, "fp32")


def _layernorm(x, g, b, eps):
    """The reference's LayerNorm (src/ops/kernels_transformer.cpp:38-52) in fp32."""
    mean = x.mean(axis=1, keepdims=True, dtype=np.float32)
    c = (x - mean).astype(np.float32)
    var = (c * c).mean(axis=1, keepdims=True, dtype=np.float32)
    return (c * (np.float32(1.0) / np.sqrt(var + np.float32(eps))) * g + b).astype(np.float32)


LN_CASES = [(1, 768, 2304), (8, 768, 3072), (3, 100, 300), (16, 768, 768), (32, 768, 3072), (8, 4096, 1000),
            (5, 1000, 520), (8, 768, 50257), (64, 768, 3072), (41, 768, 768)]


@pytest.mark.parametrize("M,K,N", LN_CASES, ids=[f"{M}x{K}x{N}" for M, K, N in LN_CASES])
@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("epilogue", ["none", "gelu", "residual"])
def test_layernorm_prologue(cuda_device, M, K, N, mode, epilogue):
    """mtrtq_matmul_ln_ex: LayerNorm of each row, then MatMulQ (+ bias, epilogue), in
    one cluster GEMV; against the reference's LayerNorm and MatMulQ on the CPU."""
    if not matmulq.supports_ln(M, K, N, mode):
        pytest.skip("shape plans another kernel")
    W = wl.weights(K, N, 700 + M)
    q, s = matmulq.quantize_per_channel(W)
    rng = np.random.default_rng(701 + M)
    X = (rng.standard_normal((M, K)) * 3 + 0.5).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    be = (0.1 * rng.standard_normal(K)).astype(np.float32)
    b = wl.bias(N, 702)
    R = wl.activations(M, N, 703)
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    T = lambda a: torch.from_numpy(a).to(cuda_device)
    # contiguous rows (16-byte loads) for even M, a padded stride (element loads) for odd M
    ldx = K + 13 if M % 2 else K
    xb = torch.zeros((M, ldx), device=cuda_device)
    xb[:, :K] = T(X)
    y = T(R).clone() if epilogue == "residual" else torch.full((M, N), float("nan"), device=cuda_device)
    matmulq.matmul_q8_ln(xb[:, :K], T(g), T(be), 1e-5, pw, bias=T(b), out=y, mode=mode, epilogue=epilogue,
                         residual=y if epilogue == "residual" else None)
    torch.cuda.synchronize()
    assert matmulq.read_device_status() == 0
    H = _layernorm(X, g, be, 1e-5)

    def finish(t):
        if epilogue == "gelu":
            u = t.astype(np.float64)
            return (0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))).astype(np.float32)
        return (R + t).astype(np.float32) if epilogue == "residual" else t

    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    err = rel_err(got, finish(oracle.matmul_q8(H, q, s, b)))
    if mode == "fp32":
        assert err <= FP32_TOL, f"fp32 rel err {err:.3e}"
    else:
        assert err <= BF16_SPEC_TOL, f"bf16 rel err {err:.3e}"
        errb = rel_err(got, finish(oracle.matmul_q8(oracle.round_bf16(H), q, s, b)))
        assert errb <= 2e-3, f"bf16 rel err vs rounded LayerNorm output {errb:.3e}"


def test_layernorm_prologue_refuses_other_kernels(cuda_device):
    q, s = matmulq.quantize_per_channel(wl.weights(768, 768, 710))
    pw = PackedWeight.from_int8(torch.from_numpy(q), torch.from_numpy(s), cuda_device)
    x = torch.zeros((65, 768), device=cuda_device)
    g = torch.ones(768, device=cuda_device)
    with pytest.raises(_lib.MtrtqError, match="decode GEMVs"):
        matmulq.matmul_q8_ln(x, g, g, 1e-5, pw)  # M = 65: the tile GEMM
    with forced(1):
        with pytest.raises(_lib.MtrtqError, match="decode GEMVs"):
            matmulq.matmul_q8_ln(x[:4], g, g, 1e-5, pw)
