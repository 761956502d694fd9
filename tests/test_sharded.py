"""Sharded MatMulQ (mini_tensorrt_b200.sharded) across ranks.

CPU: world-size 2 and 3 gloo process groups, with the oracle as each rank's local
product, check the host logic (shard ranges, the all-gather reassembly of uneven
column shards, the K-split partials summed by all-reduce with the bias added
once) against the oracle on the whole weight.

GPU: the same with libmtrtq on two GPUs over NCCL (skipped with fewer GPUs).
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from mini_tensorrt_b200 import sharded, workloads as wl
from tests.conftest import rel_err

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_and_align():
    for total, world, q in [(300, 2, 128), (50257, 8, 128), (200, 3, 64), (64, 4, 64), (4096, 8, 64)]:
        r = sharded.shard_ranges(total, world, q)
        assert r[0][0] == 0 and r[-1][1] == total
        for (b0, e0), (b1, e1) in zip(r, r[1:]):
            assert e0 == b1
        for b, e in r:
            assert b % q == 0 and b <= e
    assert sharded.shard_ranges(64, 4, 64) == [(0, 0), (0, 0), (0, 0), (0, 64)]
    assert sharded.shard_ranges(300, 2, 128) == [(0, 128), (128, 300)]


CASES = [("N", 2, 5, 200, 300), ("K", 3, 2, 1000, 130)]


def _cpu_worker(rank, world, port, split, M, K, N, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = wl.weights(K, N, 7)
        qm, s = oracle.quantize_per_channel(W)
        b = wl.bias(N, 8)
        X = wl.activations(M, K, 9)

        def pack(qs, ss, device):
            return (np.ascontiguousarray(qs), np.ascontiguousarray(ss))

        def local(x, w, bias, mode):
            y = oracle.matmul_q8(x.numpy(), w[0], w[1], None if bias is None else bias.numpy())
            return torch.from_numpy(y)

        op = sharded.ShardedMatMulQ(qm, s, b, split=split, device="cpu", mode="fp32",
                                    local_matmul=local, pack=pack)
        y = op(torch.from_numpy(X)).numpy()
        ref = oracle.matmul_q8(X, qm, s, b)
        err = rel_err(y, ref)
        q.put((rank, float(err), bool(np.isfinite(y).all())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split,world,M,K,N", CASES,
                         ids=[f"{s}_w{w}_{M}x{K}x{N}" for s, w, M, K, N in CASES])
def test_sharded_host_logic_matches_oracle(split, world, M, K, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, split, M, K, N, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=180))
    finally:
        for p in procs:
            if p.is_alive() and len(results) < world:
                p.kill()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, finite in results:
        assert finite
        # N split: each column is the same computation as unsplit (bit-exact);
        # K split: scaled partials add in another order (fp32 rounding, far
        # inside the 1e-4 fp32-mode bar).
        assert err <= (0.0 if split == "N" else 1e-5), f"rank {rank}: {err:.3e}"


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_sharded_on_two_gpus():
    """torchrun-style launch of two ranks over NCCL; each checks the full Y."""
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "tests", "sharded_gpu_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("SHARDED OK") == 2, r.stdout[-3000:]


@pytest.mark.parametrize("extent,world", [(50257, 2), (50257, 8), (768, 3), (100, 8), (14336, 4), (1, 1)])
def test_abi_shard_range_matches_host_split(extent, world):
    """mtrtq_shard_range (the C ABI's split) is the host split the NCCL path uses."""
    for split, quantum in (("N", sharded.TILE_N), ("K", sharded.UNIT_K)):
        want = sharded.shard_ranges(extent, world, quantum)
        got = [sharded.shard_range(extent, split, r, world) for r in range(world)]
        assert got == want


def test_sharded_abi_argument_errors():
    import ctypes
    from mini_tensorrt_b200 import _lib
    lib = _lib.lib()
    comm = _lib.ShardComm()
    comm.rank, comm.world = 0, 2
    x = (ctypes.c_float * 64)()
    call = lambda c, epoch=1, split=_lib.SPLIT_N: lib.mtrtq_matmul_sharded(
        x, 0, 8, x, x, None, x, 8, 1, 8, 8, 1, split, ctypes.byref(c), epoch, None, 0, None)
    assert call(comm) == _lib.ERR_INVALID_ARG                      # no peer buffers
    assert "peer's Y" in _lib.last_error()
    assert call(comm, split=_lib.SPLIT_K) == _lib.ERR_INVALID_ARG
    assert "slots" in _lib.last_error()
    comm.y[1] = 0x1000  # never dereferenced: the flags check fails first
    assert call(comm) == _lib.ERR_INVALID_ARG
    assert "flags" in _lib.last_error()
    comm.world = 9
    assert call(comm) == _lib.ERR_INVALID_ARG
    assert lib.mtrtq_matmul_sharded(x, 0, 8, x, x, None, x, 8, 1, 8, 8, 1, 0, None, 1, None, 0, None) \
        == _lib.ERR_INVALID_ARG
    assert lib.mtrtq_shard_slot_bytes(4, 10, 2) == 4 * 10 * 2 * 4
    assert lib.mtrtq_shard_slot_bytes(4, 10, 9) == -1


def test_group_allgather_argument_errors():
    """mtrtq_gemv_group_allgather refuses, before any device work: a null or
    out-of-range communicator, a non-alternating one (it has no entry barrier),
    and missing peer buffers."""
    import ctypes
    from mini_tensorrt_b200 import _lib
    lib = _lib.lib()
    probs = (_lib.GemvProblem * 1)()
    call = lambda c: lib.mtrtq_gemv_group_allgather(probs, 1, _lib.DTYPE_F32, _lib.MODE_FP32, None, 0,
                                                    ctypes.byref(c) if c is not None else None, 0, None)
    assert call(None) == _lib.ERR_INVALID_ARG
    comm = _lib.ShardComm()
    comm.rank, comm.world = 2, 2
    assert call(comm) == _lib.ERR_INVALID_ARG and "out of range" in _lib.last_error()
    comm.rank = 0
    assert call(comm) == _lib.ERR_INVALID_ARG and "alternating" in _lib.last_error()
    comm.alternating = 1
    assert call(comm) == _lib.ERR_INVALID_ARG and "null output or flag" in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("split", ["N", "K"])
def test_p2p_sharded_single_rank(cuda_device, split):
    """mtrtq_matmul_sharded with one rank (no process group): the local product and,
    for split K, the slot reduction, against the oracle."""
    M, K, N = 5, 768, 3000
    W = wl.weights(K, N, 31)
    q, s = oracle.quantize_per_channel(W)
    b = wl.bias(N, 32)
    op = sharded.P2PShardedMatMulQ(q, s, b, split=split, mode="fp32", max_m=8, device=cuda_device)
    for call in range(2):
        X = wl.activations(M, K, 33 + call)
        y = op(torch.from_numpy(X).to(cuda_device)).cpu().numpy()
        assert rel_err(y, oracle.matmul_q8(X, q, s, b)) <= 1e-4
    op.close()
