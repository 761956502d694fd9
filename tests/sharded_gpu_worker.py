"""One rank of the multi-GPU sharded MatMulQ test (launched by torch.distributed.run
from tests/test_sharded.py). Checks the full Y of every case against the oracle,
through the NCCL path (ShardedMatMulQ) and the library's own peer-memory exchange
(P2PShardedMatMulQ, several calls in a row with new activations each), and prints
SHARDED OK."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import oracle  # noqa: E402
from mini_tensorrt_b200 import matmulq, sharded, workloads as wl  # noqa: E402
from tests.conftest import rel_err  # noqa: E402

CASES = [("N", 8, 768, 50257), ("K", 8, 768, 50257), ("N", 1, 4096, 14336), ("K", 2, 4096, 4096),
         ("N", 64, 768, 3072), ("K", 64, 3072, 768), ("N", 3, 200, 300)]


def main():
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    try:
        for i, (split, M, K, N) in enumerate(CASES):
            W = wl.weights(K, N, 100 + i)
            q, s = oracle.quantize_per_channel(W)
            b = wl.bias(N, 200 + i)
            X = wl.activations(M, K, 300 + i)
            op = sharded.ShardedMatMulQ(q, s, b, split=split, mode="fp32")
            y = op(torch.from_numpy(X).cuda()).cpu().numpy()
            rows = np.unique(np.linspace(0, M - 1, min(M, 8)).astype(np.int64))
            ref = oracle.matmul_q8_rows(X, q, s, rows, b)
            err = rel_err(y[rows], ref)
            assert np.isfinite(y).all(), f"case {i}: non-finite output"
            assert err <= 1e-4, f"rank {rank} case {i} ({split}, {M}x{K}x{N}): rel err {err:.3e}"
        for i, (split, M, K, N) in enumerate(CASES):
            W = wl.weights(K, N, 400 + i)
            q, s = oracle.quantize_per_channel(W)
            b = wl.bias(N, 500 + i)
            op = sharded.P2PShardedMatMulQ(q, s, b, split=split, mode="fp32", max_m=M)
            rows = np.unique(np.linspace(0, M - 1, min(M, 8)).astype(np.int64))
            for call in range(3):  # epochs 1..3: the entry barrier guards each call's buffers
                X = wl.activations(M, K, 600 + 10 * i + call)
                y = op(torch.from_numpy(X).cuda()).cpu().numpy()
                assert np.isfinite(y).all(), f"p2p case {i} call {call}: non-finite output"
                err = rel_err(y[rows], oracle.matmul_q8_rows(X, q, s, rows, b))
                assert err <= 1e-4, f"rank {rank} p2p case {i} call {call} ({split}, {M}x{K}x{N}): {err:.3e}"
                # every rank holds the same bits (N: the same columns; K: sums in rank order)
                t = torch.from_numpy(y).cuda()
                allt = [torch.empty_like(t) for _ in range(dist.get_world_size())]
                dist.all_gather(allt, t)
                assert all(torch.equal(allt[0], a) for a in allt), f"p2p case {i}: ranks disagree"
            torch.cuda.synchronize()
            op.close()
        torch.cuda.synchronize()
        assert matmulq.read_device_status() == 0
        print("SHARDED OK", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
