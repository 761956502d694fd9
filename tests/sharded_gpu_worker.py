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
        # the exchange steps on their own: segments of a peer buffer, partials + residual
        world = dist.get_world_size()
        M, N = 5, 37
        pb = sharded.PeerBuffers(y_elems=4096, slot_elems=M * N * world)
        for call in range(3):
            base = torch.arange(4096, dtype=torch.float32, device="cuda") * (call + 1)
            # rank r owns rows r, r + world, ... of a [24, 100] block at offset 17 (ld 120)
            segs = []
            for row in range(rank, 24, world):
                segs.append((17 + row * 120, 1, 100, 100))
                pb.y[17 + row * 120:17 + row * 120 + 100] = base[17 + row * 120:17 + row * 120 + 100]
            pb.allgather(segs)
            torch.cuda.synchronize()
            got = pb.y[17:17 + 24 * 120].view(24, 120)[:, :100]
            assert torch.equal(got, base[17:17 + 24 * 120].view(24, 120)[:, :100]), f"allgather call {call}"
            g = torch.Generator(device="cuda").manual_seed(100 * call + rank)
            partial = pb.slot(M, N)
            partial.copy_(torch.randn(M, N, device="cuda", generator=g))
            res = torch.full((M, N), float(call), device="cuda")
            bias = torch.arange(N, dtype=torch.float32, device="cuda")
            out = torch.empty(M, N, device="cuda")
            pb.allreduce(partial, out, bias=bias, residual=res)
            torch.cuda.synchronize()
            parts = []
            for r in range(world):
                gr = torch.Generator(device="cuda").manual_seed(100 * call + r)
                parts.append(torch.randn(M, N, device="cuda", generator=gr))
            want = parts[0].clone()
            for r in range(1, world):
                want += parts[r]
            want = res + (want + bias)
            assert torch.equal(out, want), f"allreduce call {call}: {float((out - want).abs().max())}"
        pb.close()
        # alternating buffers (no entry barrier): all-reduces back to back
        pa = sharded.PeerBuffers(y_elems=64, slot_elems=M * N * world, alternating=True)
        for call in range(6):
            partial = pa.slot(M, N)
            partial.fill_(float(rank * 10 + call))
            out = torch.empty(M, N, device="cuda")
            pa.allreduce(partial, out)
            torch.cuda.synchronize()
            want = float(sum(r * 10 + call for r in range(world)))
            assert torch.all(out == want), f"alternating all-reduce {call}"
        pa.close()
        # the grouped GEMV with its all-gather fused in: every rank computes its column
        # shard of three problems straight into its half of the output buffer and
        # the peers'; eager calls (host epochs) alternate the halves, then a captured
        # pair of calls (device epochs) is replayed
        fused_shapes = [(8, 768, 2304), (1, 768, 50257), (3, 100, 300), (40, 1000, 1500)]
        y_elems = sum(M_ * N_ for M_, _, N_ in fused_shapes)
        for device_epochs in (False, True):
            pf = sharded.PeerBuffers(y_elems, 0, device_epochs=device_epochs, alternating=True)
            probs, off = [], 0
            for j, (M_, K_, N_) in enumerate(fused_shapes):
                q_, s_ = oracle.quantize_per_channel(wl.weights(K_, N_, 700 + j))
                n0, n1 = sharded.shard_range(N_, "N", rank, world)
                w_ = matmulq.PackedWeight.from_int8(torch.from_numpy(np.ascontiguousarray(q_[:, n0:n1])),
                                                    torch.from_numpy(np.ascontiguousarray(s_[n0:n1])), "cuda")
                probs.append((M_, K_, N_, q_, s_, n0, n1, w_, off))
                off += M_ * N_

            def make_group(h, xs):
                items = []
                for (M_, K_, N_, q_, s_, n0, n1, w_, o), x in zip(probs, xs):
                    if n1 > n0:
                        yv = pf.y[h * y_elems + o:h * y_elems + o + M_ * N_].view(M_, N_)
                        items.append({"x": x, "w": w_, "out": yv[:, n0:n1]})
                return matmulq.GemvGroup(items, mode="fp32")

            def check_half(h, xs_host, tag):
                for (M_, K_, N_, q_, s_, n0, n1, w_, o), X_ in zip(probs, xs_host):
                    got = pf.y[h * y_elems + o:h * y_elems + o + M_ * N_].view(M_, N_).cpu().numpy()
                    rows = np.unique(np.linspace(0, M_ - 1, min(M_, 4)).astype(np.int64))
                    err = rel_err(got[rows], oracle.matmul_q8_rows(X_, q_, s_, rows))
                    assert np.isfinite(got).all() and err <= 1e-4, f"fused all-gather {tag} {M_}x{K_}x{N_}: {err:.3e}"

            xs_host = [[wl.activations(M_, K_, 800 + 10 * h + j) for j, (M_, K_, N_) in enumerate(fused_shapes)]
                       for h in range(2)]
            xs = [[torch.from_numpy(a).cuda() for a in xs_host[h]] for h in range(2)]
            groups = [make_group(h, xs[h]) for h in range(2)]
            if not device_epochs:
                for call in range(4):
                    h = call % 2
                    pf.y[h * y_elems:(h + 1) * y_elems].fill_(float("nan"))
                    dist.barrier()
                    pf.group_allgather(groups[h])
                    torch.cuda.synchronize()
                    check_half(h, xs_host[h], f"call {call}")
                    dist.barrier()
            else:
                st = torch.cuda.Stream()
                with torch.cuda.stream(st):
                    pf.group_allgather(groups[0], stream=st)
                    pf.group_allgather(groups[1], stream=st)
                    torch.cuda.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=st):
                        pf.group_allgather(groups[0], stream=st)
                        pf.group_allgather(groups[1], stream=st)
                    for call in range(3):
                        pf.y.fill_(float("nan"))
                        torch.cuda.synchronize()
                        dist.barrier()
                        graph.replay()
                        torch.cuda.synchronize()
                        check_half(0, xs_host[0], f"graph replay {call} half 0")
                        check_half(1, xs_host[1], f"graph replay {call} half 1")
                        dist.barrier()
                del graph
            pf.close()
        # device-counted epochs: one all-reduce captured in a CUDA graph, replayed
        pg = sharded.PeerBuffers(y_elems=64, slot_elems=M * N * world, device_epochs=True)
        partial, out = pg.slot(M, N), torch.empty(M, N, device="cuda")
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            partial.fill_(1.0)
            pg.allreduce(partial, out, stream=st)  # epoch 1, eager
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                pg.allreduce(partial, out, stream=st)
            for call in range(3):
                partial.fill_(float(rank + call))
                graph.replay()
                torch.cuda.synchronize()
                want = float(sum(r + call for r in range(world)))
                assert torch.all(out == want), f"graph replay {call}: {out.flatten()[:4].tolist()} != {want}"
        del graph
        pg.close()
        torch.cuda.synchronize()
        assert matmulq.read_device_status() == 0
        print("SHARDED OK", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
