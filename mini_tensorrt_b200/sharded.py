"""One MatMulQ split across the GPUs of a torch.distributed process group.

The op shards without changing its result, because output columns are
independent and k partial sums add:

* split="N" (column split): rank r holds W[:, N_r] and scale/bias[N_r], computes
  Y[:, N_r] from the replicated X, and an all-gather assembles Y on every rank.
  N_r are whole 128-channel tiles (the last rank takes the ragged rest), so each
  shard packs exactly like an unsplit weight.
* split="K" (row split): rank r holds W[K_r, :] and reads X[:, K_r] (a strided
  view, no copy), computes the scaled partial s * sum_{k in K_r} X W, and an
  all-reduce(sum) adds the partials. The scale distributes over the sum, so every
  rank applies it; the bias is added by rank 0 only, so it is added once, as the
  reference's separate Add does (src/ops/kernels_elementwise.cpp:31-35). K_r are
  whole 64-k units, which keeps every shard's X view 16-byte aligned.

One process per GPU; the collectives are torch.distributed's (NCCL on GPUs).
The local product is libmtrtq's matmul_q8; a caller may pass another
`local_matmul` with the same signature (the CPU tests pass the oracle).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch
import torch.distributed as dist

TILE_N = 128   # channels per packed tile
UNIT_K = 64    # k per packed unit


def shard_ranges(total: int, world: int, quantum: int) -> list[tuple[int, int]]:
    """[begin, end) of each rank: whole `quantum` blocks split as evenly as possible,
    earlier ranks taking the extra blocks; the last range ends at `total`. Ranks
    past the last block get empty ranges."""
    blocks = -(-total // quantum)
    out = []
    for r in range(world):
        b0 = r * blocks // world
        b1 = (r + 1) * blocks // world
        out.append((min(b0 * quantum, total), min(b1 * quantum, total)))
    return out


@dataclass
class Shard:
    split: str
    rank: int
    world: int
    begin: int
    end: int
    K: int
    N: int


def _default_local_matmul(x, w, bias, mode):
    from .matmulq import matmul_q8
    return matmul_q8(x, w, bias=bias, mode=mode)


def _default_pack(q, s, device):
    from .matmulq import PackedWeight
    return PackedWeight.from_int8(torch.from_numpy(np.ascontiguousarray(q)),
                                  torch.from_numpy(np.ascontiguousarray(s)), device)


class ShardedMatMulQ:
    """Y = MatMulQ(X, W, scale) (+ bias), W int8 [K, N] split across the group.

    q, scale, bias: the full host weights (numpy). Each rank packs only its shard.
    """

    def __init__(self, q: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None,
                 split: str = "N", group=None, device=None, mode: str = "bf16",
                 local_matmul: Callable | None = None, pack: Callable | None = None):
        if split not in ("N", "K"):
            raise ValueError("split must be 'N' or 'K'")
        self.group = group
        # Without an initialized process group this is the unsplit op on one GPU.
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.mode = mode
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
            else torch.device("cpu"))
        self.local_matmul = local_matmul or _default_local_matmul
        pack = pack or _default_pack
        K, N = q.shape
        self.K, self.N = K, N
        if split == "N":
            ranges = shard_ranges(N, self.world, TILE_N)
        else:
            ranges = shard_ranges(K, self.world, UNIT_K)
        b, e = ranges[self.rank]
        self.ranges = ranges
        self.shard = Shard(split, self.rank, self.world, b, e, K, N)
        if split == "N":
            self.w = pack(q[:, b:e], scale[b:e], self.device) if e > b else None
            self.bias = (torch.from_numpy(np.ascontiguousarray(bias[b:e])).to(self.device)
                         if bias is not None and e > b else None)
        else:
            self.w = pack(q[b:e, :], scale, self.device) if e > b else None
            self.bias = (torch.from_numpy(np.ascontiguousarray(bias)).to(self.device)
                         if bias is not None and self.rank == 0 else None)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """x: [M, K] on this rank's device, the same on every rank. Returns the full
        Y [M, N] on every rank."""
        M = x.shape[0]
        if x.shape[1] != self.K:
            raise ValueError(f"x must be [M, {self.K}]")
        sh = self.shard
        if self.world == 1:
            return self.local_matmul(x, self.w, self.bias, self.mode)
        if sh.split == "N":
            widths = [e - b for b, e in self.ranges]
            wmax = max(widths)
            mine = torch.zeros((M, wmax), dtype=torch.float32, device=x.device)
            if self.w is not None:
                mine[:, :sh.end - sh.begin] = self.local_matmul(x, self.w, self.bias, self.mode)
            gathered = torch.empty((self.world * M, wmax), dtype=torch.float32, device=x.device)
            dist.all_gather_into_tensor(gathered, mine, group=self.group)
            gathered = gathered.view(self.world, M, wmax)
            y = torch.empty((M, self.N), dtype=torch.float32, device=x.device)
            for r, (b, e) in enumerate(self.ranges):
                if e > b:
                    y[:, b:e] = gathered[r, :, :e - b]
            return y
        # K split: the partial over this rank's k range, then the sum over ranks
        if self.w is not None:
            y = self.local_matmul(x[:, sh.begin:sh.end], self.w, self.bias, self.mode)
        else:
            y = torch.zeros((M, self.N), dtype=torch.float32, device=x.device)
            if self.bias is not None:
                y += self.bias
        y = y.contiguous()
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y
