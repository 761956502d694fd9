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

Two implementations of the exchange:
* ShardedMatMulQ: torch.distributed collectives (NCCL on GPUs, gloo in the CPU
  tests); the local product is libmtrtq's matmul_q8, or another `local_matmul`
  with the same signature (the CPU tests pass the oracle);
* P2PShardedMatMulQ: mtrtq_matmul_sharded, the library's own kernels over peer
  memory (every rank's output or slot buffer and flag words opened in every
  process through CUDA IPC at set-up; no collective library on the data path).
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
    """[begin, end) of each rank: whole `quantum` blocks split as evenly as possible
    (rank r starts at block floor(r * blocks / world), so later ranks take the extra
    blocks); the last range ends at `total`. With fewer blocks than ranks some
    ranges are empty."""
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


def shard_range(extent: int, split: str, rank: int, world: int) -> tuple[int, int]:
    """mtrtq_shard_range: [begin, end) of rank's shard (128-channel tiles for "N",
    64-k units for "K")."""
    import ctypes
    from . import _lib
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(_lib.lib().mtrtq_shard_range(extent, _lib.SPLIT_N if split == "N" else _lib.SPLIT_K, rank, world,
                                            ctypes.byref(b), ctypes.byref(e)), "mtrtq_shard_range")
    return b.value, e.value


class PeerBuffers:
    """Buffers every rank of a process group can store into, and the flag words of
    the library's exchange (mtrtq_shard_comm), set up collectively: each rank
    allocates a float buffer of `y_elems` (all-gather target), one of `slot_elems`
    (all-reduce slots) and MTRTQ_SHARD_FLAG_BYTES of flags, exports their CUDA IPC
    handles, gathers every rank's (torch.distributed object all-gather) and opens
    the peers'. The epoch counter advances once per exchange, the same on every
    rank as long as every rank makes the same calls in the same order; with
    device_epochs the count lives on the device instead (epoch 0 in every call),
    so that the exchanges can be captured in a CUDA graph and replayed.

    alternating: the exchanges alternate between two destination buffers, which
    lets the library skip its entry barrier (MTRTQ_SHARD comm.alternating). The
    slot buffer is allocated twice and allreduce() switches halves on every call;
    all-gather callers alternate themselves, between the halves y[:y_elems] and
    y[y_elems:] of a buffer allocated twice (`half`). Every rank must make the same
    sequence of exchanges, and a captured graph an even number of them."""

    def __init__(self, y_elems: int, slot_elems: int, group=None, device=None, device_epochs: bool = False,
                 alternating: bool = False):
        import ctypes
        from . import _lib
        self._lib, self.lib = _lib, _lib.lib()
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.world > _lib.MAX_WORLD:
            raise ValueError(f"at most {_lib.MAX_WORLD} ranks")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        z = lambda n: torch.zeros(max(int(n), 64), dtype=torch.float32, device=self.device)
        copies = 2 if alternating else 1
        self.alternating = alternating
        self.half = int(y_elems)
        self.slot_half = max(int(slot_elems), 64)
        self.y, self.slots = z(y_elems * copies), z(self.slot_half * copies)
        self.flags = torch.zeros(_lib.SHARD_FLAG_BYTES // 4, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = []
        for t in (self.y, self.slots, self.flags):
            h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            with torch.cuda.device(self.device):
                _lib.check(self.lib.mtrtq_ipc_export(t.data_ptr(), h), "mtrtq_ipc_export")
            mine.append(bytes(h))
        allh = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        self.imported = []
        comm = _lib.ShardComm()
        comm.rank, comm.world = self.rank, self.world
        comm.slot_elems = self.slots.numel()
        for r in range(self.world):
            if r == self.rank:
                ptrs = [self.y.data_ptr(), self.slots.data_ptr(), self.flags.data_ptr()]
            else:
                ptrs = []
                for hb in allh[r]:
                    p = ctypes.c_void_p()
                    h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(hb)
                    with torch.cuda.device(self.device):
                        _lib.check(self.lib.mtrtq_ipc_import(h, ctypes.byref(p)), "mtrtq_ipc_import")
                    self.imported.append(p.value)
                    ptrs.append(p.value)
            comm.y[r], comm.slots[r], comm.flags[r] = ptrs
        comm.alternating = 1 if alternating else 0
        self.comm = comm
        self._slot_turn = 0
        if alternating:  # a second comm whose slot buffers are the other halves
            comm2 = _lib.ShardComm()
            ctypes.memmove(ctypes.byref(comm2), ctypes.byref(comm), ctypes.sizeof(comm))
            for r in range(self.world):
                comm2.slots[r] = comm.slots[r] + 4 * self.slot_half
            comm.slot_elems = comm2.slot_elems = self.slot_half
            self.comms = [comm, comm2]
        else:
            self.comms = [comm]
        self.epoch = 0
        self.device_epochs = device_epochs
        if self.world > 1:
            dist.barrier(group=group)

    def next_epoch(self) -> int:
        if self.device_epochs:
            return 0
        self.epoch += 1
        return self.epoch

    def allgather(self, segments, stream=None):
        """segments: (offset, rows, cols, ld) in floats of self.y that this rank owns;
        after the call every rank's y holds every rank's segments."""
        import ctypes
        _lib = self._lib
        arr = (_lib.ShardSegment * max(1, len(segments)))(*[_lib.ShardSegment(*g) for g in segments])
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mtrtq_shard_allgather(arr, len(segments), ctypes.byref(self.comm), self.next_epoch(),
                                                      _sp(stream, self.device)), "mtrtq_shard_allgather")

    def group_allgather(self, group, stream=None):
        """Runs a GemvGroup whose outputs are this rank's column shards inside one
        half of self.y, with the all-gather fused into the kernel
        (mtrtq_gemv_group_allgather): after the call every rank's buffer holds every
        rank's shards. Needs alternating=True; callers alternate the halves."""
        import ctypes
        from .matmulq import MODES
        if not self.alternating:
            raise ValueError("the fused all-gather needs alternating buffers")
        with torch.cuda.device(self.device):
            self._lib.check(self.lib.mtrtq_gemv_group_allgather(
                group.problems, len(group.items), group.x_dtype, MODES[group.mode], group.workspace.data_ptr(),
                group.workspace.numel(), ctypes.byref(self.comm), self.next_epoch(), _sp(stream, self.device)),
                "mtrtq_gemv_group_allgather")

    def slot(self, M: int, N: int) -> torch.Tensor:
        """This rank's slot for the next all-reduce of an [M, N] partial (write the
        partial here: no copy)."""
        off = self._slot_turn * self.slot_half + self.rank * M * N
        return self.slots[off:off + M * N].view(M, N)

    def allreduce(self, partial: torch.Tensor, out: torch.Tensor, bias=None, residual=None, stream=None):
        """out = sum over ranks of partial (+ bias) (+ residual), rank order."""
        import ctypes
        _lib = self._lib
        M, N = partial.shape
        comm = self.comms[self._slot_turn]
        self._slot_turn = (self._slot_turn + 1) % len(self.comms)
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mtrtq_shard_allreduce(
                partial.data_ptr(), bias.data_ptr() if bias is not None else None,
                residual.data_ptr() if residual is not None else None,
                residual.stride(0) if residual is not None else 0, out.data_ptr(), out.stride(0), M, N,
                ctypes.byref(comm), self.next_epoch(), _sp(stream, self.device)), "mtrtq_shard_allreduce")
        return out

    def close(self):
        for p in self.imported:
            with torch.cuda.device(self.device):
                self.lib.mtrtq_ipc_close(p)
        self.imported = []


def _sp(stream, device):
    return stream.cuda_stream if stream is not None else torch.cuda.current_stream(device).cuda_stream


class P2PShardedMatMulQ:
    """Y = MatMulQ(X, W, scale) (+ bias) split across the ranks of a process group,
    one GPU each, exchanged by mtrtq_matmul_sharded over peer memory (PeerBuffers:
    every rank's output or slot buffer and flag words opened in every process).
    A call returns the full Y [M, N] on every rank (split N: a view of this rank's
    peer buffer, valid until the next call)."""

    def __init__(self, q: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None, split: str = "N",
                 group=None, device=None, mode: str = "bf16", max_m: int = 8, x_dtype=torch.float32):
        from . import _lib
        from .matmulq import MODES, PackedWeight
        if split not in ("N", "K"):
            raise ValueError("split must be 'N' or 'K'")
        self._lib, self.lib = _lib, _lib.lib()
        self.split, self.mode, self.max_m, self.x_dtype = split, mode, max_m, x_dtype
        K, N = q.shape
        self.K, self.N = K, N
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.peers = PeerBuffers(max_m * N if split == "N" else 0, max_m * N * world if split == "K" else 0,
                                 group=group, device=device)
        self.rank, self.world, self.device = self.peers.rank, self.peers.world, self.peers.device
        b, e = shard_range(N if split == "N" else K, split, self.rank, self.world)
        self.begin, self.end = b, e
        if e > b:
            qs = q[:, b:e] if split == "N" else q[b:e, :]
            ss = scale[b:e] if split == "N" else scale
            self.w = PackedWeight.from_int8(torch.from_numpy(np.ascontiguousarray(qs)),
                                            torch.from_numpy(np.ascontiguousarray(ss)), self.device)
        else:
            self.w = None
        self.bias = torch.from_numpy(np.ascontiguousarray(bias)).to(self.device) if bias is not None else None
        self._xd = _lib.DTYPE_BF16 if x_dtype == torch.bfloat16 else _lib.DTYPE_F32
        self._mode = MODES[mode]
        ws = self.lib.mtrtq_shard_workspace_bytes(max_m, K, N, self._xd, self._mode,
                                                  _lib.SPLIT_N if split == "N" else _lib.SPLIT_K, self.rank,
                                                  self.world)
        if ws < 0:
            raise _lib.MtrtqError(_lib.ERR_INVALID_ARG, "mtrtq_shard_workspace_bytes", _lib.last_error())
        self.ws = torch.zeros(max(ws, 256), dtype=torch.uint8, device=self.device)
        self._y = torch.empty((max_m, N), dtype=torch.float32, device=self.device) if split == "K" else None

    def __call__(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """x: [M, K] (M <= max_m), the same on every rank."""
        import ctypes
        _lib = self._lib
        M = x.shape[0]
        if x.dim() != 2 or x.shape[1] != self.K or x.stride(1) != 1 or M > self.max_m or x.dtype != self.x_dtype:
            raise ValueError(f"x must be [M <= {self.max_m}, {self.K}] {self.x_dtype} with unit stride along K")
        y = self.peers.y[:M * self.N].view(M, self.N) if self.split == "N" else self._y[:M]
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mtrtq_matmul_sharded(
                x.data_ptr(), self._xd, x.stride(0), self.w.packed.data_ptr() if self.w is not None else None,
                self.w.scale.data_ptr() if self.w is not None else None,
                self.bias.data_ptr() if self.bias is not None else None, y.data_ptr(), y.stride(0), M, self.K,
                self.N, self._mode, _lib.SPLIT_N if self.split == "N" else _lib.SPLIT_K,
                ctypes.byref(self.peers.comm), self.peers.next_epoch(), self.ws.data_ptr(), self.ws.numel(),
                _sp(stream, self.device)), "mtrtq_matmul_sharded")
        return y

    def close(self):
        self.peers.close()
