"""Tensor-parallel GPT-2 greedy KV-cache decoding over the GPUs of one node.

The reference decodes on one CPU thread (KVDecoder, tools/run_gpt2.cpp:88-214).
Here every rank of a process group (one GPU each) holds a slice of every layer:

* QKV and FFN-up are split by output columns -- the heads [h0, h1) of each of q, k
  and v, and the FFN columns [f0, f1) -- so attention runs on the rank's heads
  with its own slice of the KV caches, and gelu_new on its FFN columns, with no
  exchange;
* attn-out and FFN-down are split by input rows (the same heads and FFN columns):
  each rank's product is a partial sum of the full output, and one all-reduce
  (mtrtq_shard_allreduce: the library's own kernels over peer memory, summing the
  ranks' partials in rank order) adds them, then the bias once and the residual,
  straight into the replicated hidden state x -- two all-reduces per layer;
* the tied LM head is split by vocabulary columns; the ranks' logits meet in one
  all-gather (mtrtq_shard_allgather) and every rank takes the same argmax.

Heads, FFN columns and vocabulary columns are split with mtrtq_shard_range (whole
64-wide units for heads and FFN columns -- head_dim is 64 -- and 128-wide tiles for
the vocabulary). Every rank computes the same x bits (the all-reduce gives them
identical), so the argmax and the next token agree everywhere. A decode step is
one CUDA graph per rank (the exchanges count their epochs on the device; the
all-reduces alternate between two slot buffers, which removes their entry
barrier).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, matmulq, sharded
from ._lib import check, lib
from .gpt2 import GPT2Config, GPT2Weights
from .matmulq import MODES, PackedWeight, Workspace, workspace_bytes

GPT2_XL = GPT2Config(n_layer=48, d_model=1600, n_head=25, d_ff=6400, vocab=50257, n_pos=1024)


def _cols(a: np.ndarray, b: int, e: int) -> np.ndarray:
    return np.ascontiguousarray(a[:, b:e])


class TPDecoder:
    """Greedy decoding of `batch` sequences with the model split over the ranks of
    `group` (or one GPU without a process group).

    w: host weights (every rank passes the same; each keeps its slices).
    mode: MatMulQ mode of every product ("fp32" or "bf16")."""

    def __init__(self, w: GPT2Weights, batch: int, max_ctx: int, mode: str = "fp32", group=None, device=None,
                 max_steps: int | None = None, overlap: bool = True):
        cfg = w.cfg
        if cfg.head_dim != 64:
            raise ValueError("heads are split as 64-wide units: head_dim must be 64")
        self.cfg, self.B, self.max_ctx, self.mode, self.overlap = cfg, batch, max_ctx, mode, overlap
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.dev
        D, F, V, hd = cfg.d_model, cfg.d_ff, cfg.vocab, cfg.head_dim
        d0, d1 = sharded.shard_range(D, "K", self.rank, self.world)   # this rank's heads, as columns
        f0, f1 = sharded.shard_range(F, "K", self.rank, self.world)   # its FFN columns
        v0, v1 = sharded.shard_range(V, "N", self.rank, self.world)   # its vocabulary columns
        self.d0, self.d1, self.f0, self.f1, self.v0, self.v1 = d0, d1, f0, f1, v0, v1
        self.Hr, self.Dr, self.Fr = (d1 - d0) // hd, d1 - d0, f1 - f0
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)
        pk = lambda q, s: PackedWeight.from_int8(torch.from_numpy(np.ascontiguousarray(q)),
                                                 torch.from_numpy(np.ascontiguousarray(s)), dev)
        self.wte, self.wpe = f32(w.wte), f32(w.wpe)
        self.layers = []
        for L in w.layers:
            q, s = L["qkv"]
            cols = np.r_[d0:d1, D + d0:D + d1, 2 * D + d0:2 * D + d1]
            qo, so = L["o"]
            qf, sf = L["fc"]
            qp, sp = L["proj"]
            self.layers.append({
                "ln1": (f32(L["ln1"][0]), f32(L["ln1"][1])),
                "qkv": pk(q[:, cols], s[cols]), "bqkv": f32(L["bqkv"][cols]),
                "o": pk(qo[d0:d1, :], so), "bo": f32(L["bo"]),
                "ln2": (f32(L["ln2"][0]), f32(L["ln2"][1])),
                "fc": pk(_cols(qf, f0, f1), sf[f0:f1]), "bfc": f32(L["bfc"][f0:f1]),
                "proj": pk(qp[f0:f1, :], sp), "bproj": f32(L["bproj"]),
            })
        self.ln_f = (f32(w.ln_f[0]), f32(w.ln_f[1]))
        ql, sl = w.lm_head
        self.lm_head = pk(_cols(ql, v0, v1), sl[v0:v1])
        B = batch
        z = lambda *shape: torch.zeros(shape, dtype=torch.float32, device=dev)
        self.x, self.h = z(B, D), z(B, D)
        self.qkv, self.attn, self.mh = z(B, 3 * self.Dr), z(B, self.Dr), z(B, self.Fr)
        self.kc = [z(B, max_ctx, self.Dr) for _ in range(cfg.n_layer)]
        self.vc = [z(B, max_ctx, self.Dr) for _ in range(cfg.n_layer)]
        self.next_tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.best = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.max_steps = max_steps or max_ctx
        self.history = torch.zeros((self.max_steps, B), dtype=torch.int32, device=dev)
        self.prompt = torch.zeros((B, 1), dtype=torch.int32, device=dev)
        need = max(workspace_bytes(B, K, N, torch.float32, mode)
                   for K, N in [(D, 3 * self.Dr), (self.Dr, D), (D, self.Fr), (self.Fr, D), (D, v1 - v0)])
        self.ws = Workspace(dev).get(need)
        # exchanges: the all-reduces' slots (alternating halves, 2 per layer: an even
        # count per step) and the logits' all-gather target (an entry barrier each)
        self.red = sharded.PeerBuffers(0, B * D * self.world, group=group, device=dev, device_epochs=True,
                                       alternating=True)
        self.gat = sharded.PeerBuffers(B * V, 0, group=group, device=dev, device_epochs=True)
        self.logits = self.gat.y[:B * V].view(B, V)
        self.stream = torch.cuda.Stream(dev)
        self.graph = None

    @property
    def _sp(self) -> int:
        return self.stream.cuda_stream

    def _mm(self, x, w: PackedWeight, bias, y, epilogue=_lib.EPILOGUE_NONE):
        ws = self.ws
        check(lib().mtrtq_matmul_ex(x.data_ptr(), _lib.DTYPE_F32, x.stride(0), w.packed.data_ptr(),
                                    w.scale.data_ptr(), bias.data_ptr() if bias is not None else None,
                                    y.data_ptr(), y.stride(0), x.shape[0], w.K, w.N, MODES[self.mode],
                                    ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                                    epilogue, None, 0, self._sp), "mtrtq_matmul_ex")

    def _layernorm(self, x, ln, y):
        check(lib().mtrtq_layernorm(x.data_ptr(), ln[0].data_ptr(), ln[1].data_ptr(), y.data_ptr(), x.shape[0],
                                    x.shape[1], self.cfg.eps, self._sp), "layernorm")

    def _row_parallel(self, inp, w: PackedWeight, bias):
        """x += (sum over ranks of inp @ w) + bias: the partial goes straight into
        this rank's slot, the all-reduce adds the bias once and the residual."""
        part = self.red.slot(self.B, self.cfg.d_model)
        self._mm(inp, w, None, part)
        self.red.allreduce(part, self.x, bias=bias, residual=self.x, stream=self.stream)

    def _launch_step(self):
        with matmulq.option(_lib.OPT_OVERLAP_LAUNCH, 1 if self.overlap else 0):
            self._launch_step_kernels()

    def _launch_step_kernels(self):
        cfg, B, D, V, sp, L = self.cfg, self.B, self.cfg.d_model, self.cfg.vocab, self._sp, lib()
        P = self.prompt.shape[1]
        check(L.mtrtq_decode_embed(self.prompt.data_ptr(), P, self.next_tok.data_ptr(), self.pos.data_ptr(),
                                   self.wte.data_ptr(), self.wpe.data_ptr(), cfg.n_pos, self.x.data_ptr(), B, D, V,
                                   sp), "embed")
        for i, ly in enumerate(self.layers):
            self._layernorm(self.x, ly["ln1"], self.h)
            self._mm(self.h, ly["qkv"], ly["bqkv"], self.qkv)
            check(L.mtrtq_decode_attention(self.qkv.data_ptr(), self.kc[i].data_ptr(), self.vc[i].data_ptr(),
                                           self.pos.data_ptr(), self.attn.data_ptr(), B, self.Hr, cfg.head_dim,
                                           self.max_ctx, sp), "attention")
            self._row_parallel(self.attn, ly["o"], ly["bo"])
            self._layernorm(self.x, ly["ln2"], self.h)
            self._mm(self.h, ly["fc"], ly["bfc"], self.mh, _lib.EPILOGUE_GELU_TANH)
            self._row_parallel(self.mh, ly["proj"], ly["bproj"])
        self._layernorm(self.x, self.ln_f, self.h)
        self._mm(self.h, self.lm_head, None, self.logits[:, self.v0:self.v1])
        self.gat.allgather([(self.v0, B, self.v1 - self.v0, V)], stream=self.stream)
        check(L.mtrtq_argmax_rows(self.logits.data_ptr(), B, V, V, self.best.data_ptr(), sp), "argmax")
        check(L.mtrtq_decode_next(self.best.data_ptr(), B, self.next_tok.data_ptr(), self.history.data_ptr(),
                                  self.max_steps, self.pos.data_ptr(), sp), "decode_next")

    def _reset(self, prompt: torch.Tensor):
        with torch.cuda.stream(self.stream):
            if self.prompt.shape != prompt.shape:
                self.prompt = torch.empty_like(prompt, device=self.dev)
                self.graph = None
            self.prompt.copy_(prompt)
            self.pos.zero_()
            self.best.zero_()
            self.next_tok.zero_()
            self.history.zero_()

    def generate(self, prompt, max_new: int, use_graph: bool = True) -> dict:
        """prompt: int [B, P] (the same on every rank). P + max_new - 1 steps, the
        prompt consumed token by token; returns {"tokens": int32 [B, max_new],
        "prefill_s", "decode_s"} (CUDA events on this rank's stream)."""
        prompt = torch.as_tensor(np.asarray(prompt), dtype=torch.int32)
        B, P = prompt.shape
        if B != self.B:
            raise ValueError(f"batch {B} != {self.B}")
        if P + max_new - 1 > min(self.max_ctx, self.max_steps):
            raise ValueError("prompt + max_new exceeds max_ctx")
        self._reset(prompt)
        if use_graph and self.graph is None:
            with torch.cuda.stream(self.stream):
                self._launch_step()  # eager: per-device set-up; then capture one step
            torch.cuda.synchronize(self.dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self._launch_step()
            self.graph = g
            self._reset(prompt)
        run = (lambda: self.graph.replay()) if use_graph else self._launch_step
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        with torch.cuda.stream(self.stream):
            ev[0].record(self.stream)
            for _ in range(P):
                run()
            ev[1].record(self.stream)
            for _ in range(max_new - 1):
                run()
            ev[2].record(self.stream)
        torch.cuda.synchronize(self.dev)
        hist = self.history[P - 1:P - 1 + max_new].t().contiguous().cpu().numpy()
        return {"tokens": hist, "prefill_s": ev[0].elapsed_time(ev[1]) / 1e3,
                "decode_s": ev[1].elapsed_time(ev[2]) / 1e3}

    def close(self):
        self.graph = None
        self.red.close()
        self.gat.close()
