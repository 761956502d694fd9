"""GPT-2 KV-cache greedy decoding on the device, every Linear an int8 MatMulQ.

The reference decodes one token at a time on the CPU (KVDecoder,
tools/run_gpt2.cpp:88-191, with fp32 `cpu::gemm_auto` for every Linear and the LM
head). Here one decode step runs on the GPU as one CUDA graph: the embedding,
per layer LayerNorm -> QKV MatMulQ (+bias) -> attention over the KV cache ->
out-proj MatMulQ (+bias, + residual fused into its store) -> LayerNorm -> FFN-up
MatMulQ (+bias, gelu_new fused) -> FFN-down MatMulQ (+bias, + residual fused), the
final LayerNorm, the LM head
MatMulQ (weights tied to the token embedding) and the greedy argmax, all through
libmtrtq's C ABI. Q, K and V use one 768x2304 weight: per-column quantization makes
that identical to three separate 768x768 weights.

A batch of B sequences is B rows of every MatMulQ (M = B). The prompt is either
consumed token by token, as the reference's prefill does (tools/run_gpt2.cpp:205),
or -- prefill="gemm" -- in one pass in which every Linear is a single MatMulQ of
M = B * P rows (a dense contraction: the cluster GEMV up to 64 rows, the tcgen05
GEMM above in bf16 mode) and attention is causal over the prompt; the KV caches
then hold every prompt position and decoding continues from there.

Weights here are random (the architecture of GPT-2 small, N(0, 0.02) for every
matrix, embedding and bias, LayerNorm gamma 1 and beta 0), seeded per tensor.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, matmulq
from ._lib import check, lib
from .matmulq import MODES, PackedWeight, Workspace, quantize_per_channel, workspace_bytes


@dataclass(frozen=True)
class GPT2Config:
    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    d_ff: int = 3072
    vocab: int = 50257
    n_pos: int = 1024
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_head


def _seed(base: int, name: str) -> int:
    return (base * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFF


def _normal(base: int, name: str, shape) -> np.ndarray:
    g = np.random.default_rng(_seed(base, name))
    return g.standard_normal(shape, dtype=np.float32) * np.float32(0.02)


@dataclass
class GPT2Weights:
    """Host weights: fp32 embeddings, LayerNorm and biases; int8 + per-column scale
    for every Linear (W [K, N], the reference's layout), lm_head = wte^T."""
    cfg: GPT2Config
    wte: np.ndarray
    wpe: np.ndarray
    layers: list = field(default_factory=list)
    ln_f: tuple = None
    lm_head: tuple = None  # (q int8 [D, V], s [V])


def random_weights(cfg: GPT2Config = GPT2Config(), seed: int = 0) -> GPT2Weights:
    D, F = cfg.d_model, cfg.d_ff
    wte = _normal(seed, "wte", (cfg.vocab, D))
    w = GPT2Weights(cfg, wte, _normal(seed, "wpe", (cfg.n_pos, D)))
    ones, zeros = np.ones(D, np.float32), np.zeros(D, np.float32)
    for l in range(cfg.n_layer):
        p = f"l{l}_"
        w.layers.append({
            "ln1": (ones, zeros),
            "qkv": quantize_per_channel(_normal(seed, p + "Wqkv", (D, 3 * D))),
            "bqkv": _normal(seed, p + "bqkv", (3 * D,)),
            "o": quantize_per_channel(_normal(seed, p + "Wo", (D, D))),
            "bo": _normal(seed, p + "bo", (D,)),
            "ln2": (ones, zeros),
            "fc": quantize_per_channel(_normal(seed, p + "Wfc", (D, F))),
            "bfc": _normal(seed, p + "bfc", (F,)),
            "proj": quantize_per_channel(_normal(seed, p + "Wproj", (F, D))),
            "bproj": _normal(seed, p + "bproj", (D,)),
        })
    w.ln_f = (ones, zeros)
    w.lm_head = quantize_per_channel(np.ascontiguousarray(wte.T))
    return w


class DeviceDecoder:
    """Greedy KV-cache decoding of `batch` sequences on one GPU.

    mode: MatMulQ mode for every Linear ("fp32" keeps the activations in fp32;
    "bf16" rounds them to bf16 before each product).
    overlap: launch the step's kernels with programmatic dependent launch
    (MTRTQ_OPT_OVERLAP_LAUNCH while the step is recorded or launched), so each one
    starts while the one ahead finishes; the weights are never written during
    decoding, which is the option's condition.
    fold_ln: fold each LayerNorm into the MatMulQ that reads it where the shape
    runs on the cluster GEMV (one launch instead of two)."""

    def __init__(self, w: GPT2Weights, batch: int, max_ctx: int, mode: str = "fp32",
                 device="cuda", max_steps: int | None = None, overlap: bool = True, fold_ln: bool = True):
        cfg = w.cfg
        self.cfg, self.B, self.max_ctx, self.mode = cfg, batch, max_ctx, mode
        self.overlap = overlap
        if max_ctx > cfg.n_pos:
            raise ValueError("max_ctx exceeds the position table")
        self.dev = torch.device(device)
        dev = self.dev
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        pk = lambda qs: PackedWeight.from_int8(torch.from_numpy(qs[0]), torch.from_numpy(qs[1]), dev)
        self.wte, self.wpe = f32(w.wte), f32(w.wpe)
        self.layers = []
        for L in w.layers:
            self.layers.append({
                "ln1": (f32(L["ln1"][0]), f32(L["ln1"][1])), "qkv": pk(L["qkv"]), "bqkv": f32(L["bqkv"]),
                "o": pk(L["o"]), "bo": f32(L["bo"]), "ln2": (f32(L["ln2"][0]), f32(L["ln2"][1])),
                "fc": pk(L["fc"]), "bfc": f32(L["bfc"]), "proj": pk(L["proj"]), "bproj": f32(L["bproj"]),
            })
        self.ln_f = (f32(w.ln_f[0]), f32(w.ln_f[1]))
        self.lm_head = pk(w.lm_head)
        B, D, F, V = batch, cfg.d_model, cfg.d_ff, cfg.vocab
        z = lambda *s: torch.zeros(s, dtype=torch.float32, device=dev)
        self.x, self.h, self.attn, self.ao = z(B, D), z(B, D), z(B, D), z(B, D)
        self.qkv, self.mh, self.logits = z(B, 3 * D), z(B, F), z(B, V)
        self.kc = [z(B, max_ctx, D) for _ in range(cfg.n_layer)]
        self.vc = [z(B, max_ctx, D) for _ in range(cfg.n_layer)]
        self.next_tok = torch.zeros(B, dtype=torch.int32, device=dev)
        self.best = torch.zeros(B, dtype=torch.int64, device=dev)  # argmax keys, zeroed per step
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.max_steps = max_steps or max_ctx
        self.history = torch.zeros((self.max_steps, B), dtype=torch.int32, device=dev)
        self.prompt = torch.zeros((B, 1), dtype=torch.int32, device=dev)
        xd = torch.float32
        need = max(workspace_bytes(B, K, N, xd, mode)
                   for K, N in [(D, 3 * D), (D, D), (D, F), (F, D), (D, V)])
        self.ws = Workspace(dev)
        self.ws_buf = self.ws.get(need)
        self.graph = None
        self.stream = torch.cuda.Stream(dev)
        # LayerNorm folded into the MatMulQ that reads it (mtrtq_matmul_ln_ex) up to 8
        # rows, where the shape runs on the cluster GEMV; otherwise a LayerNorm
        # launch first. Every CTA of the GEMV computes the rows' statistics, which
        # costs more than the separate launch saves at 16 rows (B200: batch 16
        # decode 0.65 ms/step folded against 0.61 ms).
        self.fold_ln = {name: fold_ln and B <= 8 and matmulq.supports_ln(B, K, N, mode)
                        for name, (K, N) in {"qkv": (D, 3 * D), "fc": (D, F), "lm": (D, V)}.items()}

    # -- one decode step, as launches on self.stream ------------------------------
    def _mm(self, x, w: PackedWeight, bias, y, epilogue=_lib.EPILOGUE_NONE, residual=None):
        ws = self.ws_buf
        check(lib().mtrtq_matmul_ex(x.data_ptr(), _lib.DTYPE_F32, x.stride(0), w.packed.data_ptr(),
                                    w.scale.data_ptr(), bias.data_ptr() if bias is not None else None,
                                    y.data_ptr(), y.stride(0), x.shape[0], w.K, w.N, MODES[self.mode],
                                    ws.data_ptr() if ws is not None else None,
                                    ws.numel() if ws is not None else 0, epilogue,
                                    residual.data_ptr() if residual is not None else None,
                                    residual.stride(0) if residual is not None else 0, self._sp),
              "mtrtq_matmul_ex")

    def _mm_ln(self, x, ln, w: PackedWeight, bias, y, epilogue=_lib.EPILOGUE_NONE):
        """y = epilogue(LayerNorm(x; ln) @ w + bias) in one kernel."""
        check(lib().mtrtq_matmul_ln_ex(x.data_ptr(), x.stride(0), ln[0].data_ptr(), ln[1].data_ptr(),
                                       self.cfg.eps, w.packed.data_ptr(), w.scale.data_ptr(),
                                       bias.data_ptr() if bias is not None else None, y.data_ptr(),
                                       y.stride(0), x.shape[0], w.K, w.N, MODES[self.mode],
                                       self.ws_buf.data_ptr() if self.ws_buf is not None else None,
                                       self.ws_buf.numel() if self.ws_buf is not None else 0, epilogue,
                                       None, 0, self._sp), "mtrtq_matmul_ln_ex")

    def _ln_then(self, name, ln, w, bias, y, epilogue=_lib.EPILOGUE_NONE):
        """LayerNorm of x feeding one Linear: folded into it when the shape allows."""
        if self.fold_ln[name]:
            self._mm_ln(self.x, ln, w, bias, y, epilogue)
            return
        cfg = self.cfg
        check(lib().mtrtq_layernorm(self.x.data_ptr(), ln[0].data_ptr(), ln[1].data_ptr(), self.h.data_ptr(),
                                    self.B, cfg.d_model, cfg.eps, self._sp), "layernorm")
        self._mm(self.h, w, bias, y, epilogue)

    def _launch_step(self):
        with matmulq.option(_lib.OPT_OVERLAP_LAUNCH, 1 if self.overlap else 0):
            self._launch_step_kernels()

    def _launch_step_kernels(self):
        cfg, B, D, sp, L = self.cfg, self.B, self.cfg.d_model, self._sp, lib()
        P = self.prompt.shape[1]
        check(L.mtrtq_decode_embed(self.prompt.data_ptr(), P, self.next_tok.data_ptr(),
                                   self.pos.data_ptr(), self.wte.data_ptr(), self.wpe.data_ptr(),
                                   cfg.n_pos, self.x.data_ptr(), B, D, cfg.vocab, sp), "embed")
        for i, ly in enumerate(self.layers):
            self._ln_then("qkv", ly["ln1"], ly["qkv"], ly["bqkv"], self.qkv)
            check(L.mtrtq_decode_attention(self.qkv.data_ptr(), self.kc[i].data_ptr(),
                                           self.vc[i].data_ptr(), self.pos.data_ptr(),
                                           self.attn.data_ptr(), B, cfg.n_head, cfg.head_dim,
                                           self.max_ctx, sp), "attention")
            # x += attn @ Wo + bo, fused into the MatMulQ store
            self._mm(self.attn, ly["o"], ly["bo"], self.x, _lib.EPILOGUE_ADD_RESIDUAL, self.x)
            self._ln_then("fc", ly["ln2"], ly["fc"], ly["bfc"], self.mh, _lib.EPILOGUE_GELU_TANH)
            self._mm(self.mh, ly["proj"], ly["bproj"], self.x, _lib.EPILOGUE_ADD_RESIDUAL, self.x)
        self._ln_then("lm", self.ln_f, self.lm_head, None, self.logits)
        check(L.mtrtq_argmax_rows(self.logits.data_ptr(), B, cfg.vocab, cfg.vocab,
                                  self.best.data_ptr(), sp), "argmax")
        check(L.mtrtq_decode_next(self.best.data_ptr(), B, self.next_tok.data_ptr(),
                                  self.history.data_ptr(), self.max_steps, self.pos.data_ptr(), sp),
              "decode_next")

    @property
    def _sp(self) -> int:
        return self.stream.cuda_stream

    def _reset(self, prompt: torch.Tensor):
        with torch.cuda.stream(self.stream):
            if self.prompt.shape != prompt.shape:
                self.prompt = torch.empty_like(prompt, device=self.dev)
                self.graph = None  # the graph holds the prompt's address and length
            self.prompt.copy_(prompt)
            self.pos.zero_()
            self.best.zero_()
            self.next_tok.zero_()
            self.history.zero_()

    # -- the prompt in one pass: every Linear one MatMulQ of M = B * P rows ---------
    def _prefill_buffers(self, P: int):
        if getattr(self, "_pf_P", None) == P:
            return
        cfg, B = self.cfg, self.B
        D, F, R = cfg.d_model, cfg.d_ff, self.B * P
        z = lambda *s: torch.zeros(s, dtype=torch.float32, device=self.dev)
        self.pf_x, self.pf_h, self.pf_attn = z(R, D), z(R, D), z(R, D)
        self.pf_qkv, self.pf_mh = z(R, 3 * D), z(R, F)
        need = max(workspace_bytes(R, K, N, torch.float32, self.mode)
                   for K, N in [(D, 3 * D), (D, D), (D, F), (F, D)])
        self.pf_ws = Workspace(self.dev).get(need)
        self._pf_P = P

    def _mm_ws(self, x, w: PackedWeight, bias, y, ws, epilogue=_lib.EPILOGUE_NONE, residual=None):
        check(lib().mtrtq_matmul_ex(x.data_ptr(), _lib.DTYPE_F32, x.stride(0), w.packed.data_ptr(),
                                    w.scale.data_ptr(), bias.data_ptr() if bias is not None else None,
                                    y.data_ptr(), y.stride(0), x.shape[0], w.K, w.N, MODES[self.mode],
                                    ws.data_ptr() if ws is not None else None,
                                    ws.numel() if ws is not None else 0, epilogue,
                                    residual.data_ptr() if residual is not None else None,
                                    residual.stride(0) if residual is not None else 0, self._sp),
              "mtrtq_matmul_ex")

    def _launch_prefill(self, P: int):
        """Launches the prefill of self.prompt ([B, P]) on self.stream: positions
        0..P-1 through every layer as M = B * P products, the caches filled, then
        the LM head and argmax of each sequence's last position, which becomes the
        first generated token (history[P - 1]); decoding then starts at P."""
        cfg, B, D, sp, L = self.cfg, self.B, self.cfg.d_model, self._sp, lib()
        R = B * P
        ws = self.pf_ws
        check(L.mtrtq_prefill_embed(self.prompt.data_ptr(), B, P, self.wte.data_ptr(), self.wpe.data_ptr(),
                                    cfg.n_pos, self.pf_x.data_ptr(), D, cfg.vocab, sp), "prefill_embed")
        x, h = self.pf_x, self.pf_h
        for i, ly in enumerate(self.layers):
            check(L.mtrtq_layernorm(x.data_ptr(), ly["ln1"][0].data_ptr(), ly["ln1"][1].data_ptr(), h.data_ptr(),
                                    R, D, cfg.eps, sp), "layernorm")
            self._mm_ws(h, ly["qkv"], ly["bqkv"], self.pf_qkv, ws)
            check(L.mtrtq_prefill_attention(self.pf_qkv.data_ptr(), self.kc[i].data_ptr(), self.vc[i].data_ptr(),
                                            self.pf_attn.data_ptr(), B, P, cfg.n_head, cfg.head_dim,
                                            self.max_ctx, sp), "prefill_attention")
            self._mm_ws(self.pf_attn, ly["o"], ly["bo"], x, ws, _lib.EPILOGUE_ADD_RESIDUAL, x)
            check(L.mtrtq_layernorm(x.data_ptr(), ly["ln2"][0].data_ptr(), ly["ln2"][1].data_ptr(), h.data_ptr(),
                                    R, D, cfg.eps, sp), "layernorm")
            self._mm_ws(h, ly["fc"], ly["bfc"], self.pf_mh, ws, _lib.EPILOGUE_GELU_TANH)
            self._mm_ws(self.pf_mh, ly["proj"], ly["bproj"], x, ws, _lib.EPILOGUE_ADD_RESIDUAL, x)
        # each sequence's last position: rows P-1, 2P-1, ... (a strided view)
        last = x.view(B, P, D)[:, P - 1, :]
        check(L.mtrtq_layernorm_strided(last.data_ptr(), last.stride(0), self.ln_f[0].data_ptr(),
                                        self.ln_f[1].data_ptr(), self.h.data_ptr(), B, D, cfg.eps, sp),
              "layernorm")
        self._mm(self.h, self.lm_head, None, self.logits)
        check(L.mtrtq_argmax_rows(self.logits.data_ptr(), B, cfg.vocab, cfg.vocab, self.best.data_ptr(), sp),
              "argmax")
        check(L.mtrtq_decode_next(self.best.data_ptr(), B, self.next_tok.data_ptr(), self.history.data_ptr(),
                                  self.max_steps, self.pos.data_ptr(), sp), "decode_next")

    def generate(self, prompt, max_new: int, use_graph: bool = True, prefill: str = "tokens") -> dict:
        """prompt: int [B, P] token ids. prefill "tokens": P + max_new - 1 steps (the P
        prompt positions, then one per generated token after the first); "gemm": the
        prompt in one pass of M = B * P products, then max_new - 1 steps. Returns
        {"tokens": int32 [B, max_new], "prefill_s", "decode_s"} with times measured
        by CUDA events."""
        if prefill not in ("tokens", "gemm"):
            raise ValueError("prefill is 'tokens' or 'gemm'")
        prompt = torch.as_tensor(np.asarray(prompt), dtype=torch.int32)
        B, P = prompt.shape
        if B != self.B:
            raise ValueError(f"batch {B} != {self.B}")
        steps = P + max_new - 1
        if steps > self.max_ctx or steps > self.max_steps:
            raise ValueError("prompt + max_new exceeds max_ctx")
        if prefill == "gemm":
            return self._generate_gemm_prefill(prompt, max_new, use_graph)
        self._reset(prompt)
        if use_graph and self.graph is None:
            # one eager step (per-device setup), then capture one step and reset
            with torch.cuda.stream(self.stream):
                self._launch_step()
            torch.cuda.synchronize()
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
        torch.cuda.synchronize()
        hist = self.history[P - 1:P - 1 + max_new].t().contiguous().cpu().numpy()
        return {"tokens": hist, "prefill_s": ev[0].elapsed_time(ev[1]) / 1e3,
                "decode_s": ev[1].elapsed_time(ev[2]) / 1e3, "steps": steps}

    def _capture_step(self):
        with torch.cuda.stream(self.stream):
            self._launch_step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._launch_step()
        self.graph = g

    def _generate_gemm_prefill(self, prompt, max_new: int, use_graph: bool) -> dict:
        B, P = prompt.shape
        self._prefill_buffers(P)
        self._reset(prompt)
        if use_graph and self.graph is None:
            self._capture_step()
            self._reset(prompt)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        with torch.cuda.stream(self.stream):
            # the prefill's last position is P - 1: decode_next then records the
            # first generated token there and moves on to P
            self.pos.fill_(P - 1)
            ev[0].record(self.stream)
            with matmulq.option(_lib.OPT_OVERLAP_LAUNCH, 1 if self.overlap else 0):
                self._launch_prefill(P)
            ev[1].record(self.stream)
            for _ in range(max_new - 1):
                self.graph.replay() if use_graph else self._launch_step()
            ev[2].record(self.stream)
        torch.cuda.synchronize()
        hist = self.history[P - 1:P - 1 + max_new].t().contiguous().cpu().numpy()
        return {"tokens": hist, "prefill_s": ev[0].elapsed_time(ev[1]) / 1e3,
                "decode_s": ev[1].elapsed_time(ev[2]) / 1e3, "steps": max_new}
