"""CPU restatement of the reference's KV-cache greedy decoder with int8 Linears.

Test infrastructure (the checker for mini_tensorrt_b200.gpt2), not a product path.

The reference's KVDecoder::step (tools/run_gpt2.cpp:135-191) in numpy fp32, with
every Linear routed to the reference MatMulQ (+ its Add for the bias): the
reference's own kernel from oracle/_ref when it is built, else the oracle's C
restatement (bit-identical to it, pinned in tests/test_oracle.py). LayerNorm
(:113-122, eps 1e-5, biased variance), attention over the cache (:143-172),
gelu_new (:178-181) and argmax (:42-47, first index of the maximum) follow the
reference's formulas; rows of a batch are independent sequences.
"""
from __future__ import annotations

import numpy as np

import oracle


def _mm(x, qs, bias=None):
    q, s = qs
    if oracle.ref_available():
        return oracle.ref_matmul_q8(x, q, s, bias)
    return oracle.matmul_q8(x, q, s, bias)


def _layernorm(x, g, b, eps):
    mean = x.mean(axis=1, keepdims=True, dtype=np.float32)
    c = (x - mean).astype(np.float32)
    var = (c * c).mean(axis=1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32)
    return (c * inv * g + b).astype(np.float32)


def _gelu_new(u):
    k = np.float32(0.7978845608028654)
    return (np.float32(0.5) * u * (np.float32(1.0) + np.tanh(k * (u + np.float32(0.044715) * u * u * u)))
            ).astype(np.float32)


def _argmax_first(row):
    return int(np.argmax(row))  # numpy returns the first index of the maximum


class OracleDecoder:
    """w: mini_tensorrt_b200.gpt2.GPT2Weights (host weights, int8 Linears)."""

    def __init__(self, w, batch: int, max_ctx: int):
        self.w, self.cfg, self.B = w, w.cfg, batch
        D = self.cfg.d_model
        self.kc = [np.zeros((batch, max_ctx, D), np.float32) for _ in range(self.cfg.n_layer)]
        self.vc = [np.zeros((batch, max_ctx, D), np.float32) for _ in range(self.cfg.n_layer)]

    def step(self, tokens, pos: int):
        """tokens: int [B]; returns (argmax [B], logits [B, V])."""
        cfg, w = self.cfg, self.w
        D, H, hd = cfg.d_model, cfg.n_head, cfg.head_dim
        x = (w.wte[np.asarray(tokens)] + w.wpe[pos]).astype(np.float32)
        scale = np.float32(1.0) / np.sqrt(np.float32(hd), dtype=np.float32)
        for l, L in enumerate(w.layers):
            h = _layernorm(x, L["ln1"][0], L["ln1"][1], cfg.eps)
            qkv = _mm(h, L["qkv"], L["bqkv"])
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            self.kc[l][:, pos] = k
            self.vc[l][:, pos] = v
            ctx = np.empty((self.B, D), np.float32)
            for b in range(self.B):
                for hh in range(H):
                    sl = slice(hh * hd, (hh + 1) * hd)
                    kj = self.kc[l][b, :pos + 1, sl]
                    s = (kj @ q[b, sl]).astype(np.float32) * scale
                    e = np.exp(s - s.max(), dtype=np.float32)
                    wgt = e * (np.float32(1.0) / e.sum(dtype=np.float32))
                    ctx[b, sl] = (wgt @ self.vc[l][b, :pos + 1, sl]).astype(np.float32)
            x = (x + _mm(ctx, L["o"], L["bo"])).astype(np.float32)
            h = _layernorm(x, L["ln2"][0], L["ln2"][1], cfg.eps)
            m = _gelu_new(_mm(h, L["fc"], L["bfc"]))
            x = (x + _mm(m, L["proj"], L["bproj"])).astype(np.float32)
        h = _layernorm(x, w.ln_f[0], w.ln_f[1], cfg.eps)
        logits = _mm(h, w.lm_head)
        return np.array([_argmax_first(r) for r in logits], dtype=np.int32), logits

    def generate(self, prompt, max_new: int):
        """The reference's generate_kv (tools/run_gpt2.cpp:195-214) for B rows:
        prompt token by token, then max_new greedy tokens. Returns int32 [B, max_new]."""
        prompt = np.asarray(prompt)
        B, P = prompt.shape
        pos = 0
        nxt = None
        for i in range(P):
            nxt, _ = self.step(prompt[:, i], pos)
            pos += 1
        out = np.zeros((B, max_new), np.int32)
        for i in range(max_new):
            out[:, i] = nxt
            if i + 1 < max_new:  # the reference's last step is never read
                nxt, _ = self.step(nxt, pos)
                pos += 1
        return out
