"""Seeded synthetic workloads at the GPT-2 / large-model shapes the MatMulQ path serves.

All inputs are deterministic (numpy PCG64 with fixed seeds), so the CUDA path and
the CPU reference see identical bytes. Value distributions: activations ~ N(0,1),
weights ~ N(0, 0.02) (the GPT-2 initializer), biases ~ N(0, 0.02); weights are
quantized per output channel with the reference packer's rule.

Algorithmic cost per call (the roofline basis): FLOPs = 2 M K N; bytes =
K N (int8 W) + 4 N (scale) + x_bytes M K (activations) + 4 M N (fp32 Y) + 4 N (bias).
Pre-packing is load-time work and padding is not counted.
"""
from __future__ import annotations

import numpy as np

# FFN-up single op with bias (Y = X dequant(W) + b), GPT-2 small.
SINGLE_OP = {"name": "ffn_up_m64", "M": 64, "K": 768, "N": 3072, "bias": True}

# Decode GEMV set at GPT-2-small shapes, M in {1, 8}; the LM head is tied to the
# token embedding (W = wte^T) and has the vocabulary's odd width 50257.
DECODE_SHAPES = [
    ("qkv", 768, 2304),
    ("attn_out", 768, 768),
    ("ffn_up", 768, 3072),
    ("ffn_down", 3072, 768),
    ("lm_head", 768, 50257),
]
DECODE_M = (1, 8)

# Large-shape sweep (Llama-style projections), activations bf16.
LARGE_SHAPES = [(4096, 4096), (4096, 11008), (4096, 14336), (14336, 4096)]
LARGE_M = (1, 16, 128, 2048)


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def weights(K: int, N: int, seed: int) -> np.ndarray:
    """W f32 [K, N] ~ N(0, 0.02)."""
    return rng(seed).standard_normal((K, N), dtype=np.float32) * np.float32(0.02)


def tied_lm_head(V: int, D: int, seed: int) -> np.ndarray:
    """LM head W [D, V] = wte^T with wte [V, D] ~ N(0, 0.02)."""
    wte = rng(seed).standard_normal((V, D), dtype=np.float32) * np.float32(0.02)
    return np.ascontiguousarray(wte.T)


def activations(M: int, K: int, seed: int) -> np.ndarray:
    """X f32 [M, K] ~ N(0, 1)."""
    return rng(seed).standard_normal((M, K), dtype=np.float32)


def bias(N: int, seed: int) -> np.ndarray:
    return rng(seed).standard_normal((N,), dtype=np.float32) * np.float32(0.02)


def shape_seed(name: str, K: int, N: int) -> int:
    """Stable per-shape seed so every user of a shape draws the same weights."""
    h = 1469598103934665603
    for ch in f"{name}:{K}x{N}".encode():
        h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h & 0x7FFFFFFF


def decode_weight(name: str, K: int, N: int) -> np.ndarray:
    if name == "lm_head":
        return tied_lm_head(N, K, shape_seed(name, K, N))
    return weights(K, N, shape_seed(name, K, N))


def algorithmic_bytes(M: int, K: int, N: int, x_bytes: int = 4, with_bias: bool = False) -> int:
    return K * N + 4 * N + x_bytes * M * K + 4 * M * N + (4 * N if with_bias else 0)


def flops(M: int, K: int, N: int) -> int:
    return 2 * M * K * N
