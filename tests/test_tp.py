"""Tensor-parallel GPT-2 decoding (mini_tensorrt_b200.tp): column-split QKV (by
heads) and FFN-up, row-split attn-out and FFN-down with the library's all-reduce,
vocabulary-split LM head with its all-gather. Checked against the reference's
decoder restated on the CPU (oracle/gpt2_decode.py) and against the unsplit
device decoder, on one GPU (world 1) and on two (tests/tp_gpu_worker.py)."""
import dataclasses
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from mini_tensorrt_b200 import gpt2, tp
from oracle.gpt2_decode import OracleDecoder
from tests.conftest import rel_err

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
# head_dim 64 (the unit of the head split), 4 heads, small enough for the CPU oracle
SMALL64 = gpt2.GPT2Config(n_layer=2, d_model=256, n_head=4, d_ff=1024, vocab=1000, n_pos=64)


def test_xl_config_splits_evenly_by_heads():
    """GPT-2-XL's 25 heads, 6400 FFN columns and 50257 vocabulary columns split into
    whole units at every world size the node offers."""
    from mini_tensorrt_b200 import sharded
    cfg = tp.GPT2_XL
    assert cfg.head_dim == 64
    for world in (1, 2, 4, 8):
        heads = [sharded.shard_ranges(cfg.d_model, world, 64)[r] for r in range(world)]
        assert sum((e - b) // 64 for b, e in heads) == 25 and all(e > b for b, e in heads)
        assert all((e - b) % 64 == 0 for b, e in heads)
        ffn = sharded.shard_ranges(cfg.d_ff, world, 64)
        assert ffn[-1][1] == 6400 and all(e > b for b, e in ffn)


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3])
def test_tp_single_rank_matches_oracle(cuda_device, batch):
    w = gpt2.random_weights(SMALL64, seed=11)
    prompt = np.random.default_rng(12).integers(0, SMALL64.vocab, (batch, 5), dtype=np.int32)
    dec = tp.TPDecoder(w, batch, max_ctx=24, mode="fp32", device=cuda_device)
    got = dec.generate(prompt, 10)
    want = OracleDecoder(w, batch, 24).generate(prompt, 10)
    np.testing.assert_array_equal(got["tokens"], want)
    ref = OracleDecoder(w, batch, 24)
    toks = np.concatenate([prompt, want[:, :-1]], axis=1)
    for pos in range(toks.shape[1]):
        _, logits = ref.step(toks[:, pos], pos)
    assert rel_err(dec.logits.cpu().numpy(), logits) <= 1e-4
    again = dec.generate(prompt, 10, use_graph=False)  # eager launches: the same tokens
    np.testing.assert_array_equal(again["tokens"], want)
    dec.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_on_two_gpus():
    """Two ranks: a 2-layer GPT-2-XL-shaped model (25 heads split 12 / 13) against
    the oracle, and GPT-2-small-shaped tokens against the unsplit decoder."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "tp_gpu_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=900,
                       env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("TP OK") == 2, r.stdout[-3000:]
