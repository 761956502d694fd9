"""Makes tests/golden/gpt2_decode.json: greedy tokens of the reference's KV-cache
decoder (oracle/gpt2_decode.py: the reference MatMulQ from oracle/_ref for every
Linear) on random-init GPT-2-small weights (mini_tensorrt_b200.gpt2.random_weights,
seed 0), for a batch of 1 and a batch of 16 sequences: prompts of 64 token ids
uniform in [0, 50257) (numpy seed 1234), then 64 generated tokens.

    python tests/golden/gen_gpt2_decode.py          # a few minutes on one core
"""
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle.gpt2_decode import OracleDecoder  # noqa: E402
from mini_tensorrt_b200 import gpt2  # noqa: E402

PROMPT_LEN, MAX_NEW, SEED, PROMPT_SEED = 64, 64, 0, 1234


def prompts(batch: int) -> np.ndarray:
    return np.random.default_rng(PROMPT_SEED + batch).integers(0, gpt2.GPT2Config().vocab,
                                                              (batch, PROMPT_LEN), dtype=np.int32)


def main():
    assert oracle.ref_available(), "build oracle/_ref first (oracle/build_ref.sh)"
    w = gpt2.random_weights(gpt2.GPT2Config(), SEED)
    out = {"config": "GPT-2 small, random init seed 0, int8 per-channel Linears, fp32 activations",
           "prompt_len": PROMPT_LEN, "max_new": MAX_NEW, "weights_seed": SEED, "cases": {}}
    for batch in (1, 16):
        t0 = time.time()
        p = prompts(batch)
        toks = OracleDecoder(w, batch, PROMPT_LEN + MAX_NEW).generate(p, MAX_NEW)
        out["cases"][str(batch)] = {"prompt": p.tolist(), "tokens": toks.tolist()}
        print(f"batch {batch}: {time.time() - t0:.1f} s", flush=True)
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "gpt2_decode.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
