"""One rank of the two-GPU tensor-parallel decoding test (launched by
torch.distributed.run from tests/test_tp.py); prints TP OK."""
import dataclasses
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from mini_tensorrt_b200 import gpt2, matmulq, tp  # noqa: E402
from oracle.gpt2_decode import OracleDecoder  # noqa: E402
from tests.conftest import rel_err  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        # GPT-2-XL layer shapes, 2 layers: 25 heads split unevenly (12 / 13)
        cfg = dataclasses.replace(tp.GPT2_XL, n_layer=2, n_pos=64)
        w = gpt2.random_weights(cfg, seed=21)
        prompt = np.random.default_rng(22).integers(0, cfg.vocab, (2, 4), dtype=np.int32)
        dec = tp.TPDecoder(w, 2, max_ctx=16, mode="fp32", device=dev)
        assert dec.Hr == (12 if rank == 0 else 13)
        got = dec.generate(prompt, 6)
        want = OracleDecoder(w, 2, 16).generate(prompt, 6)
        np.testing.assert_array_equal(got["tokens"], want)
        ref = OracleDecoder(w, 2, 16)
        toks = np.concatenate([prompt, want[:, :-1]], axis=1)
        for pos in range(toks.shape[1]):
            _, logits = ref.step(toks[:, pos], pos)
        err = rel_err(dec.logits.cpu().numpy(), logits)
        assert err <= 1e-4, f"rank {rank}: XL logits rel err {err:.3e}"
        dec.close()
        # GPT-2 small: the split decoder and the unsplit one give the same tokens
        ws = gpt2.random_weights(gpt2.GPT2Config(), seed=23)
        pr = np.random.default_rng(24).integers(0, 50257, (4, 16), dtype=np.int32)
        split = tp.TPDecoder(ws, 4, max_ctx=48, mode="fp32", device=dev)
        full = gpt2.DeviceDecoder(ws, 4, max_ctx=48, mode="fp32", device=dev)
        a = split.generate(pr, 32)["tokens"]
        b = full.generate(pr, 32)["tokens"]
        np.testing.assert_array_equal(a, b)
        split.close()
        torch.cuda.synchronize()
        assert matmulq.read_device_status() == 0
        print("TP OK", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
