"""Prefill latency sweep (parity: ``evaluation/prefill-profile.py:22-110``):
TTFT of batches of ``--batch`` prompts of ``--lens`` tokens, optionally on top
of a cached prefix of ``--prefix`` tokens (a chunked continuation), through
one native engine; also the FLOOR_CHUNK knee (tokens/s vs chunk size).

    python evaluation/prefill_profile.py --model llama-3-8b --batch 1 4 --lens 256 1024 4096
"""
import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(argv=None):
    from kunserve_b200.config import CacheConfig, ModelConfig, ParallelConfig
    from kunserve_b200.engine.step import StepInput
    from kunserve_b200.engine.worker import Worker

    p = argparse.ArgumentParser()
    p.add_argument("--model", default="llama-3-8b")
    p.add_argument("--batch", type=int, nargs="+", default=[1, 4])
    p.add_argument("--lens", type=int, nargs="+", default=[256, 512, 1024, 2048, 4096])
    p.add_argument("--prefix", type=int, default=0)
    p.add_argument("--iters", type=int, default=5)
    a = p.parse_args(argv)
    mc = ModelConfig(a.model, dtype="bf16")
    bs = 16
    w = Worker(0, mc, CacheConfig(block_size=bs), ParallelConfig(), backend="native", device="cuda:0")
    max_tok = max(b * n for b in a.batch for n in a.lens)
    pages_per = (a.prefix + max(a.lens) + bs - 1) // bs
    w.init_model(pages_per * max(a.batch), max_batch_tokens=max_tok, max_batch_size=max(a.batch))
    L = mc.get_num_layers()
    for B in a.batch:
        for n in a.lens:
            tables = [list(range(i * pages_per, (i + 1) * pages_per)) for i in range(B)]
            step = StepInput(list(range(B)), [[1] * n] * B, [a.prefix] * B, tables, [1] * B, 0, L,
                             temperature=[0.0] * B, seeds=[0] * B)
            w.step(step)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(a.iters):
                w.step(step)
            torch.cuda.synchronize()
            dt = (time.perf_counter() - t0) / a.iters
            print(json.dumps({"batch": B, "len": n, "prefix": a.prefix, "ttft_ms": round(dt * 1e3, 3),
                              "tok_s": round(B * n / dt, 1)}), flush=True)


if __name__ == "__main__":
    main()
