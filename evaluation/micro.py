"""Long-prompt burst micro-benchmark (parity: ``evaluation/micro.py:22-63``):
17 long prompts (16284, 14230, 4936, 4 x 4096, 2048 ...) each decoding 200
tokens, submitted once the pending queue has drained; prints TTFT and TBT
per request.  Lengths are clipped to the model's context."""
import argparse
import asyncio
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from kunserve_b200.config import ModelConfig, add_cli_args, get_cli_args  # noqa: E402
from kunserve_b200.request import SamplingParams  # noqa: E402

LENGTHS = [16284, 14230, 4936, 4096, 4096, 4096, 4096] + [2048] * 10


async def run(cfg, cpu):
    from kunserve_b200.llm import AsyncLLM
    mc = ModelConfig(cfg.bench_config.model or "tiny-llama", dtype=cfg.engine_config.dtype)
    kw = {"backend": "torch", "devices": ["cpu"]} if cpu else {}
    llm = await AsyncLLM.create(cfg, model_config=mc, num_gpu_blocks=cfg.bench_config.num_gpu_blocks, **kw)
    rng = np.random.default_rng(0)
    cap = min(mc.get_max_model_len(), cfg.bench_config.max_model_len) - 200
    while llm.check_pending_num():
        await asyncio.sleep(0.05)
    sp = SamplingParams(temperature=0.0, max_tokens=200, ignore_eos=True)
    outs = await asyncio.gather(*[llm.generate(prompt_token_ids=rng.integers(0, mc.get_vocab_size(),
                                                                             min(n, cap)).tolist(),
                                               sampling_params=sp) for n in LENGTHS])
    for n, o in zip(LENGTHS, outs):
        m = o["metrics"]
        print(f"prompt {min(n, cap):6d}: ttft {m.ttft:.3f}s tbt {m.tbt * 1e3:.2f}ms")
    await llm.terminate()


def main(argv=None):
    p = add_cli_args(argparse.ArgumentParser("micro"))
    p.add_argument("--cpu", action="store_true")
    a = p.parse_args(argv)
    asyncio.run(run(get_cli_args(a), a.cpu))


if __name__ == "__main__":
    main()
