"""Response generation for a benchmark table (parity:
``evaluation/data/vllm_gen.py``, which runs vLLM over a dataset's prompts to
record how long real responses are).  Here the prompts go through this
framework's own ``AsyncLLM`` (native kernels on a GPU, the PyTorch backend
on CPU), and the table gets the generated token counts as its
``response_len`` (and the text, with a tokenizer).

As in the reference, prompts of 16384 tokens or more are skipped and a
short table is repeated up to ``--n`` prompts
(``evaluation/data/vllm_gen.py:13-22``).  Without a tokenizer a prompt is
replayed as ``prompt_len`` seeded random token ids.  With random weights
(no checkpoint here) the lengths mean nothing about the model; the script
is for a converted checkpoint (``--weights``).

    python evaluation/data/generate_responses.py --table data/sharegpt.parquet --out data/sharegpt-gen.parquet \
        --model llama-3-8b --weights /models/llama-3-8b --tokenizer /models/llama-3-8b --n 2000
"""
import argparse
import asyncio
import math
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def select_prompts(df, n: int, offset: int = 0, max_prompt: int = 16384):
    """Rows offset .. offset + n of the prompts shorter than ``max_prompt``,
    the slice repeated when the table is shorter."""
    import pandas as pd
    rows = df[df["prompt_len"] < max_prompt].iloc[offset:offset + n]
    if len(rows) == 0:
        raise ValueError("no prompt below the length limit")
    if len(rows) < n:
        rows = pd.concat([rows] * int(math.ceil(n / len(rows))), ignore_index=True).iloc[:n]
    return rows.reset_index(drop=True)


async def generate(rows, model: str, device: str, max_tokens: int, tokenizer=None, weights=None, seed: int = 0,
                   kv_pages=None):
    from kunserve_b200.config import KunServeConfig, ModelConfig
    from kunserve_b200.llm import AsyncLLM
    from kunserve_b200.request import SamplingParams

    cfg = KunServeConfig()
    on_gpu = device.startswith("cuda")
    cfg.engine_config.dtype = "bf16" if on_gpu else "fp32"
    mc = ModelConfig(model, dtype=cfg.engine_config.dtype)
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="auto" if on_gpu else "torch", actor_kind="local",
                                devices=[device], seed=seed, tokenizer=tokenizer, weights_path=weights or "",
                                num_gpu_blocks=kv_pages)
    rng = np.random.default_rng(seed)
    vocab = mc.arch.vocab_size
    try:
        reqs = []
        for i, r in enumerate(rows.itertuples()):
            sp = SamplingParams(temperature=0.0, max_tokens=max_tokens)
            if tokenizer is not None:
                reqs.append(dict(prompt=str(r.prompt), sampling_params=sp, request_id=i))
            else:
                ids = rng.integers(0, vocab, int(r.prompt_len)).tolist()
                reqs.append(dict(prompt_token_ids=ids, sampling_params=sp, request_id=i))
        return await llm.batch_generate(reqs)
    finally:
        await llm.terminate()


def main(argv=None):
    import pandas as pd
    p = argparse.ArgumentParser()
    p.add_argument("--table", required=True, help="a benchmark table (prompt, prompt_len, response_len)")
    p.add_argument("--out", required=True)
    p.add_argument("--model", default="llama-3-8b")
    p.add_argument("--weights", help="a converted checkpoint directory (random weights without it)")
    p.add_argument("--tokenizer")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--n", type=int, default=1000)
    p.add_argument("--offset", type=int, default=0)
    p.add_argument("--max-tokens", type=int, default=8192)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--kv-pages", type=int, help="KV pages of the instance (default: sized from free memory)")
    a = p.parse_args(argv)
    rows = select_prompts(pd.read_parquet(a.table), a.n, a.offset)
    tok = None
    if a.tokenizer:
        from kunserve_b200.utils.tokenizer import get_tokenizer
        tok = get_tokenizer(a.tokenizer)
    results = asyncio.run(generate(rows, a.model, a.device, a.max_tokens, tok, a.weights, a.seed, a.kv_pages))
    results = sorted(results, key=lambda r: r["request_id"])
    out = rows.copy()
    out["response_len"] = [len(r["outputs"]) for r in results]
    if tok is not None:
        out["response"] = [r["text"] or "" for r in results]
    out.to_parquet(a.out, index=False)
    lens = out["response_len"].to_numpy()
    print(f"{len(out)} responses; length mean {lens.mean():.1f}, p50 {np.percentile(lens, 50):.0f}, "
          f"max {lens.max()}")


if __name__ == "__main__":
    main()
