"""Dataset builder: writes ``{prompt, prompt_len, response_len}`` parquet
files (the schema of the reference's ``evaluation/data/*.py``).

Without network access the public datasets cannot be fetched, so every
dataset the reference prepares is built from a local copy (a file or a
directory of parquet / JSON lines / JSON / CSV files) with its recipe in
``kunserve_b200.evaluation.datasets`` (``--list`` prints them); there is
also (a) BurstGPT-style synthetic prompts (Lorem-ipsum text of a target
token length) with lognormal lengths and (b) a plain conversion of a local
file that already has prompt and response columns.

    python evaluation/data/build_dataset.py --out data/synthetic.parquet --n 2000
    python evaluation/data/build_dataset.py --dataset longbench --from ~/LongBench/ --out data/longbench.parquet \
        --tokenizer meta-llama/Meta-Llama-3-8B
    python evaluation/data/build_dataset.py --out data/mine.parquet --from local.jsonl \
        --prompt-col prompt --response-col response
"""
import argparse
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

LOREM = ("lorem ipsum dolor sit amet consectetur adipiscing elit sed do eiusmod tempor incididunt ut labore et "
         "dolore magna aliqua").split()


def synthetic(n, prompt_mean, output_mean, sigma, seed):
    from kunserve_b200.evaluation.trace import lognormal_lengths
    rng = np.random.default_rng(seed)
    pl = lognormal_lengths(n, prompt_mean, sigma, 16, 16384, rng)
    ol = lognormal_lengths(n, output_mean, sigma, 1, 4096, rng)
    prompts = [" ".join(LOREM[i % len(LOREM)] for i in range(p)) for p in pl]
    return {"prompt": prompts, "prompt_len": pl, "response_len": ol}


def from_local(path, pcol, rcol, tokenizer):
    import pandas as pd
    ext = os.path.splitext(path)[1]
    df = {".parquet": pd.read_parquet, ".csv": pd.read_csv}.get(ext, lambda p: pd.read_json(p, lines=ext == ".jsonl"))(path)
    if tokenizer:
        from kunserve_b200.utils.tokenizer import get_tokenizer
        tok = get_tokenizer(tokenizer)
        count = lambda s: len(tok.encode(str(s)))
    else:
        count = lambda s: max(1, int(len(str(s).split()) * 1.3))   # word-based estimate
    return {"prompt": df[pcol].astype(str).tolist(), "prompt_len": [count(s) for s in df[pcol]],
            "response_len": [count(s) for s in df[rcol]]}


def main(argv=None):
    import pandas as pd
    p = argparse.ArgumentParser()
    p.add_argument("--out")
    p.add_argument("--n", type=int, default=1000)
    p.add_argument("--prompt-mean", type=float, default=700)
    p.add_argument("--output-mean", type=float, default=250)
    p.add_argument("--sigma", type=float, default=1.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--from", dest="src")
    p.add_argument("--prompt-col", default="prompt")
    p.add_argument("--response-col", default="response")
    p.add_argument("--tokenizer")
    p.add_argument("--dataset", help="a recipe of kunserve_b200.evaluation.datasets (needs --from)")
    p.add_argument("--max-prompt-tokens", type=int, default=16384)
    p.add_argument("--list", action="store_true", help="print the dataset recipes and exit")
    a = p.parse_args(argv)
    from kunserve_b200.evaluation import datasets as ds
    if a.list:
        for n in ds.names():
            r = ds.RECIPES[n]
            print(f"{n:18s} {r.source}  [{r.ref}]")
        return
    if a.dataset:
        if not a.src:
            raise SystemExit("--dataset needs --from: a local copy of the dataset")
        tok = None
        if a.tokenizer:
            from kunserve_b200.utils.tokenizer import get_tokenizer
            tok = get_tokenizer(a.tokenizer)
        rows = ds.read_local(a.src, ds.RECIPES[a.dataset].subsets)
        d = ds.build(a.dataset, rows, tok, a.max_prompt_tokens)
    elif a.src:
        d = from_local(a.src, a.prompt_col, a.response_col, a.tokenizer)
    else:
        d = synthetic(a.n, a.prompt_mean, a.output_mean, a.sigma, a.seed)
    if not a.out:
        raise SystemExit("--out is required")
    os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
    pd.DataFrame(d).to_parquet(a.out)
    print(f"wrote {len(d['prompt'])} rows to {a.out}")


if __name__ == "__main__":
    main()
