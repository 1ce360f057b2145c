"""Request datasets: turn a local copy of a public dataset into the
``{prompt, prompt_len, response_len}`` table the benchmarks replay.

Every dataset the reference prepares (``evaluation/data/*.py``) has a recipe
here: which fields make the prompt and the response (for example LongBench
joins ``context`` and ``input``, ShareGPT takes every turn but the last as
the prompt), which subsets it concatenates, and for trace-only datasets
(BurstGPT, Azure) which columns already hold token counts.  The field
mappings follow the reference scripts (cited per recipe) because they define
what each dataset means to the benchmark; the loading is new: there is no
network here, so a recipe reads a local copy (parquet, JSON lines, JSON or
CSV files, a directory of them, or a Hugging Face snapshot directory) with
pandas.  Prompts are truncated to ``max_prompt_tokens`` tokens (16384 in the
reference).  Without a tokenizer, lengths are estimated from words.

Trace-only recipes synthesise Lorem-ipsum prompts of the recorded token
count, as the reference does (``evaluation/data/burstgpt.py:13-67``).
"""
import glob
import os
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

LOREM = ("lorem ipsum dolor sit amet consectetur adipiscing elit sed do eiusmod tempor incididunt ut labore et "
         "dolore magna aliqua").split()


def _first(x):
    """First element of a list-valued field (``answers``, ``outputs``)."""
    if isinstance(x, (list, tuple)) or hasattr(x, "tolist"):
        x = list(x.tolist() if hasattr(x, "tolist") else x)
        return x[0] if x else ""
    return x


def _join_docs(x):
    if isinstance(x, (list, tuple)) or hasattr(x, "tolist"):
        return "\n".join(str(d) for d in (x.tolist() if hasattr(x, "tolist") else x))
    return str(x)


@dataclass
class Recipe:
    name: str
    source: str                                  # the public dataset it describes
    ref: str                                     # the reference script (path:line)
    prompt: Optional[Callable[[dict], str]] = None
    response: Optional[Callable[[dict], str]] = None
    # trace-only datasets: token counts are columns, prompts are synthesised
    prompt_len_col: Optional[str] = None
    response_len_col: Optional[str] = None
    subsets: Sequence[str] = ()                  # subset names the reference concatenates
    keep: Sequence[str] = ()                     # extra columns carried into the table
    prune_percentile: float = 0.0                # drop both tails of the lengths (ShareGPT)


CODE_BENCH_SYSTEM = ("You are an expert Python programmer. You will be given a question (problem specification) "
                     "and will generate a correct Python program that matches the specification and passes all "
                     "tests.")

RECIPES: Dict[str, Recipe] = {r.name: r for r in [
    Recipe("burstgpt", "BurstGPT trace (CSV)", "evaluation/data/burstgpt.py:40-60",
           prompt_len_col="Request tokens", response_len_col="Response tokens", keep=("Model", "Log Type")),
    Recipe("burstgpt-full", "BurstGPT trace, every row", "evaluation/data/burstgpt-full.py:40-55",
           prompt_len_col="Request tokens", response_len_col="Response tokens"),
    Recipe("burstgpt-473200", "BurstGPT trace slice", "evaluation/data/burstgpt-473200.py:41-56",
           prompt_len_col="Request tokens", response_len_col="Response tokens"),
    Recipe("burstgpt-473800", "BurstGPT trace slice", "evaluation/data/burstgpt-473800.py:41-56",
           prompt_len_col="Request tokens", response_len_col="Response tokens"),
    Recipe("azureconv", "Azure LLM inference trace, conversation (CSV)", "evaluation/data/azureconv.py:58-70",
           prompt_len_col="ContextTokens", response_len_col="GeneratedTokens", keep=("TIMESTAMP",)),
    Recipe("sharegpt", "ShareGPT conversations (JSON lines)", "evaluation/data/sharegpt.py:27-60",
           prompt=lambda s: "\n".join(t["value"] for t in list(s["conversations"])[:-1]),
           response=lambda s: list(s["conversations"])[-1]["value"], prune_percentile=1.0),
    Recipe("longbench", "THUDM/LongBench multi_news + gov_report", "evaluation/data/longbench.py:33-50",
           prompt=lambda s: s["context"] + "\n" + s["input"], response=lambda s: _first(s["answers"]),
           subsets=("multi_news", "gov_report")),
    Recipe("longbench-summary", "THUDM/LongBench multi_news + gov_report",
           "evaluation/data/longbench-summary.py:33-50",
           prompt=lambda s: s["context"] + "\n" + s["input"], response=lambda s: _first(s["answers"]),
           subsets=("multi_news", "gov_report")),
    Recipe("longbench-code", "THUDM/LongBench repobench-p + repobench-p_e",
           "evaluation/data/longbench-code.py:31-50",
           prompt=lambda s: s["context"] + "\n" + s["input"], response=lambda s: _first(s["answers"]),
           subsets=("repobench-p", "repobench-p_e")),
    Recipe("leval", "L4NLP/LEval QA subsets", "evaluation/data/leval.py:28-45",
           prompt=lambda s: s["input"], response=lambda s: _first(s["outputs"]),
           subsets=("financial_qa", "legal_contract_qa", "multidoc_qa", "narrative_qa", "natural_question",
                    "scientific_qa")),
    Recipe("longdata", "long prompt/completion pairs", "evaluation/data/longdata.py",
           prompt=lambda s: s["prompt"], response=lambda s: s["completion"]),
    Recipe("chinese", "Congliu/Chinese-DeepSeek-R1-Distill-data-110k", "evaluation/data/chinese.py:22-32",
           prompt=lambda s: s["input"], response=lambda s: s["reasoning_content"] + " " + s["content"]),
    Recipe("code-assistant", "glaiveai/glaive-code-assistant-v3", "evaluation/data/code-assistant.py:22-33",
           prompt=lambda s: s["question"], response=lambda s: s["answer"]),
    Recipe("code-bench", "livecodebench/code_generation_lite", "evaluation/data/code-bench.py:30-55",
           prompt=lambda s: (CODE_BENCH_SYSTEM + "\nTitle\n" + s["question_title"] + "\nDescription\n"
                             + s["question_content"] + "\nTest cases\n" + str(s["public_test_cases"])),
           response=lambda s: ""),
    Recipe("code-cot", "open-r1/codeforces-cots", "evaluation/data/code-cot.py:22-33",
           prompt=lambda s: s["prompt"], response=lambda s: s["generation"]),
    Recipe("func-call", "WhiteRabbitNeo/Code-Functions-Level-General", "evaluation/data/func-call.py:25-45",
           prompt=lambda s: s["instruction"], response=lambda s: s["response"]),
    Recipe("func-call-v2", "WhiteRabbitNeo/Code-Functions-Level-Cyber", "evaluation/data/func-call-v2.py:25-45",
           prompt=lambda s: s["instruction"], response=lambda s: s["response"]),
    Recipe("func-call-cot", "ThinkAgents/Function-Calling-with-Chain-of-Thoughts",
           "evaluation/data/func-call-cot.py:25-45",
           prompt=lambda s: s["prompt"], response=lambda s: s["r1-gen"]),
    Recipe("hermes-func-call", "NousResearch/hermes-function-calling-v1",
           "evaluation/data/hermes-func-call.py:25-45",
           prompt=lambda s: s["instruction"], response=lambda s: s["response"]),
    Recipe("tooluse", "AymanTarig/function-calling-v0.2-with-r1-cot", "evaluation/data/tooluse.py:22-33",
           prompt=lambda s: s["prompt"], response=lambda s: s["r1-gen"]),
    Recipe("rag", "glaiveai/rag_sample", "evaluation/data/rag.py:25-45",
           prompt=lambda s: s["prompt"], response=lambda s: s["response"]),
    Recipe("rag-v1", "glaiveai/RAG-v1", "evaluation/data/rag-v1.py:25-45",
           prompt=lambda s: s["question"], response=lambda s: s["answer"]),
    Recipe("rag-instruct", "FreedomIntelligence/RAG-Instruct", "evaluation/data/rag-instruct.py:25-45",
           prompt=lambda s: _join_docs(s["documents"]) + "\n" + s["question"], response=lambda s: s["answer"]),
    Recipe("rag-bench", "rungalileo/ragbench", "evaluation/data/rag-bench.py:25-45",
           prompt=lambda s: _join_docs(s["documents"]) + "\n" + s["question"], response=lambda s: s["response"],
           keep=("generation_model_name",)),
]}


def _read_table(path: str):
    import pandas as pd
    ext = os.path.splitext(path)[1].lower()
    if ext == ".parquet":
        return pd.read_parquet(path)
    if ext == ".csv":
        return pd.read_csv(path)
    if ext == ".jsonl":
        return pd.read_json(path, lines=True)
    if ext == ".json":
        try:
            return pd.read_json(path)
        except ValueError:
            return pd.read_json(path, lines=True)
    raise ValueError(f"unsupported file {path}")


def read_local(path: str, subsets: Sequence[str] = ()):
    """Rows of a local dataset copy: one file, or every data file under a
    directory (for a multi-subset dataset, the files whose path names one of
    ``subsets``, when any does)."""
    import pandas as pd
    if os.path.isfile(path):
        return _read_table(path)
    files = sorted(f for ext in ("parquet", "jsonl", "json", "csv")
                   for f in glob.glob(os.path.join(path, "**", f"*.{ext}"), recursive=True))
    if subsets:
        chosen = [f for f in files if any(s in f for s in subsets)]
        files = chosen or files
    if not files:
        raise FileNotFoundError(f"no data files under {path}")
    return pd.concat([_read_table(f) for f in files], ignore_index=True)


def _counter(tokenizer):
    if tokenizer is None:
        return lambda s: max(1, int(round(len(str(s).split()) * 1.3))), None
    return (lambda s: len(tokenizer.encode(str(s)))), tokenizer


def lorem_prompt(n_tokens: int) -> str:
    return " ".join(LOREM[i % len(LOREM)] for i in range(max(1, int(n_tokens))))


def build(name: str, rows, tokenizer=None, max_prompt_tokens: int = 16384) -> Dict[str, list]:
    """The benchmark table of dataset ``name`` from its rows (a pandas frame
    or a list of dicts)."""
    import numpy as np
    r = RECIPES[name]
    records = rows.to_dict("records") if hasattr(rows, "to_dict") else list(rows)
    count, tok = _counter(tokenizer)
    out: Dict[str, list] = {"prompt": [], "prompt_len": [], "response_len": []}
    for k in r.keep:
        out[k] = []
    for s in records:
        if r.prompt_len_col is not None:
            pl = min(int(s[r.prompt_len_col]), max_prompt_tokens)
            rl = int(s[r.response_len_col])
            prompt = lorem_prompt(pl)
        else:
            prompt = str(r.prompt(s))
            pl = count(prompt)
            if pl > max_prompt_tokens:
                if tok is not None:
                    prompt = tok.decode(tok.encode(prompt)[:max_prompt_tokens])
                else:
                    prompt = " ".join(prompt.split()[:int(max_prompt_tokens / 1.3)])
                pl = max_prompt_tokens
            rl = count(r.response(s)) if r.response is not None else 0
        out["prompt"].append(prompt)
        out["prompt_len"].append(pl)
        out["response_len"].append(max(1, rl))
        for k in r.keep:
            out[k].append(s.get(k))
    if r.prune_percentile > 0 and out["prompt"]:
        p, q = r.prune_percentile, 100 - r.prune_percentile
        pl, rl = np.asarray(out["prompt_len"]), np.asarray(out["response_len"])
        ok = ((pl >= np.percentile(pl, p)) & (pl <= np.percentile(pl, q)) &
              (rl >= np.percentile(rl, p)) & (rl <= np.percentile(rl, q)))
        out = {k: [v for v, o in zip(vals, ok) if o] for k, vals in out.items()}
    return out


def names() -> List[str]:
    return sorted(RECIPES)
