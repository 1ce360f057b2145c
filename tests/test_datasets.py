"""Dataset recipes: every dataset the reference prepares builds the
benchmark table from a local copy with the same field mapping."""
import json
import os
import subprocess
import sys

import pandas as pd
import pytest

from kunserve_b200.evaluation import datasets as ds

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SAMPLES = {
    "sharegpt": {"conversations": [{"from": "human", "value": "hello there"}, {"from": "gpt", "value": "hi"},
                                   {"from": "human", "value": "tell me more"},
                                   {"from": "gpt", "value": "sure here is more text"}]},
    "longbench": {"context": "a b c d", "input": "q r", "answers": ["x y z"]},
    "leval": {"input": "what is it", "outputs": ["an answer here"]},
    "chinese": {"input": "q", "reasoning_content": "r1 r2", "content": "c"},
    "code-bench": {"question_title": "t", "question_content": "do x", "public_test_cases": "[]"},
    "rag-instruct": {"documents": ["d1 d1", "d2"], "question": "q", "answer": "a a"},
    "rag-bench": {"documents": ["d1"], "question": "q", "response": "r", "generation_model_name": "m"},
    "burstgpt": {"Request tokens": 40000, "Response tokens": 12, "Model": "ChatGPT", "Log Type": "Conversation"},
    "azureconv": {"ContextTokens": 100, "GeneratedTokens": 7, "TIMESTAMP": "2023-11-16 18:15:46"},
}


def _sample(name):
    r = ds.RECIPES[name]
    if name in SAMPLES:
        return SAMPLES[name]
    if name.startswith("longbench"):
        return SAMPLES["longbench"]
    if r.prompt_len_col:
        return {r.prompt_len_col: 50, r.response_len_col: 9}
    # the generic question/answer recipes: give every field a recipe may read
    return {k: "some words here" for k in ("prompt", "response", "question", "answer", "instruction", "generation",
                                            "completion", "r1-gen", "input", "context")}


def test_every_reference_dataset_has_a_recipe():
    # the reference's evaluation/data holds 25 scripts; vllm_gen.py generates
    # responses with vLLM rather than preparing a dataset
    assert len(ds.names()) == 24
    for n in ds.names():
        out = ds.build(n, [_sample(n)] * 3)
        assert set(out) >= {"prompt", "prompt_len", "response_len"}
        assert len(out["prompt"]) == 3 and all(x >= 1 for x in out["response_len"])


def test_field_mappings():
    lb = ds.build("longbench", [SAMPLES["longbench"]])
    assert lb["prompt"][0] == "a b c d\nq r"
    sg = ds.build("sharegpt", [SAMPLES["sharegpt"]])
    assert sg["prompt"][0] == "hello there\nhi\ntell me more"
    bg = ds.build("burstgpt", [SAMPLES["burstgpt"]])
    assert bg["prompt_len"][0] == 16384 and bg["response_len"][0] == 12 and bg["Model"][0] == "ChatGPT"


def test_cli_builds_from_a_local_directory(tmp_path):
    d = tmp_path / "LongBench"
    (d / "multi_news").mkdir(parents=True)
    (d / "other").mkdir()
    rows = [SAMPLES["longbench"]] * 5
    pd.DataFrame(rows).to_json(d / "multi_news" / "test.jsonl", orient="records", lines=True)
    pd.DataFrame([{"context": "zz", "input": "zz", "answers": ["zz"]}]).to_json(
        d / "other" / "test.jsonl", orient="records", lines=True)
    out = tmp_path / "lb.parquet"
    r = subprocess.run([sys.executable, os.path.join(ROOT, "evaluation", "data", "build_dataset.py"),
                        "--dataset", "longbench", "--from", str(d), "--out", str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    df = pd.read_parquet(out)
    assert len(df) == 5 and list(df.columns)[:3] == ["prompt", "prompt_len", "response_len"]


def test_generated_responses_replace_the_lengths(tmp_path):
    """The vLLM generation step of the reference, through this framework:
    prompts over the limit are skipped, a short table repeats, and the
    response lengths are the generated token counts (PyTorch backend)."""
    table = tmp_path / "t.parquet"
    pd.DataFrame({"prompt": ["p0", "p1", "long"], "prompt_len": [12, 20, 30000],
                  "response_len": [100, 100, 100]}).to_parquet(table)
    out = tmp_path / "gen.parquet"
    r = subprocess.run([sys.executable, "evaluation/data/generate_responses.py", "--table", str(table), "--out",
                        str(out), "--model", "tiny-llama", "--device", "cpu", "--n", "3", "--max-tokens", "5",
                        "--kv-pages", "64"], cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, OMP_NUM_THREADS="2"))
    assert r.returncode == 0, r.stderr[-3000:]
    df = pd.read_parquet(out)
    assert df["prompt"].tolist() == ["p0", "p1", "p0"]
    assert (df["response_len"] == 5).all()
