"""Workload reports (parity: ``evaluation/profile.py`` and
``evaluation/trace_profile.py``): the prompt / output length statistics of
a benchmark table, and how far into a trace a given span of time reaches.

Lengths are capped as the benchmarks replay them: a request whose prompt
and output exceed ``--max-len`` tokens (16384) keeps its output and is
cut at the prompt (``evaluation/profile.py:33-38``).  For a trace, the
report gives the request count, the span, the mean rate and the index of
the first request at or after ``--until`` seconds
(``evaluation/trace_profile.py:62-76``).

    python evaluation/dataset_profile.py --table data/longbench.parquet
    python evaluation/dataset_profile.py --trace burstgpt.parquet --until 2000
"""
import argparse
import json
import os
import sys
from typing import Dict, Optional

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def length_report(prompt_len, response_len, max_len: int = 16384) -> Dict[str, float]:
    p = np.asarray(prompt_len, dtype=np.int64)
    o = np.asarray(response_len, dtype=np.int64)
    over = p + o > max_len
    p = np.where(over, np.maximum(max_len - o, 0), p)
    out = {"requests": int(p.size), "capped": int(over.sum())}
    for name, v in (("prompt", p), ("output", o)):
        if v.size == 0:
            continue
        out.update({f"{name}_mean": float(v.mean()), f"{name}_min": int(v.min()), f"{name}_max": int(v.max()),
                    f"{name}_p50": float(np.percentile(v, 50)), f"{name}_p90": float(np.percentile(v, 90)),
                    f"{name}_p99": float(np.percentile(v, 99))})
    return out


def trace_report(timestamps, until: Optional[float] = None) -> Dict[str, float]:
    t = np.sort(np.asarray(timestamps, dtype=np.float64))
    out = {"requests": int(t.size)}
    if t.size == 0:
        return out
    rel = t - t[0]
    span = float(rel[-1])
    out.update({"span_s": span, "mean_rate": (t.size - 1) / span if span > 0 else float("inf")})
    if until is not None:
        i = int(np.searchsorted(rel, until, side="left"))
        out["index_at_until"] = i if i < t.size else None
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--table", help="a benchmark table (parquet with prompt_len and response_len)")
    p.add_argument("--trace", help="a timestamp parquet")
    p.add_argument("--max-len", type=int, default=16384)
    p.add_argument("--until", type=float, help="trace: report the first request at or after this many seconds")
    a = p.parse_args(argv)
    if not a.table and not a.trace:
        p.error("give --table and/or --trace")
    import pandas as pd
    if a.table:
        df = pd.read_parquet(a.table)
        print(json.dumps({"table": a.table, **length_report(df["prompt_len"], df["response_len"], a.max_len)}))
    if a.trace:
        df = pd.read_parquet(a.trace)
        col = next(c for c in df.columns if "time" in c.lower())
        print(json.dumps({"trace": a.trace, **trace_report(df[col].to_numpy(), a.until)}))


if __name__ == "__main__":
    main()
