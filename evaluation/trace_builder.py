"""Trace builders (parity: ``evaluation/trace/*.py``): turn a local copy of a
public request trace into a timestamp parquet that the benchmarks replay,
and print its request-rate profile.

With ``--trace`` a recipe of ``kunserve_b200.evaluation.traces`` (``--list``
prints them) says how a row becomes an arrival time and which window the
reference replays (BurstGPT, the Azure LLM inference traces, the Azure
Functions trace and its debug window); ``--offset``, ``--limit`` and
``--scale`` override the window and the time compression.  Without
``--trace``, any CSV with one timestamp column is converted as is (a
datetime or a number of seconds), time-scaled and cut to [start, end).

    python evaluation/trace_builder.py --trace burstgpt --csv BurstGPT.csv --out burstgpt.parquet
    python evaluation/trace_builder.py --trace maf --csv maf.csv --out maf-1000x.parquet --scale 1000
    python evaluation/trace_builder.py --csv my_trace.csv --column Timestamp --out trace.parquet --scale 10
"""
import argparse
import os
import sys

import numpy as np
import pandas as pd

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from kunserve_b200.evaluation import traces  # noqa: E402


def build(csv: str, column: str, out: str, scale: float = 1.0, start: float = None, end: float = None):
    """Generic conversion: one timestamp column, seconds from the first row."""
    df = pd.read_csv(csv)
    ts = pd.to_datetime(df[column], errors="coerce")
    if ts.notna().all():
        t = (ts - ts.min()).dt.total_seconds().to_numpy()
    else:
        t = df[column].astype(float).to_numpy()
        t = t - t.min()
    t = np.sort(t) / scale
    if start is not None:
        t = t[t >= start]
    if end is not None:
        t = t[t < end]
    pd.DataFrame({"timestamp": t}).to_parquet(out)
    return t


def build_recipe(name: str, path: str, out: str, offset=None, limit=None, scale=None, seed: int = 42):
    """Recipe conversion: the arrival times of trace ``name`` (seconds, in
    the recipe's time scale), cut to its window."""
    table = pd.read_parquet(path) if path.endswith(".parquet") else pd.read_csv(path)
    t = traces.build(name, table, offset=offset, limit=limit, scale=scale, seed=seed)
    pd.DataFrame({"timestamp": t}).to_parquet(out, index=False)
    return t


def rate_profile(t: np.ndarray, bin_s: float = 60.0):
    return traces.rate_profile(t, bin_s)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--trace", choices=traces.names(), help="a trace recipe (see --list)")
    p.add_argument("--list", action="store_true", help="print the trace recipes and exit")
    p.add_argument("--csv", help="the local trace copy (CSV, or parquet for --trace debug)")
    p.add_argument("--column", default="Timestamp", help="generic mode: the timestamp column")
    p.add_argument("--out")
    p.add_argument("--scale", type=float, help="divide arrival times by this (recipe default, or 1)")
    p.add_argument("--offset", type=int, help="recipe mode: first row of the window")
    p.add_argument("--limit", type=int, help="recipe mode: rows in the window")
    p.add_argument("--start", type=float, help="generic mode: first second kept")
    p.add_argument("--end", type=float, help="generic mode: end of the kept span (s)")
    p.add_argument("--bin", type=float, default=1.0, help="seconds per bin of the printed rate profile")
    a = p.parse_args(argv)
    if a.list:
        for n in traces.names():
            r = traces.RECIPES[n]
            window = f"rows {r.offset}..+{r.limit}" if r.limit else f"rows from {r.offset}"
            print(f"{n:10s} {r.source}; {window}, time scale {r.scale:g}  ({r.ref})")
        return
    if not a.csv or not a.out:
        p.error("--csv and --out are required")
    if a.trace:
        t = build_recipe(a.trace, a.csv, a.out, a.offset, a.limit, a.scale)
    else:
        t = build(a.csv, a.column, a.out, a.scale or 1.0, a.start, a.end)
    r = rate_profile(t, a.bin)
    span = float(t.max() - t.min()) if t.size else 0.0
    peak = float(r.max()) if r.size else 0.0
    mean = float(r.mean()) if r.size else 0.0
    print(f"{t.size} requests over {span:.1f}s; rate per {a.bin:g}s bin: mean {mean:.2f} max {peak:.2f} req/s")


if __name__ == "__main__":
    main()
