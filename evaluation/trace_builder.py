"""Trace builders (parity: ``evaluation/trace/*.py``): turn a CSV of request
timestamps (BurstGPT, Azure LLM inference, MAF) into a timestamp parquet,
optionally time-scaled, and print its rate profile.

    python evaluation/trace_builder.py --csv BurstGPT.csv --column Timestamp --out trace.parquet --scale 10
"""
import argparse

import numpy as np
import pandas as pd


def build(csv: str, column: str, out: str, scale: float = 1.0, start: float = None, end: float = None):
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


def rate_profile(t: np.ndarray, bin_s: float = 60.0):
    if t.size == 0:
        return np.array([])
    return np.histogram(t, bins=np.arange(0, t.max() + bin_s, bin_s))[0] / bin_s


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--csv", required=True)
    p.add_argument("--column", default="Timestamp")
    p.add_argument("--out", required=True)
    p.add_argument("--scale", type=float, default=1.0)
    p.add_argument("--start", type=float)
    p.add_argument("--end", type=float)
    a = p.parse_args(argv)
    t = build(a.csv, a.column, a.out, a.scale, a.start, a.end)
    r = rate_profile(t)
    print(f"{t.size} requests over {t.max() if t.size else 0:.1f}s; rate/min mean {r.mean():.2f} max {r.max():.2f}")


if __name__ == "__main__":
    main()
