"""Arrival-time recipes for the public request traces the benchmarks replay.

The reference turns each trace into a timestamp parquet with a script of its
own (``evaluation/trace/*.py``); a recipe here states the same meaning in
one place: which column (or columns) give a request's arrival, in which
unit, how the trace is compressed in time, and which slice of it the
reference's evaluation replays by default.

* ``burstgpt`` (BurstGPT CSV): ``Timestamp`` is already seconds since the
  trace start; divided by a time scale (default 10: ten times denser);
  default slice rows 474438 .. +775 (``evaluation/trace/burstgpt.py:13-60``).
* ``azurecode`` / ``azureconv`` (Azure LLM inference traces): the
  ``TIMESTAMP`` wall-clock column as seconds.  The 2023 files write
  ``2023-11-16 18:15:46.6805900``, the 2024 ones append ``+00:00`` and may
  drop the fraction; both parse here (``evaluation/trace/azurecode.py``,
  ``azureconv.py``).  azurecode's default slice is rows 5100 .. +927.
* ``maf`` (Azure Functions invocation trace): an invocation starts at
  ``end_timestamp - duration``; times are divided by ``timex`` (default
  1000) and the kept rows are down-sampled to one in ``timex`` (a seeded
  sample, then sorted; its rows differ from those of the reference's pandas
  sampler), so that the compressed trace keeps the original request rate;
  default slice from row 319091 (``evaluation/trace/maf.py:33-59``).
* ``debug``: the 200-second window [536350, 536550) of a MAF timestamp
  table, the burst the reference inspects (``evaluation/trace/debug.py``).

Differences from the reference scripts: wall-clock stamps are read as UTC
(the reference converts them with the host's local time zone; only the
differences between requests matter to a replay), and the slice is cut
when the table is built, so the parquet holds exactly the replayed window
(replay it with offset 0).  Plots are left out (no plotting library here);
``rate_profile`` gives the per-bin request rate instead.
"""
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import numpy as np


def _wallclock_seconds(col) -> np.ndarray:
    """Seconds since the epoch of Azure ``TIMESTAMP`` strings (2023 and
    2024 layouts)."""
    import pandas as pd
    s = col.astype(str).str.strip()
    s = s.str.replace(r"\+00:00$", "", regex=True)
    # 2023 stamps carry seven fractional digits, 2024 ones six or none
    t = pd.to_datetime(s, format="mixed", utc=True)
    return (t - pd.Timestamp(0, tz="UTC")).dt.total_seconds().to_numpy(dtype=np.float64)


@dataclass
class TraceRecipe:
    name: str
    source: str
    ref: str
    arrivals: Callable[[object], np.ndarray]      # table -> arrival seconds, row order
    offset: int = 0
    limit: Optional[int] = None
    scale: float = 1.0                             # divide arrival times by this
    subsample: bool = False                        # keep one row in `scale` (maf)
    window: Optional[tuple] = None                 # keep arrivals in [lo, hi) after scaling


RECIPES: Dict[str, TraceRecipe] = {r.name: r for r in [
    TraceRecipe("burstgpt", "BurstGPT request log (CSV)", "evaluation/trace/burstgpt.py:13-60",
                lambda df: df["Timestamp"].to_numpy(dtype=np.float64), offset=474438, limit=775, scale=10.0),
    TraceRecipe("azurecode", "Azure LLM inference trace, code", "evaluation/trace/azurecode.py:13-92",
                lambda df: _wallclock_seconds(df["TIMESTAMP"]), offset=5100, limit=927),
    TraceRecipe("azureconv", "Azure LLM inference trace, conversation", "evaluation/trace/azureconv.py:13-85",
                lambda df: _wallclock_seconds(df["TIMESTAMP"])),
    TraceRecipe("maf", "Azure Functions invocation trace (CSV)", "evaluation/trace/maf.py:33-59",
                lambda df: (df["end_timestamp"] - df["duration"]).to_numpy(dtype=np.float64), offset=319091,
                scale=1000.0, subsample=True),
    TraceRecipe("debug", "a window of a MAF timestamp table", "evaluation/trace/debug.py:33-53",
                lambda df: df["timestamp"].to_numpy(dtype=np.float64), window=(0.53635e6, 0.53655e6)),
]}


def build(name: str, table, offset: Optional[int] = None, limit: Optional[int] = None,
          scale: Optional[float] = None, seed: int = 42) -> np.ndarray:
    """Arrival times (seconds) of trace ``name`` from its table (a pandas
    frame), cut to the recipe's slice unless ``offset`` / ``limit`` /
    ``scale`` override it."""
    r = RECIPES[name]
    off = r.offset if offset is None else offset
    lim = r.limit if limit is None else limit
    sc = r.scale if scale is None else scale
    t = r.arrivals(table) / sc
    t = t[off:]
    if lim is not None:
        t = t[:lim]
    if r.subsample and sc > 1:
        rng = np.random.default_rng(seed)
        keep = max(1, int(round(t.size / sc)))
        t = np.sort(rng.choice(t, size=keep, replace=False))
    if r.window is not None:
        lo, hi = r.window
        t = t[(t >= lo) & (t < hi)]
    return t


def rate_profile(t: np.ndarray, bin_s: float = 1.0) -> np.ndarray:
    """Requests per second in consecutive bins of ``bin_s`` seconds from the
    first arrival."""
    if t.size == 0:
        return np.zeros(0)
    rel = np.asarray(t, dtype=np.float64) - float(np.min(t))
    edges = np.arange(0.0, rel.max() + bin_s, bin_s)
    if edges.size < 2:
        edges = np.array([0.0, bin_s])
    return np.histogram(rel, bins=edges)[0] / bin_s


def names() -> List[str]:
    return sorted(RECIPES)
