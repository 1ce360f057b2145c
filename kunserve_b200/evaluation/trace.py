"""Request traces: arrival processes and prompt/output length distributions.

Parity: ``evaluation/trace.py`` — dataset slices (:11-38), real-trace
intervals scaled by a time factor (:40-60), Gamma / exponential / uniform
inter-arrivals (:62-72, Gamma with shape 1/cv^2 and scale cv^2*mean) and a
seeded async generator (:84-96) — plus what the benchmark configurations
need: bursts (windows where the rate is multiplied) and lognormal lengths
clipped to a range.  Everything is seeded, so a trace is reproducible.
"""
import asyncio
import math
from dataclasses import dataclass, field
from typing import Iterator, List, Optional, Sequence, Tuple

import numpy as np


@dataclass
class TraceRequest:
    arrival: float       # seconds from trace start
    prompt_len: int
    output_len: int
    prompt: Optional[List[int]] = None


@dataclass
class Burst:
    start: float         # seconds
    duration: float
    factor: float        # rate multiplier inside the window


def periodic_bursts(start: float, length: float, period: float, factor: float, duration: float) -> List[Burst]:
    """Bursts of ``length`` seconds every ``period`` seconds from ``start``:
    the offered load is bursty at the period's scale but stationary over
    longer windows (mean rate x (1 + (factor - 1) * length / period))."""
    if period <= 0:
        return [Burst(start, length, factor)]
    n = max(0, int(math.ceil((duration - start) / period)))
    return [Burst(start + k * period, length, factor) for k in range(n)]


def _rate_at(t: float, rate: float, bursts: Sequence[Burst]) -> float:
    r = rate
    for b in bursts:
        if b.start <= t < b.start + b.duration:
            r *= b.factor
    return r


def arrivals(duration: float, rate: float, dist: str = "poisson", cv: float = 1.0, seed: int = 42,
             bursts: Sequence[Burst] = ()) -> np.ndarray:
    """Arrival times in ``[0, duration)``.  Inter-arrival gaps are drawn at the
    base rate and divided by the burst factor in force (time change), which
    keeps Gamma burstiness inside bursts."""
    rng = np.random.default_rng(seed)
    out, t = [], 0.0
    while True:
        if dist == "poisson":
            gap = rng.exponential(1.0 / rate)
        elif dist == "gamma":
            shape = 1.0 / (cv * cv)
            gap = rng.gamma(shape, (cv * cv) / rate)
        elif dist == "uniform":
            gap = 1.0 / rate
        else:
            raise ValueError(f"unknown arrival distribution {dist!r}")
        t += gap * rate / _rate_at(t, rate, bursts)
        if t >= duration:
            break
        out.append(t)
    return np.asarray(out)


def trace_intervals(timestamps: Sequence[float], time_scale: float = 1.0) -> np.ndarray:
    """Arrival offsets of a real trace (first arrival at 0), time-scaled."""
    ts = np.sort(np.asarray(timestamps, dtype=np.float64))
    return (ts - ts[0]) / time_scale


def thin(times: np.ndarray, keep: float, seed: int = 42) -> np.ndarray:
    """Bernoulli thinning (the reference's ``dataset_scale_factor``)."""
    if keep >= 1.0:
        return times
    rng = np.random.default_rng(seed)
    return times[rng.random(times.size) < keep]


def lognormal_lengths(n: int, mean: float, sigma: float, lo: int, hi: int, rng) -> np.ndarray:
    """Lognormal with the given *mean* (not median), clipped to [lo, hi]."""
    mu = math.log(mean) - sigma * sigma / 2.0
    return np.clip(np.round(rng.lognormal(mu, sigma, n)), lo, hi).astype(np.int64)


def uniform_lengths(n: int, lo: int, hi: int, rng) -> np.ndarray:
    """Integers uniform in [lo, hi] (both ends included)."""
    return rng.integers(lo, hi + 1, n).astype(np.int64)


def build_trace(duration: float, rate: float, dist: str = "poisson", cv: float = 1.0, seed: int = 42,
                bursts: Sequence[Burst] = (), prompt_mean: float = 700, prompt_sigma: float = 1.0,
                prompt_range=(16, 8192), output_mean: float = 250, output_sigma: float = 1.0,
                output_range=(1, 2048), vocab: int = 32000, with_tokens: bool = True,
                lengths: str = "lognormal", backlog: int = 0) -> List[TraceRequest]:
    """Seeded requests.  ``lengths="uniform"`` draws prompt and output lengths
    uniformly from their ranges (the tiny-model configuration); otherwise
    lognormal with the given means.  ``backlog`` requests arrive at time 0
    before the arrival process starts (a burst already queued)."""
    ts = arrivals(duration, rate, dist, cv, seed, bursts)
    if backlog:
        ts = np.concatenate([np.zeros(backlog), ts])
    rng = np.random.default_rng(seed + 1)
    if lengths == "uniform":
        pl = uniform_lengths(ts.size, *prompt_range, rng)
        ol = uniform_lengths(ts.size, *output_range, rng)
    else:
        pl = lognormal_lengths(ts.size, prompt_mean, prompt_sigma, *prompt_range, rng)
        ol = lognormal_lengths(ts.size, output_mean, output_sigma, *output_range, rng)
    out = []
    for t, p, o in zip(ts, pl, ol):
        toks = rng.integers(0, vocab, int(p)).tolist() if with_tokens else None
        out.append(TraceRequest(float(t), int(p), int(o), toks))
    return out


def load_parquet_trace(path: str, time_scale: float = 1.0, offset: int = 0, limit: Optional[int] = None):
    """Timestamps from a trace parquet (e.g. the BurstGPT traces)."""
    import pandas as pd

    df = pd.read_parquet(path)
    col = next(c for c in df.columns if "time" in c.lower())
    ts = df[col].to_numpy(dtype=np.float64)[offset:]
    if limit is not None:
        ts = ts[:limit]
    return trace_intervals(ts, time_scale)


async def replay(trace: Sequence[TraceRequest], submit, t0: Optional[float] = None, clock=None):
    """Call ``submit(req)`` at each request's arrival time (seconds after t0)."""
    loop = asyncio.get_running_loop()
    now = clock or loop.time
    t0 = now() if t0 is None else t0
    tasks = []
    for r in trace:
        delay = t0 + r.arrival - now()
        if delay > 0:
            await asyncio.sleep(delay)
        res = submit(r)
        if asyncio.iscoroutine(res):
            tasks.append(asyncio.create_task(res))
    return tasks
