"""Per-request latency metrics and aggregate serving statistics.

Per-request metrics follow ``kunserve/metrics.py:4-24``: queueing delay,
time-to-first-token (TTFT), mean time-between-tokens (TBT, also called TPOT),
end-to-end latency and the per-token timestamps.  The aggregate helpers add
what the reference's bench driver prints (``evaluation/bench.py:273-284``:
mean/P50/P90/P99/P999) plus SLO goodput: requests per second that met both
the TTFT and the TPOT objective.
"""
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np


@dataclass
class RequestMetrics:
    request_id: int
    arrival: float
    queue: float          # arrival -> first scheduled
    ttft: float           # arrival -> first token
    tbt: float            # mean gap between consecutive tokens (0 if < 2 tokens)
    e2e: float            # arrival -> last token
    num_tokens: int
    token_times: List[float] = field(default_factory=list)


def calculate_metrics(token_times: Sequence[float], arrival_time: float,
                      start_time: Optional[float] = None,
                      request_id: int = -1) -> RequestMetrics:
    """Metrics of one finished request from its token timestamps."""
    times = list(token_times)
    if not times:
        return RequestMetrics(request_id, arrival_time, 0.0, float("inf"), 0.0,
                              float("inf"), 0, [])
    first, last = times[0], times[-1]
    tbt = (last - first) / (len(times) - 1) if len(times) > 1 else 0.0
    queue = (start_time - arrival_time) if start_time is not None else 0.0
    return RequestMetrics(request_id, arrival_time, max(queue, 0.0), first - arrival_time,
                          tbt, last - arrival_time, len(times), times)


def percentiles(values: Iterable[float], qs=(50, 90, 99, 99.9)) -> Dict[str, float]:
    arr = np.asarray(list(values), dtype=np.float64)
    out = {"mean": float(arr.mean()) if arr.size else float("nan")}
    for q in qs:
        key = f"p{q:g}".replace(".", "")
        out[key] = float(np.percentile(arr, q)) if arr.size else float("nan")
    return out


@dataclass
class SLO:
    ttft_s: float
    tpot_s: float


def goodput(metrics: Sequence[RequestMetrics], slo: SLO, duration_s: float) -> float:
    """Requests per second that met both SLOs over ``duration_s``."""
    if duration_s <= 0:
        return 0.0
    ok = sum(1 for m in metrics if m.ttft <= slo.ttft_s and m.tbt <= slo.tpot_s)
    return ok / duration_s


def summarize(metrics: Sequence[RequestMetrics], slo: SLO, duration_s: float) -> Dict[str, float]:
    ttft = percentiles(m.ttft for m in metrics)
    tbt = percentiles(m.tbt for m in metrics if m.num_tokens > 1)
    queue = percentiles(m.queue for m in metrics)
    tokens = sum(m.num_tokens for m in metrics)
    return {
        "num_requests": len(metrics),
        "duration_s": duration_s,
        "throughput_req_s": len(metrics) / duration_s if duration_s > 0 else 0.0,
        "throughput_tok_s": tokens / duration_s if duration_s > 0 else 0.0,
        "goodput_req_s": goodput(metrics, slo, duration_s),
        **{f"ttft_{k}": v for k, v in ttft.items()},
        **{f"tpot_{k}": v for k, v in tbt.items()},
        **{f"queue_{k}": v for k, v in queue.items()},
    }
