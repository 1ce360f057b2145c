import numpy as np
import pandas as pd

from kunserve_b200.evaluation.trace import Burst, arrivals, build_trace, load_parquet_trace, lognormal_lengths, thin
from kunserve_b200.utils.metrics import SLO, calculate_metrics, goodput, summarize


def test_periodic_bursts_make_a_stationary_load():
    from kunserve_b200.evaluation.trace import periodic_bursts
    b = periodic_bursts(0.0, 1.0, 2.0, 5.0, 600.0)
    assert len(b) == 300 and b[1].start == 2.0 and b[-1].start == 598.0
    t = arrivals(600, 5.0, "poisson", seed=3, bursts=b)
    # the mean over any 20 s window is close to the whole trace's mean
    mean = t.size / 600
    for s0 in (0, 100, 333, 500):
        assert abs(((t >= s0) & (t < s0 + 20)).sum() / 20 - mean) < 0.3 * mean
    on = sum(((t >= x.start) & (t < x.start + 1.0)).sum() for x in b[:100])
    off = sum(((t >= x.start + 1.0) & (t < x.start + 2.0)).sum() for x in b[:100])
    assert on > 3 * off


def test_poisson_rate_and_burst():
    t = arrivals(400, 5.0, "poisson", seed=1, bursts=[Burst(100, 100, 4.0)])
    base = ((t < 100).sum() + (t >= 200).sum()) / 300
    burst = ((t >= 100) & (t < 200)).sum() / 100
    assert abs(base - 5.0) < 0.6 and abs(burst - 20.0) < 2.0


def test_gamma_cv():
    t = arrivals(4000, 2.0, "gamma", cv=3.0, seed=2)
    gaps = np.diff(t)
    assert abs(gaps.mean() - 0.5) < 0.1
    assert 2.3 < gaps.std() / gaps.mean() < 3.7


def test_lognormal_mean_and_clip():
    x = lognormal_lengths(20000, 700, 1.0, 16, 8192, np.random.default_rng(0))
    assert x.min() >= 16 and x.max() <= 8192 and abs(x.mean() - 700) < 40


def test_trace_reproducible_and_parquet(tmp_path):
    a = build_trace(20, 3, seed=7)
    b = build_trace(20, 3, seed=7)
    assert [(r.arrival, r.prompt_len) for r in a] == [(r.arrival, r.prompt_len) for r in b]
    f = tmp_path / "t.parquet"
    pd.DataFrame({"timestamp": [10.0, 12.0, 11.0, 20.0]}).to_parquet(f)
    ts = load_parquet_trace(str(f), time_scale=2.0)
    assert list(ts) == [0.0, 0.5, 1.0, 5.0]
    assert len(thin(np.arange(1000.0), 0.3, seed=1)) < 400


def test_metrics_and_goodput():
    m = calculate_metrics([1.5, 1.6, 1.8], arrival_time=1.0, start_time=1.2)
    assert abs(m.ttft - 0.5) < 1e-9 and abs(m.tbt - 0.15) < 1e-9 and abs(m.queue - 0.2) < 1e-9
    slow = calculate_metrics([5.0, 5.1], arrival_time=1.0)
    assert goodput([m, slow], SLO(1.0, 0.2), duration_s=2.0) == 0.5
    s = summarize([m, slow], SLO(1.0, 0.2), 2.0)
    assert s["num_requests"] == 2 and s["ttft_p99"] > 3.9
