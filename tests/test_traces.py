"""Trace recipes: each public trace the reference converts becomes the same
arrival times (unit, time compression, window) from a local copy, and the
builder's parquet replays through the trace loader."""
import os
import subprocess
import sys

import numpy as np
import pandas as pd

from kunserve_b200.evaluation import traces
from kunserve_b200.evaluation.trace import load_parquet_trace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_every_reference_trace_has_a_recipe():
    assert traces.names() == ["azurecode", "azureconv", "burstgpt", "debug", "maf"]


def test_burstgpt_scales_seconds_and_cuts_the_window():
    df = pd.DataFrame({"Timestamp": np.arange(100, dtype=float) * 5.0})
    t = traces.build("burstgpt", df, offset=10, limit=20)
    assert t.size == 20
    np.testing.assert_allclose(t, np.arange(10, 30) * 5.0 / 10.0)   # ten times denser by default
    t1 = traces.build("burstgpt", df, offset=0, limit=None, scale=1.0)
    np.testing.assert_allclose(t1, df["Timestamp"].to_numpy())


def test_azure_wall_clock_stamps_of_both_layouts():
    old = pd.DataFrame({"TIMESTAMP": ["2023-11-16 18:15:46.6805900", "2023-11-16 18:15:47.1805900",
                                      "2023-11-16 18:15:49.0000000"]})
    t = traces.build("azureconv", old)
    np.testing.assert_allclose(np.diff(t), [0.5, 1.81941], atol=1e-4)
    new = pd.DataFrame({"TIMESTAMP": ["2024-05-10 00:00:00.250000+00:00", "2024-05-10 00:00:01+00:00",
                                      "2024-05-10 00:01:00+00:00"]})
    t = traces.build("azureconv", new)
    np.testing.assert_allclose(np.diff(t), [0.75, 59.0], atol=1e-6)
    assert t[0] > 1.7e9                                             # seconds since the epoch
    # azurecode's default window starts at row 5100: a short table keeps nothing
    assert traces.build("azurecode", new).size == 0
    assert traces.build("azurecode", new, offset=1, limit=1).size == 1


def test_maf_start_times_compressed_and_down_sampled():
    n = 5000
    end = np.arange(n, dtype=float) * 100.0 + 50.0
    df = pd.DataFrame({"end_timestamp": end, "duration": np.full(n, 50.0)})
    t = traces.build("maf", df, offset=0, scale=10.0)
    assert t.size == n // 10                                        # one in ten rows kept
    assert np.all(np.diff(t) >= 0)                                  # sorted
    starts = np.arange(n, dtype=float) * 100.0 / 10.0
    assert np.isin(t, starts).all()                                 # invocation starts, compressed
    # one row in ten over a tenth of the time: the original rate (one per 100 s)
    rate = t.size / (t.max() - t.min())
    assert abs(rate - 0.01) < 0.002
    again = traces.build("maf", df, offset=0, scale=10.0)
    np.testing.assert_array_equal(t, again)                         # seeded


def test_debug_window():
    ts = np.array([536000.0, 536350.0, 536400.5, 536549.9, 536550.0])
    t = traces.build("debug", pd.DataFrame({"timestamp": ts}))
    np.testing.assert_allclose(t, [536350.0, 536400.5, 536549.9])


def test_rate_profile():
    r = traces.rate_profile(np.array([10.0, 10.2, 10.9, 12.5]), 1.0)
    np.testing.assert_allclose(r, [3.0, 0.0, 1.0])
    assert traces.rate_profile(np.zeros(0)).size == 0


def test_builder_cli_round_trip(tmp_path):
    csv = tmp_path / "burst.csv"
    pd.DataFrame({"Timestamp": np.arange(50, dtype=float)}).to_csv(csv, index=False)
    out = tmp_path / "burst.parquet"
    r = subprocess.run([sys.executable, "evaluation/trace_builder.py", "--trace", "burstgpt", "--csv", str(csv),
                        "--out", str(out), "--offset", "5", "--limit", "20", "--scale", "2"],
                       cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "20 requests" in r.stdout
    arrivals = load_parquet_trace(str(out))
    assert len(arrivals) == 20
    listing = subprocess.run([sys.executable, "evaluation/trace_builder.py", "--list"], cwd=ROOT,
                             capture_output=True, text=True, timeout=120)
    assert listing.returncode == 0 and "maf" in listing.stdout


def test_workload_reports(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "evaluation"))
    import dataset_profile as dp
    r = dp.length_report([100, 16000, 50], [10, 1000, 5], max_len=16384)
    assert r["requests"] == 3 and r["capped"] == 1
    assert r["prompt_max"] == 15384 and r["output_max"] == 1000      # the prompt is cut, the output kept
    tr = dp.trace_report([5.0, 1.0, 3.0, 9.0], until=4.0)
    assert tr["requests"] == 4 and tr["span_s"] == 8.0
    assert tr["index_at_until"] == 2                                  # arrivals at 0, 2, 4, 8 s after the first
    table = tmp_path / "t.parquet"
    pd.DataFrame({"prompt": ["a", "b"], "prompt_len": [3, 4], "response_len": [1, 2]}).to_parquet(table)
    out = subprocess.run([sys.executable, "evaluation/dataset_profile.py", "--table", str(table)], cwd=ROOT,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and '"requests": 2' in out.stdout
