"""SLO accounting of the headline benchmark (bench.summarize)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_finished_and_on_track_requests_count():
    t_end = 100.0
    recs = [
        (0.0, [0.5, 0.6, 0.7], True),          # finished, good
        (0.0, [3.0, 3.1], True),               # finished, TTFT 3 s: bad
        (90.0, [90.2] + [90.2 + 0.05 * i for i in range(1, 30)], False),   # running, on track
        (99.0, [], False),                     # queued 1 s: still on track
        (95.0, [], False),                     # queued 5 s: TTFT already missed
        (96.0, [96.1, 96.5], False),           # running, TPOT 0.4 s: bad
        (101.0, [], False),                    # arrives after the window: ignored
        (10.0, [10.1, 200.0], True),           # finished after the window: judged on what it had
    ]
    ttft, tpot, ok = bench.summarize(recs, t_end, 2.0, 0.1)
    assert ok == 4
    assert len(ttft) == 5 and len(tpot) == 4
