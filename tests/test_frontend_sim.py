"""The front-end pipeline simulation runs the real scheduler against two
sleeping stage workers and accounts for the host's share of each step."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_two_stage_pipeline_stays_mostly_busy():
    sys.path.insert(0, os.path.join(ROOT, "evaluation"))
    import frontend_sim
    out = frontend_sim.simulate(stage_ms=10.0, requests=120)
    assert out["stage0_busy"] > 0.6 and out["stage1_busy"] > 0.6, out
    t = out["turnaround_ms"]
    assert t["total"] > 0 and abs(sum(v for k, v in t.items() if k != "total") - t["total"]) < 0.01
