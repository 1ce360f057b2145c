"""The headline benchmark: its SLO accounting (bench.summarize) and its whole
flow on CPU ranks (fill to KV overload, timed window with the coordinator's
votes, drain through restore) with the PyTorch backend."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_only_requests_finished_inside_the_window_count():
    t0, t1 = 100.0, 101.0
    recs = {
        1: (99.0, [100.2, 100.25, 100.3], True, 3),      # finished inside, good
        2: (90.0, [96.0, 100.1, 100.3], True, 3),         # finished inside, TTFT 6 s: bad
        3: (99.9, [100.0, 100.5], True, 2),               # finished inside, TPOT 0.5 s: bad
        4: (99.0, [99.5, 99.55, 99.6, 100.5], False, 8),  # running, on track: 1 of 8 tokens inside
        5: (99.0, [99.1, 99.2], True, 2),                 # finished before the window: ignored
        6: (100.5, [100.9, 101.5], True, 4),              # first token inside, finishes after the window
        7: (100.8, [], False, 4),                         # queued: no token
    }
    sm = bench.summarize(recs, t0, t1, 2.0, 0.1)
    good, finished, ttft, tpot, gaps = sm["good"], sm["finished"], sm["ttft"], sm["tpot"], sm["gaps"]
    assert (good, finished) == (1, 3)
    # request-equivalents: 3/3 of request 1, 1/8 of request 4 (TPOT 0.33 s: bad), 1/4 of request 6
    assert abs(sm["equiv"] - (1.0 + 0.25)) < 1e-9
    assert sorted(round(x, 3) for x in ttft) == [0.1, 0.4, 1.2]   # first tokens inside the window: 3, 6, 1
    assert len(tpot) == 4                                      # requests 1-4 have two or more tokens
    assert gaps == 2 + 2 + 1 + 1


def _run(cmd, timeout=900):
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, r.stdout[-3000:]
    return json.loads(lines[-1])


SMALL = ["--device", "cpu", "--model", "tiny-llama", "--backlog", "64", "--max-batch", "32", "--budget", "512",
         "--steps", "12", "--warmup", "3", "--drain-timeout", "60"]


@pytest.mark.slow
def test_bench_cpu_one_rank_starts_loaded():
    line = _run([sys.executable, "bench.py", "--gpus", "1", "--kv-gb", "0.003", "--no-baseline"] + SMALL)
    assert line["kv_used_at_start"] >= 0.95 and line["queued_at_start"] >= 32
    assert line["running_at_start"] > 0 and line["tpot_samples"] > 0
    assert line["e2e"]["api"] == "AsyncLLM.generate"
    assert line["value"] >= 0


@pytest.mark.slow
def test_bench_cpu_four_ranks_balloon_cycle():
    """Two TP2 instances in one balloon group on four gloo ranks: the vote
    fires inside the timed window and the group restores and splits after
    the burst ends."""
    line = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "4",
                 "--master-addr", "127.0.0.1", "--master-port", "29641", "bench.py", "--gpus", "4",
                 "--kv-gb", "0.0015", "--no-e2e"] + SMALL)
    assert line["config"]["parallelism"].startswith("tp2xdp2")
    assert line["transitions_in_window"] == [["INITIAL->BALLOON"]]
    names = [t[0] for t in line["transitions"][0]]
    assert names == ["INITIAL->BALLOON", "BALLOON->RESTORE", "RESTORE->INITIAL"]
    assert line["restored_gb"] > 0
    assert line["baseline"]["value"] >= 0 and line["vs_baseline"] is not None
