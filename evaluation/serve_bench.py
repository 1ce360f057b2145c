"""Serving benchmark driver with the reference's command line
(parity: ``evaluation/bench.py:38-310``).

    python evaluation/serve_bench.py -c configs/llama3-8b.yaml [flags]
    python evaluation/serve_bench.py --model tiny-llama --dtype fp32 --nlimit 50 --qps 4 --cpu

Loads a dataset parquet (``prompt``/``prompt_len``/``response_len``; without
one, lognormal synthetic lengths), draws arrivals (Poisson, Gamma with
``--cv``, uniform, or a real trace parquet scaled by
``--time-scale-factor`` and thinned by ``--dataset-scale-factor``), starts
``nservers`` front ends and sends every request to the least-loaded one.
Every second it records an epoch (throughput, received, finished, mean
TTFT/TBT, memory demand, group states) to ``<log-path>/<log-name>.csv``;
per-request metrics go to ``.parquet``; the report prints mean/P50/P90/P99/
P999 of queueing, TTFT and TBT, throughput and SLO goodput.
"""
import argparse
import asyncio
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from kunserve_b200.config import ModelConfig, add_cli_args, get_cli_args  # noqa: E402
from kunserve_b200.evaluation.trace import arrivals, lognormal_lengths, load_parquet_trace, thin  # noqa: E402
from kunserve_b200.request import SamplingParams  # noqa: E402
from kunserve_b200.utils.metrics import SLO, percentiles, summarize  # noqa: E402

EPOCH_S = 1.0


def load_requests(cfg, vocab: int, rng):
    bc = cfg.bench_config
    n = bc.nlimit
    if bc.dataset:
        import pandas as pd
        df = pd.read_parquet(bc.dataset).iloc[bc.dataset_offset:bc.dataset_offset + n]
        if bc.shuffle_dataset:
            df = df.sample(frac=1.0, random_state=int(bc.seed))
        lens = list(zip(df["prompt_len"].astype(int), df["response_len"].astype(int)))
    else:
        pl = lognormal_lengths(n, 700, 1.0, 16, 8192, rng)
        ol = lognormal_lengths(n, 250, 1.0, 1, 2048, rng)
        lens = list(zip(pl, ol))
    out = []
    for p, o in lens:
        o = max(1, min(int(o), bc.max_model_len - 1))
        p = max(1, min(int(p), bc.max_model_len - o))
        out.append((rng.integers(0, vocab, p).tolist(), o))
    return out


def arrival_times(cfg, n, rng):
    bc = cfg.bench_config
    if bc.trace:
        ts = load_parquet_trace(bc.trace, bc.time_scale_factor, bc.trace_offset)
        ts = thin(ts, bc.dataset_scale_factor, int(bc.seed))
        return ts[:n]
    horizon = max(10.0, 4.0 * n / bc.qps)
    ts = arrivals(horizon, bc.qps, bc.dist, bc.cv, int(bc.seed))
    return ts[:n]


async def collect_epochs(servers, stop, rows):
    prev = time.perf_counter()
    t0 = prev
    while not stop.is_set():
        await asyncio.sleep(EPOCH_S)
        now = time.perf_counter()
        tok = fin = 0
        dem, states, ttft, tbt = [], [], [], []
        for s in servers:
            m = s.report_server_metrics()
            tok += m["tokens"]
            fin += m["finished"]
            dem += m["demand"]
            states += m["state"]
            a, b = s.pop_metrics()
            ttft += a
            tbt += b
        rows.append({"time": now - t0, "thpt": tok / (now - prev), "finished requests": fin,
                     "memory demand": float(np.mean(dem)) if dem else 0.0,
                     "mean ttft": float(np.mean(ttft)) if ttft else 0.0,
                     "mean tbt": float(np.mean(tbt)) if tbt else 0.0, "states": ";".join(states)})
        prev = now


async def run(args, cfg):
    from kunserve_b200.bootstrap import setup_kunserve
    mc = ModelConfig(cfg.bench_config.model or "tiny-llama", dtype=cfg.engine_config.dtype)
    rng = np.random.default_rng(int(cfg.bench_config.seed))
    reqs = load_requests(cfg, mc.get_vocab_size(), rng)
    times = arrival_times(cfg, len(reqs), rng)
    kw = {"num_gpu_blocks": cfg.bench_config.num_gpu_blocks}
    if args.cpu:
        kw.update(backend="torch", devices=["cpu"] * (cfg.engine_config.ngroups * cfg.engine_config.group_size *
                                                     cfg.engine_config.pp * cfg.engine_config.tp))
    servers = await setup_kunserve(cfg, model_config=mc, **kw)
    stop = asyncio.Event()
    rows = []
    epochs = asyncio.create_task(collect_epochs(servers, stop, rows))
    results = []
    t0 = time.time()

    async def one(i, prompt, olen, at):
        srv = min(servers, key=lambda s: s.get_unfinised_num())
        sp = SamplingParams(temperature=0.0, max_tokens=olen, ignore_eos=True)
        results.append(await srv.generate(prompt_token_ids=prompt, sampling_params=sp, request_id=i,
                                          arrival_time=t0 + at))

    tasks = []
    for i, ((prompt, olen), at) in enumerate(zip(reqs, times)):
        delay = t0 + at - time.time()
        if delay > 0:
            await asyncio.sleep(delay)
        tasks.append(asyncio.create_task(one(i, prompt, olen, float(at))))
    await asyncio.gather(*tasks)
    duration = time.time() - t0
    stop.set()
    await epochs
    for s in servers:
        await s.terminate()
    return results, rows, duration


def report(results, rows, duration, cfg, args):
    import pandas as pd
    ms = [r["metrics"] for r in results]
    slo = SLO(args.ttft_slo, args.tpot_slo)
    summ = summarize(ms, slo, duration)
    os.makedirs(cfg.bench_config.log_path, exist_ok=True)
    base = os.path.join(cfg.bench_config.log_path, cfg.bench_config.log_name)
    pd.DataFrame(rows).to_csv(base + ".csv", index=False)
    pd.DataFrame([{"request_id": m.request_id, "queue": m.queue, "ttft": m.ttft, "tbt": m.tbt, "e2e": m.e2e,
                   "num_tokens": m.num_tokens} for m in ms]).to_parquet(base + ".parquet")
    for name, vals in (("queue", [m.queue for m in ms]), ("ttft", [m.ttft for m in ms]),
                       ("tbt", [m.tbt for m in ms if m.num_tokens > 1])):
        p = percentiles(vals, (50, 90, 99, 99.9))
        print(f"{name:6s} mean {p['mean']:.4f}s  p50 {p['p50']:.4f}  p90 {p['p90']:.4f}  p99 {p['p99']:.4f}  "
              f"p999 {p['p999']:.4f}")
    print(f"throughput {summ['throughput_req_s']:.3f} req/s, {summ['throughput_tok_s']:.1f} tok/s; "
          f"SLO goodput {summ['goodput_req_s']:.3f} req/s (TTFT<={slo.ttft_s}s, TPOT<={slo.tpot_s}s)")
    return summ


def main(argv=None):
    p = add_cli_args(argparse.ArgumentParser("serve_bench"))
    p.add_argument("--cpu", action="store_true", help="torch backend on CPU ranks (no GPU)")
    p.add_argument("--ttft-slo", type=float, default=2.0)
    p.add_argument("--tpot-slo", type=float, default=0.1)
    args = p.parse_args(argv)
    cfg = get_cli_args(args)
    results, rows, duration = asyncio.run(run(args, cfg))
    return report(results, rows, duration, cfg, args)


if __name__ == "__main__":
    main()
