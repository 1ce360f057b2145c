"""Headline benchmark: serving goodput with P99 TTFT/TPOT under a bursty,
KV-overloading request trace (Llama-3-8B, bf16, one data-parallel instance
per GPU, random-init weights, synthetic seeded trace).

    python bench.py --gpus N --steps K --warmup W            # N=1
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Every rank serves its own instance with the same per-GPU arrival rate (weak
scaling): Poisson arrivals with periodic 5x bursts (1 s every 2 s), so the
offered load is bursty but the same over any window of the trace.  After W warm-up steps the trace is replayed in real time and
exactly K engine steps are timed with CUDA events on the engine's stream
(barrier + synchronize on both sides, max over ranks).  ``value`` is the
whole-job SLO goodput: requests that finished inside the window and met both
the TTFT and the TPOT objective, divided by the window.  ``e2e`` repeats the
measurement through the public API (``AsyncLLM.generate``), timed on the
host, with every step's inputs copied host-to-device from pinned memory and
its sampled ids read back.

``--impl reference`` runs the reference implementation through its own API;
its native engine is absent from its source tree, so it reports why it is
unavailable.
"""
import argparse
import asyncio
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

MAX_LEN = 8192      # Llama-3-8B context: prompt + output are clipped to it
METRIC = "P99 TTFT/TPOT + SLO goodput (req/s) under bursty overload, max over ranks"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2500)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="llama-3-8b")
    p.add_argument("--rate", type=float, default=5.0, help="base arrivals per second per GPU")
    # 1 s bursts at 5x every 2 s (15 req/s/GPU on average): the window is a
    # fixed number of steps, so the offered load must not depend on how far
    # into the trace it reaches, or a faster engine would see a lower rate;
    # --burst-period 0 gives one burst [start, start + len)
    p.add_argument("--burst-factor", type=float, default=5.0)
    p.add_argument("--burst-start", type=float, default=0.0)
    p.add_argument("--burst-len", type=float, default=1.0)
    p.add_argument("--burst-period", type=float, default=2.0)
    p.add_argument("--kv-gb", type=float, default=20.0)
    # 64-token pages: the decode attention kernel streams K/V in one TMA box
    # per 64 keys and head half (16-token pages need four, and cap it near
    # 0.6 of HBM bandwidth); fragmentation stays near 32 tokens per request
    p.add_argument("--block-size", type=int, default=64)
    p.add_argument("--budget", type=int, default=2048, help="chunked-prefill token budget per step")
    p.add_argument("--max-batch", type=int, default=256)
    p.add_argument("--ttft-slo", type=float, default=2.0)
    p.add_argument("--tpot-slo", type=float, default=0.1)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--no-e2e", action="store_true")
    return p.parse_args()


def reference_unavailable(args):
    why = None
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isdir(ref):
        why = "reference not installed under baseline/_ref"
    else:
        code = f"import sys; sys.path.insert(0, {ref!r}); import kunserve"
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            last = (r.stderr.strip().splitlines() or ["import failed"])[-1]
            why = ("the reference's native engine (FlashTransformer submodule) is absent from its source tree; "
                   f"`import kunserve` fails: {last[:200]}")
    if why is None:
        why = "the reference imported, but its serving path needs Ray and its native LlamaOp, neither present"
    return {"impl": "reference", "unavailable": why, "metric": METRIC, "n_gpus": args.gpus}


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", ",".join(str(g) for g in self.gpus), "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def pct(vals, q):
    return float(np.percentile(np.asarray(vals), q)) if len(vals) else float("nan")


async def timed_engine_run(inst, trace, steps, t_window_start_cb, sync, sp_factory):
    """Replay ``trace`` into the instance in real time until ``steps`` engine
    steps ran.  Returns finished-request records and step count."""
    from kunserve_b200.request import Request

    finished = {}
    first_tok = {}

    def on_out(outs):
        for o in outs:
            finished[o.request_id] = (o.arrival_time, [t.new_token_time for t in o.outputs], True)

    inst.output_callback = on_out
    inst.step_log = []
    t0 = time.time()
    t_window_start_cb()
    loop_task = asyncio.create_task(inst.start_event_loop())

    async def feed():
        for i, r in enumerate(trace):
            delay = t0 + r.arrival - time.time()
            if delay > 0:
                await asyncio.sleep(delay)
            prompt = r.prompt[:max(1, MAX_LEN - r.output_len)]
            inst.add_request(Request(t0 + r.arrival, i, None, prompt, sp_factory(r)))

    feeder = asyncio.create_task(feed())
    while len(inst.step_log) < steps:
        if loop_task.done():
            loop_task.result()
        await asyncio.sleep(0.0005)
    inst.stopped = True
    end_wall = time.time()
    sync()
    feeder.cancel()
    inst.terminate()
    await asyncio.wait_for(loop_task, 30)
    return list(finished.values()) + in_flight(inst), end_wall, t0


def in_flight(inst):
    """(arrival, token times, finished=False) of every request still in the
    instance (queued or running) when the window closes."""
    reqs = list(inst.unaccepted_queue) + [r for s in inst.scheduler for r in s.all_requests()]
    return [(r.arrival_time, [o.new_token_time for o in r.outputs], False) for r in reqs]


def summarize(records, t_end, slo_ttft, slo_tpot):
    """SLO accounting at the end of the window.  A request that arrived in
    the window counts as good when it finished inside it within both
    objectives, or is still on track at the window's end: first token within
    the TTFT objective and mean inter-token time so far within the TPOT
    objective, or no token yet but younger than the TTFT objective.  Counting
    on-track requests keeps the goodput a rate of the offered load that does
    not depend on how many requests happen to straddle the window's end."""
    ttft, tpot, ok = [], [], 0
    for arrival, times, finished in records:
        if arrival > t_end:
            continue
        times = [t for t in times if t <= t_end]
        if times:
            a = times[0] - arrival
            b = (times[-1] - times[0]) / (len(times) - 1) if len(times) > 1 else 0.0
            ttft.append(a)
            if len(times) > 1:
                tpot.append(b)
            good = a <= slo_ttft and b <= slo_tpot
        else:
            good = not finished and t_end - arrival <= slo_ttft
        ok += int(good)
    return ttft, tpot, ok


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(reference_unavailable(args)), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    from kunserve_b200.config import (BalloonConfig, BenchConfig, CacheConfig, ModelConfig, ParallelConfig,
                                      SchedConfig)
    from kunserve_b200.control.group import GroupEngine
    from kunserve_b200.engine.instance import InstanceEngine
    from kunserve_b200.engine.worker import Worker
    from kunserve_b200.evaluation.trace import build_trace, periodic_bursts
    from kunserve_b200.llm import AsyncLLM
    from kunserve_b200.config.kunserve_config import KunServeConfig
    from kunserve_b200.request import SamplingParams
    from kunserve_b200.runtime import LocalActor
    from kunserve_b200.runtime.streams import StreamRouter
    from kunserve_b200.ops import check_error

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=dev)

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    mc = ModelConfig(args.model, dtype="bf16")
    pc = ParallelConfig()
    kv_bytes = int(args.kv_gb * 1e9)
    cc = CacheConfig(block_size=args.block_size, kv_budget_bytes=kv_bytes)
    sc = SchedConfig(policy="mixed", enable_chunked_prefill=True, chunked_prefill_budget=args.budget,
                     max_batch_size=args.max_batch, max_tokens_per_batch=args.budget)
    worker = Worker(rank, mc, cc, pc, backend="native", device=f"cuda:{local}", seed=args.seed)
    bench_cfg = BenchConfig(model=args.model, max_model_len=MAX_LEN)
    inst = InstanceEngine(0, rank, mc, pc, cc, sc, BalloonConfig(), bench_cfg, [[LocalActor(worker)]])
    pages = kv_bytes // worker.block_bytes(args.block_size)

    async def init():
        await inst.initialize(num_gpu_blocks=pages)
    asyncio.run(init())
    runner = worker.runner
    sp = lambda r: SamplingParams(temperature=0.0, max_tokens=max(1, r.output_len), ignore_eos=True)

    # ---------------- warm-up: W steps on a small request set
    warm = build_trace(1.0, 8.0, seed=args.seed + 7 + rank, prompt_mean=600, output_mean=8,
                       output_range=(2, 16), vocab=mc.get_vocab_size())

    async def warmup():
        from kunserve_b200.request import Request
        inst.output_callback = lambda outs: None
        for i, r in enumerate(warm):
            inst.add_request(Request(time.time(), 10_000_000 + i, None, r.prompt, sp(r)))
        task = asyncio.create_task(inst.start_event_loop())
        while len(inst.step_log) < args.warmup and not task.done():
            await asyncio.sleep(0.001)
        inst.stopped = True
        inst.terminate()
        await asyncio.wait_for(task, 60)
    asyncio.run(warmup())
    inst.reset()
    check_error()

    trace = build_trace(600.0, args.rate, "poisson", seed=args.seed + 1000 * rank,
                        bursts=periodic_bursts(args.burst_start, args.burst_len, args.burst_period,
                                               args.burst_factor, 600.0),
                        vocab=mc.get_vocab_size())

    # ---------------- timed run through the instance engine (device-timed)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(list(range(world)) if rank == 0 else [])
    barrier_sync()
    launches0, h2d0, d2h0, steps0 = runner.eng.launches(), runner.h2d_bytes, runner.d2h_bytes, runner.num_steps
    gpu0 = runner.gpu_ms
    if rank == 0:
        clocks.start()

    def window_start():
        ev0.record(torch.cuda.current_stream(dev))

    def window_end():
        ev1.record(torch.cuda.current_stream(dev))
        torch.cuda.synchronize(dev)

    records, t_end, t0 = asyncio.run(timed_engine_run(inst, trace, args.steps, window_start, window_end, sp))
    clock_info = clocks.stop() if rank == 0 else None
    dev_ms = ev0.elapsed_time(ev1)
    barrier_sync()
    n_steps = runner.num_steps - steps0
    launches = runner.eng.launches() - launches0
    h2d = (runner.h2d_bytes - h2d0) / max(n_steps, 1)
    d2h = (runner.d2h_bytes - d2h0) / max(n_steps, 1)
    check_error()
    ttft, tpot, ok = summarize(records, t0 + dev_ms / 1000.0, args.ttft_slo, args.tpot_slo)
    preempt = inst.get_num_preemption()
    local_res = {"dev_ms": dev_ms, "ttft": ttft, "tpot": tpot, "ok": ok, "launches": launches,
                 "fwd_gpu_ms": runner.gpu_ms - gpu0,
                 "h2d": h2d, "d2h": d2h, "n_steps": n_steps, "preempt": preempt,
                 "finished": sum(1 for a, tt, fin in records if fin and tt and tt[-1] <= t0 + dev_ms / 1000.0),
                 "arrived": sum(1 for r in trace if r.arrival <= dev_ms / 1000.0)}
    inst.reset()

    # ---------------- end-to-end through the public API (host-timed)
    e2e_res = None
    if not args.no_e2e:
        cfg = KunServeConfig(bench_config=bench_cfg)

        async def e2e():
            router = StreamRouter(asyncio.get_running_loop())
            inst.output_callback = router
            llm = AsyncLLM(cfg, mc, [GroupEngine(0, [inst])], router)
            llm.start()
            inst.step_log = []
            results = []
            t_start = time.time()

            async def one(i, r):
                res = await llm.generate(prompt_token_ids=r.prompt[:max(1, MAX_LEN - r.output_len)],
                                         sampling_params=sp(r), request_id=i,
                                         arrival_time=t_start + r.arrival)
                results.append(res)

            async def feed():
                tasks = []
                for i, r in enumerate(trace):
                    delay = t_start + r.arrival - time.time()
                    if delay > 0:
                        await asyncio.sleep(delay)
                    tasks.append(asyncio.create_task(one(i, r)))
                return tasks
            feeder = asyncio.create_task(feed())
            while len(inst.step_log) < args.steps:
                await asyncio.sleep(0.0005)
            t_stop = time.time()
            inst.stopped = True
            feeder.cancel()
            llm.coordinator.stop()
            inst.terminate()
            await asyncio.sleep(0.05)
            recs = [(t_start + trace[r["request_id"]].arrival, r["metrics"].token_times, True) for r in results]
            return recs + in_flight(inst), t_stop - t_start, t_start
        recs, wall, ts = asyncio.run(e2e())
        e_ttft, e_tpot, e_ok = summarize(recs, ts + wall, args.ttft_slo, args.tpot_slo)
        e2e_res = {"wall_s": wall, "ok": e_ok, "ttft": e_ttft, "tpot": e_tpot}

    # ---------------- reduce over ranks
    if world > 1:
        allres = [None] * world
        dist.all_gather_object(allres, (local_res, e2e_res))
    else:
        allres = [(local_res, e2e_res)]
    if rank == 0:
        win_s = max(r[0]["dev_ms"] for r in allres) / 1000.0
        ok = sum(r[0]["ok"] for r in allres)
        ttft = [x for r in allres for x in r[0]["ttft"]]
        tpot = [x for r in allres for x in r[0]["tpot"]]
        value = ok / win_s
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "req/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(win_s * 1000.0 / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": (f"synthetic: seeded Poisson {args.rate} req/s/GPU with {args.burst_factor}x bursts of "
                     f"{args.burst_len} s every {args.burst_period} s from {args.burst_start} s"
                     f" (one burst when the period is 0), lognormal prompt (mean 700, "
                     "sigma 1, [16,8192]) and output (mean 250, [1,2048]) lengths; random-init N(0,0.02) weights"),
            "config": {"model": args.model, "global_batch": args.max_batch * world, "seq_len": MAX_LEN,
                       "parallelism": f"dp{world}", "kv_budget_gb_per_gpu": args.kv_gb,
                       "block_size": args.block_size, "chunked_prefill_budget": args.budget,
                       "slo": {"ttft_s": args.ttft_slo, "tpot_s": args.tpot_slo},
                       "l2": "inputs larger than L2: the 16 GB of weights stream through every step",
                       "policy": "mixed prefill+decode batches, recompute preemption"},
            "p99_ttft_s": round(pct(ttft, 99), 4), "p99_tpot_s": round(pct(tpot, 99), 5),
            "p50_ttft_s": round(pct(ttft, 50), 4), "p50_tpot_s": round(pct(tpot, 50), 5),
            "finished": sum(r[0]["finished"] for r in allres), "arrived": sum(r[0]["arrived"] for r in allres),
            "preemptions": sum(r[0]["preempt"] for r in allres), "window_s": round(win_s, 3),
            "gpu_launches": int(sum(r[0]["launches"] for r in allres)),
            # share of the window the device spent inside forward() (the rest is
            # host-side scheduling between steps and idle time between arrivals)
            "forward_busy_frac": round(max(r[0]["fwd_gpu_ms"] / r[0]["dev_ms"] for r in allres), 3),
            "clocks": clock_info,
        }
        if e2e_res is not None:
            ew = max(r[1]["wall_s"] for r in allres)
            eok = sum(r[1]["ok"] for r in allres)
            ettft = [x for r in allres for x in r[1]["ttft"]]
            etpot = [x for r in allres for x in r[1]["tpot"]]
            line["e2e"] = {"value": round(eok / ew, 4), "unit": "req/s", "api": "AsyncLLM.generate",
                           "p99_ttft_s": round(pct(ettft, 99), 4), "p99_tpot_s": round(pct(etpot, 99), 5),
                           "h2d_bytes_per_step": int(np.mean([r[0]["h2d"] for r in allres])),
                           "d2h_bytes_per_step": int(np.mean([r[0]["d2h"] for r in allres])),
                           "window_s": round(ew, 3)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
