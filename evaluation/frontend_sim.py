"""Front-end pipeline simulation: how much of a two-stage pipeline's time the
host control plane leaves idle, with no GPU.

An instance with two pipeline stages and two virtual engines runs its real
scheduler, step building and output handling, but each stage worker is a
thread that sleeps ``--stage-ms`` per step (the device time) and hands the
step to the next stage through an event (the activation send).  The report
gives each stage's busy fraction and, per step, where the time between a
virtual engine's last stage finishing and its next step reaching stage 0
goes: result hand-back, output handling and next-batch preparation, the
event loop, step building, and dispatch to stage 0.  With no host time each
stage would be busy all the time; each millisecond of turnaround per step
costs about 1 / (2T + 1) of it.

    python evaluation/frontend_sim.py --stage-ms 14 --requests 600
"""
import argparse
import asyncio
import contextvars
import json
import os
import sys
import threading
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


class SleepStage:
    """A pipeline stage worker whose step takes ``t_s`` seconds."""

    def __init__(self, idx, t_s, pages, events, lock):
        self.idx, self.t_s, self.pages = idx, t_s, pages
        self.events, self.lock = events, lock
        self.log = []   # (step id, start, end, requests)

    def _event(self, key):
        with self.lock:
            return self.events.setdefault(key, threading.Event())

    def _profile_num_available_blocks(self, *args):
        return (self.pages, 0, 1)

    def init_model(self, *args):
        return None

    def clear_request_resource_batched(self, *args, **kwargs):
        return None

    def step(self, step, recv_from=None, send_to=None, last_stage=True):
        if recv_from is not None:
            self._event(step.step_id).wait(30)
        t0 = time.perf_counter()
        time.sleep(self.t_s)
        self.log.append((step.step_id, t0, time.perf_counter(), step.num_requests))
        if send_to is not None:
            self._event(step.step_id).set()
        return [1] * step.num_requests if last_stage else None


def simulate(stage_ms: float = 14.0, requests: int = 600, pages: int = 4000, seed: int = 1,
             prompt_range=(16, 128), output_range=(8, 64)) -> dict:
    from kunserve_b200.config import BalloonConfig, BenchConfig, CacheConfig, ModelConfig, ParallelConfig, SchedConfig
    from kunserve_b200.engine.instance import InstanceEngine
    from kunserve_b200.request import Request, SamplingParams
    from kunserve_b200.runtime.actors import ThreadActor

    mc = ModelConfig("tiny-llama", dtype="fp32")
    pc = ParallelConfig(pipeline_parallel_size=2, num_virtual_engine=2)
    cc = CacheConfig(block_size=16)
    sc = SchedConfig(policy="mixed", enable_chunked_prefill=True, chunked_prefill_budget=2048, max_batch_size=256)
    events, lock = {}, threading.Lock()
    stages = [SleepStage(i, stage_ms / 1000.0, pages, events, lock) for i in range(2)]
    eng = InstanceEngine(0, 0, mc, pc, cc, sc, BalloonConfig(), BenchConfig(),
                         [[ThreadActor(stages[0], "stage0")], [ThreadActor(stages[1], "stage1")]])
    rng = np.random.default_rng(seed)
    work = [(rng.integers(0, mc.arch.vocab_size, int(rng.integers(*prompt_range, endpoint=True))).tolist(),
             int(rng.integers(*output_range, endpoint=True))) for _ in range(requests)]

    # per virtual-engine step: start, forward dispatch, result back, end
    cur = contextvars.ContextVar("step", default=None)
    records = []
    orig_step, orig_fwd, orig_build = InstanceEngine._step, InstanceEngine._forward, InstanceEngine._build_step

    async def step(self, ve):
        rec = {"ve": ve, "t0": time.perf_counter()}
        cur.set(rec)
        await orig_step(self, ve)
        rec["t1"] = time.perf_counter()
        if "dispatch" in rec:
            records.append(rec)

    async def forward(self, reqs, fusion_exec, kv_rank, restore=None):
        rec = cur.get()
        if rec is not None:
            rec["dispatch"] = time.perf_counter()
        out = await orig_fwd(self, reqs, fusion_exec, kv_rank, restore)
        if rec is not None:
            rec["result"] = time.perf_counter()
        return out

    def build(self, reqs, inst, stage_layers, fusion_exec):
        st = orig_build(self, reqs, inst, stage_layers, fusion_exec)
        rec = cur.get()
        if rec is not None:
            rec["id"] = st.step_id
        return st

    done = set()

    async def run():
        InstanceEngine._step, InstanceEngine._forward, InstanceEngine._build_step = step, forward, build
        try:
            await eng.initialize()
            eng.output_callback = lambda outs: done.update(o.request_id for o in outs)
            for i, (prompt, n_out) in enumerate(work):
                eng.add_request(Request(0.0, i, None, prompt,
                                        SamplingParams(temperature=0.0, max_tokens=n_out, ignore_eos=True)))
            task = eng.launch()
            while len(done) < len(work):
                if task.done():
                    task.result()
                await asyncio.sleep(0.005)
            eng.terminate()
            await asyncio.wait_for(task, 30)
        finally:
            InstanceEngine._step, InstanceEngine._forward, InstanceEngine._build_step = orig_step, orig_fwd, orig_build

    asyncio.run(run())
    out = {"stage_ms": stage_ms, "requests": requests}
    for s in stages:
        span = s.log[-1][2] - s.log[0][1]
        out[f"stage{s.idx}_busy"] = round(sum(b - a for _, a, b, _ in s.log) / span, 3)
    end1 = {sid: b for sid, a, b, n in stages[1].log}
    start0 = {sid: a for sid, a, b, n in stages[0].log}
    chain = []
    recs = sorted((r for r in records if "id" in r and "result" in r), key=lambda r: r["t0"])
    for ve in {r["ve"] for r in recs}:
        lst = [r for r in recs if r["ve"] == ve]
        for a, b in zip(lst, lst[1:]):
            if a["id"] in end1 and b["id"] in start0:
                chain.append((a["result"] - end1[a["id"]], a["t1"] - a["result"], b["t0"] - a["t1"],
                              b["dispatch"] - b["t0"], start0[b["id"]] - b["dispatch"]))
    if chain:
        m = np.mean(np.array(chain), axis=0) * 1e3
        out["turnaround_ms"] = {"result_back": round(float(m[0]), 3), "outputs_and_next_batch": round(float(m[1]), 3),
                                "event_loop": round(float(m[2]), 3), "build_and_dispatch": round(float(m[3]), 3),
                                "dispatch_to_stage0": round(float(m[4]), 3), "total": round(float(m.sum()), 3)}
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--stage-ms", type=float, default=14.0, help="device time of one stage step")
    p.add_argument("--requests", type=int, default=600)
    p.add_argument("--pages", type=int, default=4000)
    a = p.parse_args(argv)
    print(json.dumps(simulate(a.stage_ms, a.requests, a.pages)))


if __name__ == "__main__":
    main()
