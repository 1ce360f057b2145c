"""Headline benchmark: SLO goodput with P99 TTFT/TPOT while a burst
overloads KV memory (Llama-2-13B, bf16, random-init weights, synthetic
seeded trace).

    python bench.py --gpus 1 --steps K --warmup W
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Serving shape: one GPU serves the model alone (TP1); N >= 2 GPUs serve N/2
tensor-parallel (TP2) instances, grouped in balloon groups of two instances
when there are at least two, so that KV overload triggers the parameter drop
into TP2 x PP2 pipelines with live KV migration (the benchmark
configuration's config 3, scaled to N).  Rank 0 runs the front end
(coordinator, group and instance engines); every rank hosts its GPU's worker.

Timed region.  The trace starts with a burst already queued (a backlog of
``--backlog`` requests per instance at time 0) followed by Gamma(CV) arrivals
at the burst rate.  Untimed: W warm-up steps on a small request set, then a
fill phase that serves the backlog until every instance's KV pages are at
least 95 % used and more than ``max_batch`` requests wait, then W more steps.
Then the engines pause, every worker records a CUDA event, the coordinator's
load collection and balloon state machine start, serving resumes, and
exactly K engine steps (forward passes of GPU 0) run; every worker records a
second event.  The window is the largest device time between the two events
over all workers.  After the window the burst ends (queued requests are
dropped) and serving continues untimed until every group is back in its
initial state, which measures parameter restore.

``value`` is the SLO goodput in request-equivalents per second of window,
over the whole job: every token emitted inside the window counts
1/output-length of a request when its request met TTFT <= ``--ttft-slo`` and
keeps a mean inter-token time <= ``--tpot-slo`` (``summarize``); the plain
count of requests that finished inside the window within both objectives is
reported as ``finished_goodput``.  ``vs_baseline`` divides it by the
same measurement in library-baseline mode, run in the same invocation on the
same job and trace: every GEMM through ATen/cuBLAS with unfused epilogues,
NCCL all-reduce, NCCL send/recv for KV migration and parameter restore.
``e2e`` repeats the measurement through the public API
(``AsyncLLM.generate``), timed on the host; every step copies its metadata
host-to-device from pinned memory and reads the sampled ids back.

``--impl reference`` runs the reference implementation through its own API;
its native engine is absent from its source tree, so it reports why it is
unavailable.
"""
import argparse
import asyncio
import gc
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

METRIC = "P99 TTFT/TPOT + SLO goodput (req/s) under bursty overload, max over ranks"


# interval of the front end's polls of worker 0 during warm-up and the
# timed window (the window's end is marked on the device by worker 0 itself)
POLL_S = 0.002


class GcWatch:
    """Seconds the front end spent in garbage collections (gc.callbacks): a
    full collection over the heap of thousands of live requests pauses the
    event loop, and with it every step dispatch."""

    def __init__(self):
        self.total, self.longest, self.count, self._t = 0.0, 0.0, 0, None

    def __call__(self, phase, info):
        if phase == "start":
            self._t = time.perf_counter()
        elif self._t is not None:
            dt = time.perf_counter() - self._t
            self.total += dt
            self.longest = max(self.longest, dt)
            self.count += 1
            self._t = None

def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="llama-2-13b")
    p.add_argument("--tp", type=int, default=None, help="default: 1 on one GPU, else 2")
    p.add_argument("--group-size", type=int, default=None,
                   help="instances per balloon group (default: 2 when there are at least two instances)")
    p.add_argument("--balloon-mode", default="reshard", choices=["recompute", "reshard", "livereshard"])
    p.add_argument("--kv-gb", type=float, default=8.0, help="KV-cache budget per GPU (GB)")
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--budget", type=int, default=2048, help="chunked-prefill token budget per step")
    p.add_argument("--max-batch", type=int, default=256)
    p.add_argument("--rate", type=float, default=1.5, help="mean arrivals per second per GPU outside bursts")
    p.add_argument("--cv", type=float, default=4.0, help="coefficient of variation of Gamma inter-arrivals")
    p.add_argument("--burst-factor", type=float, default=5.0)
    p.add_argument("--backlog", type=int, default=768, help="requests per instance queued when the trace starts")
    p.add_argument("--prompt-range", type=int, nargs=2, default=[16, 128])
    p.add_argument("--output-range", type=int, nargs=2, default=[8, 64])
    p.add_argument("--ttft-slo", type=float, default=2.0)
    p.add_argument("--tpot-slo", type=float, default=0.1)
    p.add_argument("--drain-timeout", type=float, default=90.0,
                   help="seconds after the window to wait for restore and split")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-baseline", action="store_true")
    p.add_argument("--device", default="cuda", choices=["cuda", "cpu"],
                   help="cpu: plumbing check of the same flow on gloo ranks with the PyTorch backend")
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
    """nvidia-smi samples (SM clock, throttle reasons) kept for the timed
    region: sampling starts before the window (nvidia-smi takes a moment to
    start) and only samples stamped inside it, widened by one sampling
    period on each side, are summarised."""

    PERIOD_S = 0.1
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", ",".join(str(g) for g in self.gpus), "-lms",
                                          str(int(self.PERIOD_S * 1000))],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, t0: float, t1: float):
        """Summary of the samples stamped in [t0, t1] (host clock)."""
        import datetime
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        rows = []
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        lo, hi = t0 - self.PERIOD_S, t1 + self.PERIOD_S
        inside = [r for r in rows if lo <= r[0] <= hi]
        if not inside and rows:      # a window shorter than one period: the nearest samples
            inside = sorted(rows, key=lambda r: abs(r[0] - (t0 + t1) / 2))[:max(1, len(self.gpus))]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {n for r in inside for n, v in zip(names, r[3]) if v.lower() == "active"}
        sm = [r[1] for r in inside]
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max((r[2] for r in inside), default=None),
                "reasons": sorted(reasons), "samples": len(sm)}


def pct(vals, q):
    return float(np.percentile(np.asarray(vals), q)) if len(vals) else float("nan")


def serving_shape(args, world):
    tp = args.tp or (1 if world == 1 else 2)
    if world % tp:
        raise SystemExit(f"{world} GPUs do not split into TP={tp} instances")
    ninst = world // tp
    gs = args.group_size or (2 if ninst >= 2 else 1)
    if ninst % gs:
        raise SystemExit(f"{ninst} instances do not split into balloon groups of {gs}")
    return tp, gs, ninst // gs, ninst


def summarize(recs, t0, t1, slo_ttft, slo_tpot):
    """SLO accounting of one window [t0, t1] (host clock).  ``recs``:
    rid -> (arrival, token times, finished, output length).  Returns a dict:

    * ``equiv``: SLO goodput in request-equivalents: every token a request
      emitted inside the window counts 1/output-length of a request, when
      the request met the TTFT objective and its mean inter-token time up to
      the window's end meets the TPOT objective (a request that finishes
      inside the window within both objectives thus counts in full over its
      lifetime).  In steady state this equals the rate of requests finished
      within the objectives, with far less sampling noise over a short
      window, and it rises when steps get faster.
    * ``good`` / ``finished``: requests that finished inside the window
      within both objectives / at all;
    * ``ttft``: TTFT of requests whose first token came inside the window;
    * ``tpot``: running TPOT of requests with two or more tokens, emitting
      inside the window;
    * ``gaps``: inter-token gaps that ended inside the window."""
    good, finished, ttft, tpot, gaps, equiv = 0, 0, [], [], 0, 0.0
    for arrival, times, fin, out_len in recs.values():
        inside = [t for t in times if t <= t1]
        if not inside or inside[-1] < t0:
            continue
        first = inside[0]
        if first >= t0:
            ttft.append(first - arrival)
        gaps += sum(1 for x, y in zip(inside, inside[1:]) if y >= t0)
        per_tok = (inside[-1] - first) / (len(inside) - 1) if len(inside) > 1 else 0.0
        if len(inside) > 1:
            tpot.append(per_tok)
        ok = first - arrival <= slo_ttft and per_tok <= slo_tpot
        if ok:
            equiv += sum(1 for t in inside if t >= t0) / max(out_len, 1)
        if fin and len(inside) == len(times):
            finished += 1
            good += int(ok)
    return {"equiv": equiv, "good": good, "finished": finished, "ttft": ttft, "tpot": tpot, "gaps": gaps}


class Job:
    """The serving job as rank 0 sees it."""

    def __init__(self, args, world, groups, handles, mc, cfg, on_gpu=True):
        self.args, self.world, self.mc, self.cfg = args, world, mc, cfg
        self.on_gpu = on_gpu
        self.inst_groups, self.handles = groups, handles
        self.workers = [handles[r] for r in sorted(handles)]

    async def setup(self, pages):
        from kunserve_b200.control.group import GroupEngine
        from kunserve_b200.llm import AsyncLLM
        from kunserve_b200.runtime.streams import StreamRouter
        a = self.args
        self.router = StreamRouter(asyncio.get_running_loop())
        self.gcw = GcWatch()
        gc.callbacks.append(self.gcw)
        self.groups = [GroupEngine(gi, insts, a.balloon_mode, self.cfg.balloon_config.max_balloon_memory_ratio)
                       for gi, insts in enumerate(self.inst_groups)]
        for g in self.groups:
            await asyncio.gather(*[i.initialize(num_gpu_blocks=pages) for i in g.instances])
        for g in self.groups:
            if len(g.instances) > 1:
                await g.setup_peer_memory()
        self.instances = [i for g in self.groups for i in g.instances]
        for inst in self.instances:
            inst.set_vote_window(10)
        self.llm = AsyncLLM(self.cfg, self.mc, self.groups, self.router)
        from kunserve_b200.llm import tune_gc
        tune_gc()   # as AsyncLLM.create does
        # the bench polls load and the state machine ten times a second so a
        # balloon can start inside a window of a few hundred milliseconds
        self.llm.coordinator.load_interval = 0.05
        self.llm.coordinator.fsm_interval = 0.02

    # ------------------------------------------------------------ helpers
    async def call_all(self, name, *args):
        from kunserve_b200.runtime import aw
        return await asyncio.gather(*[aw(getattr(w, name).remote(*args)) for w in self.workers])

    async def gpu0_steps(self):
        """Forward passes GPU 0's worker has run."""
        from kunserve_b200.runtime import aw
        return (await aw(self.workers[0].counters.remote()))["steps"]

    def live(self):
        return [i for i in self.instances if i.state != "merged"]

    async def start_loops(self):
        for g in self.groups:
            g.start()

    async def stop_loops(self):
        for g in self.groups:
            g.terminate()
        for g in self.groups:
            for t in list(g.tasks.values()):
                try:
                    await asyncio.wait_for(t, 60)
                except asyncio.TimeoutError:
                    raise RuntimeError("an instance loop did not stop")
            g.tasks.clear()

    async def pause(self):
        for inst in self.live():
            inst.stopped = True
        for inst in self.live():
            await inst.stop_and_wait()

    def resume(self):
        for inst in self.live():
            inst.stopped = False

    def reset(self):
        for inst in self.instances:
            if inst.state != "merged":
                inst.reset()

    async def back_to_initial(self):
        """Every group unfused with all its layers, every instance empty."""
        from kunserve_b200.utils.misc import EngineState
        for g in self.groups:
            if g.state == EngineState.BALLOON:
                await g.trigger_restore()
            if g.state == EngineState.RESTORE:
                await g.trigger_init()
        await self.stop_loops()
        self.reset()
        for g in self.groups:
            assert g.state == EngineState.INITIAL, g.state

    # ------------------------------------------------------------ phases
    async def warmup(self, steps):
        """``steps`` forward passes on GPU 0 over a small request set."""
        from kunserve_b200.evaluation.trace import build_trace
        from kunserve_b200.request import Request, SamplingParams
        a = self.args
        for inst in self.instances:
            inst.output_callback = lambda outs: None
        warm = build_trace(1.0, 4.0 * len(self.instances), seed=a.seed + 7, lengths="uniform",
                           prompt_range=(200, 600), output_range=(4, 16), vocab=self.mc.get_vocab_size())
        for i, r in enumerate(warm):
            gi, ii = self.llm.coordinator.get_next_assign()
            self.groups[gi].add_request(ii, Request(time.time(), 10_000_000 + i, None, r.prompt,
                                                    SamplingParams(temperature=0.0, max_tokens=r.output_len,
                                                                   ignore_eos=True)))
        s0 = await self.gpu0_steps()
        await self.start_loops()
        t0 = time.time()
        while await self.gpu0_steps() - s0 < steps:
            self._check()
            if time.time() - t0 > 300:
                raise RuntimeError("warm-up made no progress")
            await asyncio.sleep(0.001)
        await self.stop_loops()
        self.reset()

    def _check(self):
        for g in self.groups:
            if g.failed is not None:
                raise RuntimeError(f"group {g.group_id} failed") from g.failed
            for t in g.tasks.values():
                if t.done() and t.exception() is not None:
                    raise t.exception()

    def _loaded(self):
        mb = self.args.max_batch
        for inst in self.live():
            cap = max(inst.get_capacity_units(), 1)
            if inst.get_used_gpu_blocks() / cap < 0.95 or inst.check_pending_num() < mb:
                return False
        return True

    async def measure(self, label, via_api):
        """Fill, warm, timed window, drain.  Returns this run's summary."""
        from kunserve_b200.runtime import aw
        from kunserve_b200.evaluation.trace import build_trace
        from kunserve_b200.request import Request, SamplingParams
        from kunserve_b200.utils.misc import EngineState
        a, N = self.args, self.world
        ninst = len(self.instances)
        trace = build_trace(600.0, a.rate * a.burst_factor * N, "gamma", a.cv, seed=a.seed, lengths="uniform",
                            prompt_range=tuple(a.prompt_range), output_range=tuple(a.output_range),
                            vocab=self.mc.get_vocab_size(), backlog=a.backlog * ninst)
        sp = lambda r: SamplingParams(temperature=0.0, max_tokens=r.output_len, ignore_eos=True)
        recs = {}          # rid -> [arrival, token times, finished, output length]
        tasks = []

        def on_out(outs):
            for o in outs:
                rec = recs.get(o.request_id)
                if rec is not None:
                    rec[1] = [t.new_token_time for t in o.outputs]
                    rec[2] = True

        if not via_api:
            for inst in self.instances:
                inst.output_callback = on_out
        else:
            for inst in self.instances:
                inst.output_callback = self.router

        async def api_one(i, r, arrival):
            res = await self.llm.generate(prompt_token_ids=r.prompt, sampling_params=sp(r), request_id=i,
                                          arrival_time=arrival)
            recs[i][1] = list(res["metrics"].token_times)
            recs[i][2] = True

        def submit(i, r, arrival):
            recs[i] = [arrival, [], False, r.output_len]
            if via_api:
                tasks.append(asyncio.create_task(api_one(i, r, arrival)))
            else:
                gi, ii = self.llm.coordinator.get_next_assign()
                self.groups[gi].add_request(ii, Request(arrival, i, None, r.prompt, sp(r)))

        # ---- fill: the queued burst
        clocks = ClockSampler(list(range(N)) if self.on_gpu else [])
        if self.on_gpu:
            clocks.start()
        t_fill = time.time()
        nb = a.backlog * ninst
        for i in range(nb):
            submit(i, trace[i], t_fill)
        await asyncio.sleep(0)
        s_fill = await self.gpu0_steps()
        await self.start_loops()
        while not self._loaded():
            self._check()
            if time.time() - t_fill > 120:
                state = [(inst.instance_id, inst.get_used_gpu_blocks(), inst.get_capacity_units(),
                          inst.check_pending_num(), len(inst.step_log)) for inst in self.live()]
                raise RuntimeError("the backlog did not load the instances (KV >= 95 % and a queue): "
                                   f"(instance, used, capacity, pending, steps) = {state}")
            await asyncio.sleep(0.001)
        # the W warm steps right before the window also time the
        # tensor-parallel collectives (CUDA events around them, on every GPU)
        await self.call_all("set_profile", True)
        s_w = await self.gpu0_steps()
        # polls of GPU 0's step count are RPCs through the front end's event
        # loop and worker 0's request queue: every few milliseconds, so that
        # they do not compete with the steps being measured
        while await self.gpu0_steps() - s_w < a.warmup:
            self._check()
            await asyncio.sleep(POLL_S)
        fill_steps = await self.gpu0_steps() - s_fill
        await self.pause()
        prof = await self.call_all("profile")
        await self.call_all("set_profile", False)
        coll = sum(p[0] for p in prof)
        tot = sum(p[1] for p in prof)
        coll_share = round(coll / tot, 4) if tot > 0 else None
        running0 = sum(len(s.running_queue) for inst in self.live() for s in inst.scheduler)
        pending0 = sum(inst.check_pending_num() for inst in self.live())
        kv_used0 = min(inst.get_used_gpu_blocks() / max(inst.get_capacity_units(), 1) for inst in self.live())
        preempt0 = sum(inst.get_num_preemption() for inst in self.live())
        c0 = await self.call_all("counters")
        ht0 = [dict(inst.host_time) for inst in self.instances]
        await self.call_all("mark", "w0")
        trans0 = [len(g.transitions) for g in self.groups]

        # ---- timed window
        # the loaded state's objects (requests, outputs, page tables) move to
        # the permanent generation: the window's collections scan only new
        # objects instead of pausing the event loop over the whole heap
        gc.collect()
        gc.freeze()
        gc0 = (self.gcw.total, self.gcw.count)
        t0 = time.time()
        await aw(self.workers[0].arm_mark.remote("w1", a.steps))
        self.llm.coordinator.enable_balloon = any(len(g.instances) > 1 for g in self.groups)
        self.llm.coordinator.start()
        self.resume()

        async def feed():
            for i in range(nb, len(trace)):
                delay = t0 + trace[i].arrival - time.time()
                if delay > 0:
                    await asyncio.sleep(delay)
                submit(i, trace[i], t0 + trace[i].arrival)
        feeder = asyncio.create_task(feed())
        c1_gpu0 = None
        while c1_gpu0 is None:
            self._check()
            await asyncio.sleep(POLL_S)
            c1_gpu0 = await aw(self.workers[0].armed_counters.remote())
        # GPU 0 marked the window's end inside its K-th step; the others mark
        # theirs behind whatever they have in flight now
        await asyncio.gather(*[aw(w.mark.remote("w1")) for w in self.workers[1:]])
        t1 = time.time()
        clock_info = clocks.stop(t0, t1) if self.on_gpu else None
        win_ms = max(await asyncio.gather(*[self._elapsed(w) for w in self.workers]))
        c1 = await self.call_all("counters")
        c1[0] = c1_gpu0
        ht = {k: round(sum(inst.host_time[k] - h[k] for inst, h in zip(self.instances, ht0)), 4)
              for k in ht0[0]}
        gc_win = (round(self.gcw.total - gc0[0], 4), self.gcw.count - gc0[1])
        host_profile = {"frontend_s": ht, "gc_s": gc_win[0], "gc_collections": gc_win[1],
                        "gpu0": {"steps": c1[0]["steps"] - c0[0]["steps"],
                                 "gpu_s": round((c1[0]["gpu_ms"] - c0[0]["gpu_ms"]) / 1000.0, 4),
                                 "step_call_s": round(c1[0]["step_s"] - c0[0]["step_s"], 4),
                                 "pack_s": round(c1[0]["pack_s"] - c0[0]["pack_s"], 4),
                                 **{k: round(c1[0].get(k, 0.0) - c0[0].get(k, 0.0), 4)
                                    for k in ("recv_s", "launch_s", "sync_s", "send_s")}}}
        # token times of the requests still in flight at the window's end
        for inst in self.live():
            for r in list(inst.unaccepted_queue) + [r for s in inst.scheduler for r in s.all_requests()]:
                rec = recs.get(r.request_id)
                if rec is not None and not rec[2]:
                    rec[1] = [o.new_token_time for o in r.outputs]
        preempt1 = sum(inst.get_num_preemption() for inst in self.live())
        in_window = [g.transitions[k:] for g, k in zip(self.groups, trans0)]

        # ---- the burst ends: queued requests are dropped; wait for restore
        feeder.cancel()
        for inst in self.live():
            dropped = list(inst.unaccepted_queue)
            inst.unaccepted_queue.clear()
            for s in inst.scheduler:
                dropped += list(s.unaccepted_queue) + list(s.long_unaccepted_queue)
                s.unaccepted_queue.clear()
                s.long_unaccepted_queue.clear()
            for r in dropped:
                if via_api:
                    self.router.abort(r.request_id)
        t_drain = time.time()
        while time.time() - t_drain < a.drain_timeout:
            self._check()
            if all(g.state == EngineState.INITIAL for g in self.groups) and not any(
                    s.all_requests() for inst in self.live() for s in inst.scheduler):
                break
            await asyncio.sleep(0.01)
        drain_s = time.time() - t_drain
        c2 = await self.call_all("counters")
        restore_dev = [(y["restore_bytes"] - x["restore_bytes"], y["restore_s"] - x["restore_s"])
                       for x, y in zip(c1, c2) if y["restore_bytes"] > x["restore_bytes"]]
        # inter-token gaps while the parameters were being restored, against the
        # fused pipeline's gaps in the second before the restore started
        spans = [(t - dt, t) for inst in self.instances for t, name, dt in inst.event_log
                 if name == "pmm_restore" and t >= t_drain]
        gaps_in, gaps_before = [], []
        for _, times, _, _ in recs.values():
            for x, y in zip(times, times[1:]):
                for r0, r1 in spans:
                    if r0 <= y <= r1:
                        gaps_in.append(y - x)
                    elif r0 - 1.0 <= y < r0:
                        gaps_before.append(y - x)
        self.llm.coordinator.stop()
        for t in tasks:
            t.cancel()
        restore = [x for inst in self.instances for x in inst.restore_log]
        for inst in self.instances:
            inst.restore_log.clear()
        transitions = [[(name, round(dt, 4)) for _, name, dt in g.transitions] for g in self.groups]
        for g in self.groups:
            g.transitions.clear()
        await self.back_to_initial()
        gc.unfreeze()

        win_s = win_ms / 1000.0
        t_end = t0 + (win_s if not via_api else (t1 - t0))
        sm = summarize({k: tuple(v) for k, v in recs.items()}, t0, t_end, a.ttft_slo, a.tpot_slo)
        span = win_s if not via_api else (t1 - t0)
        dsteps = [y["steps"] - x["steps"] for x, y in zip(c0, c1)]
        return {
            "label": label, "window_s": win_s, "host_window_s": t1 - t0, "good": sm["good"],
            "finished": sm["finished"], "value": sm["equiv"] / span, "finished_goodput": sm["good"] / span,
            "ttft": sm["ttft"], "tpot": sm["tpot"], "tpot_samples": sm["gaps"],
            "running_at_start": running0, "queued_at_start": pending0, "kv_used_at_start": round(kv_used0, 3),
            "fill_steps": fill_steps, "preemptions": preempt1 - preempt0,
            "launches": sum(y["launches"] - x["launches"] for x, y in zip(c0, c1)),
            "h2d_per_step": (sum(y["h2d"] - x["h2d"] for x, y in zip(c0, c1)) / max(1, sum(dsteps))),
            "d2h_per_step": (sum(y["d2h"] - x["d2h"] for x, y in zip(c0, c1)) / max(1, sum(dsteps))),
            "fwd_busy": max((y["gpu_ms"] - x["gpu_ms"]) / max(win_ms, 1e-6) for x, y in zip(c0, c1)),
            "transitions_in_window": [[n for _, n, _ in t] for t in in_window],
            "transitions": transitions, "drain_s": round(drain_s, 3),
            "restored_gb": round(sum(b for b, _ in restore) / 1e9, 3),
            "restore_gbps": round(sum(b for b, _ in restore) / 1e9 / max(sum(s for _, s in restore), 1e-9), 1)
            if restore else None,
            "restore_device": {"gb_per_gpu": round(np.mean([b for b, _ in restore_dev]) / 1e9, 3),
                               "gbps_per_gpu": round(np.mean([b / max(d, 1e-9) for b, d in restore_dev]) / 1e9, 1),
                               "tbt_p50_during_s": round(pct(gaps_in, 50), 4),
                               "tbt_p99_during_s": round(pct(gaps_in, 99), 4),
                               "tbt_p50_before_s": round(pct(gaps_before, 50), 4),
                               "tbt_p99_before_s": round(pct(gaps_before, 99), 4),
                               "gaps_during": len(gaps_in)} if restore_dev else None,
            "clocks": clock_info, "host_profile": host_profile, "tp_collective_share": coll_share,
        }

    async def _elapsed(self, w):
        from kunserve_b200.runtime import aw
        return await aw(w.mark_elapsed_ms.remote("w0", "w1"))


async def run(job, args, pages):
    await job.setup(pages)
    await job.warmup(args.warmup)
    native = await job.measure("native", via_api=False)
    e2e = None if args.no_e2e else await job.measure("native-e2e", via_api=True)
    base = None
    if not args.no_baseline:
        # same scheduler and balloon policy; only the kernels and the transport
        # (NCCL collectives and send/recv instead of fused kernels and P2P pulls) differ
        await job.call_all("set_library_mode", True)
        await job.warmup(args.warmup)
        base = await job.measure("library-baseline", via_api=False)
        await job.call_all("set_library_mode", False)
    return native, e2e, base


def make_configs(args, world):
    """Serving shape and configurations of the run (every process derives
    the same ones from the arguments)."""
    from kunserve_b200.config import CacheConfig, ModelConfig, SchedConfig
    from kunserve_b200.config.kunserve_config import KunServeConfig
    on_gpu = args.device == "cuda"
    tp, gs, ngroups, ninst = serving_shape(args, world)
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.tp, e.pp = ngroups, gs, tp, 1
    e.block_size, e.max_batch_size, e.max_batch_tokens = args.block_size, args.max_batch, args.budget
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, args.budget
    cfg.balloon_config.enable_balloon = gs > 1
    cfg.balloon_config.balloon_mode = args.balloon_mode
    cfg.bench_config.enable_restore = True
    cfg.bench_config.model = args.model
    mc = ModelConfig(args.model, dtype="bf16" if on_gpu else "fp32")
    cfg.bench_config.max_model_len = mc.get_max_model_len()
    cc = CacheConfig(block_size=args.block_size, kv_budget_bytes=int(args.kv_gb * 1e9))
    sc = SchedConfig(policy="mixed", enable_chunked_prefill=True, chunked_prefill_budget=args.budget,
                     max_batch_size=args.max_batch, max_tokens_per_batch=args.budget)
    return cfg, mc, cc, sc, (tp, gs, ngroups, ninst)


def frontend_main(args, world, ports, authkey, conn):
    """The front end of a multi-rank run, in its own process: connects to
    every rank's worker, runs the measurements and sends back the result
    line (or the error)."""
    import traceback
    from kunserve_b200.bootstrap import connect_launched_job
    handles = {}
    try:
        cfg, mc, cc, sc, shape = make_configs(args, world)
        groups, handles = connect_launched_job(cfg, mc, cc, sc, ports, authkey)
        from kunserve_b200.runtime import get
        bb = get(handles[0].block_bytes.remote(args.block_size), timeout=600)
        pages = int(args.kv_gb * 1e9) // bb
        job = Job(args, world, groups, handles, mc, cfg, on_gpu=args.device == "cuda")
        nat, e2e, base = asyncio.run(run(job, args, pages))
        errs = get([h.device_error.remote() for h in handles.values()], timeout=120)
        if any(errs):
            raise RuntimeError(f"device error flags after the run: {errs}")
        conn.send(("ok", result_line(args, world, *shape, nat, e2e, base)))
    except BaseException:  # noqa: BLE001 - reported by rank 0
        conn.send(("error", traceback.format_exc()))
    finally:
        for h in handles.values():
            h.kill()


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

    on_gpu = args.device == "cuda"
    if on_gpu:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        device, backend = f"cuda:{local}", "native"
    else:
        device, backend = "cpu", "torch"
    cfg, mc, cc, sc, shape = make_configs(args, world)
    tp, gs, ngroups, ninst = shape
    if world == 1:
        from kunserve_b200.bootstrap import instances_from_handles, rank_parallel_config
        from kunserve_b200.engine.worker import Worker
        from kunserve_b200.parallel.topology import Topology
        from kunserve_b200.runtime import LocalActor
        topo = Topology(1, ngroups, gs, 1, tp)
        w = Worker(0, mc, cc, rank_parallel_config(topo, 0), backend=backend, device=device, seed=args.seed)
        handles = {0: LocalActor(w)}
        groups = instances_from_handles(cfg, mc, cc, sc, topo, handles)
        pages = int(args.kv_gb * 1e9) // w.block_bytes(args.block_size)
        job = Job(args, world, groups, handles, mc, cfg, on_gpu=on_gpu)
        nat, e2e, base = asyncio.run(run(job, args, pages))
        if on_gpu:
            from kunserve_b200.ops import check_error
            check_error()
        print(json.dumps(result_line(args, world, tp, gs, ngroups, ninst, nat, e2e, base)), flush=True)
        return 0

    import multiprocessing as mp
    from datetime import timedelta
    from kunserve_b200.bootstrap import join_launched_job
    if on_gpu:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=180), device_id=dev)
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=180))
    lr = join_launched_job(cfg, mc, cc, rank, device, seed=args.seed, backend=backend)
    fe = parent = None
    if rank == 0:
        ctx = mp.get_context("spawn")
        parent, child = ctx.Pipe()
        fe = ctx.Process(target=frontend_main, args=(args, world, lr.ports, lr.authkey, child), daemon=True)
        fe.start()
        child.close()
    lr.serve()          # until the front end lets this rank go
    rc = 0
    if rank == 0:
        msg = parent.recv() if parent.poll(60) else ("error", "the front end exited without a result")
        fe.join(30)
        if msg[0] == "ok":
            print(json.dumps(msg[1]), flush=True)
        else:
            print(msg[1], file=sys.stderr, flush=True)
            rc = 1
    if on_gpu:
        torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    return rc


def weight_gb_per_gpu(model: str, tp: int) -> float:
    """bf16 weights of `model` held by one of `tp` tensor-parallel GPUs."""
    from kunserve_b200.config import ModelConfig
    a = ModelConfig(model, dtype="bf16").arch
    hd = a.head_dim or a.hidden_size // a.num_attention_heads
    H, F = a.hidden_size, a.intermediate_size
    layer = H * (a.num_attention_heads + 2 * a.num_key_value_heads) * hd + a.num_attention_heads * hd * H + 3 * H * F
    return 2.0 * (a.num_hidden_layers * layer + 2 * a.vocab_size * H) / tp / 1e9


def result_line(args, world, tp, gs, ngroups, ninst, nat, e2e, base):
    par = f"tp{tp}xdp{ninst}" + (f" (balloon groups of {gs} -> tp{tp}xpp{gs})" if gs > 1 else "")
    line = {
        "metric": METRIC, "value": round(nat["value"], 4), "unit": "req/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(nat["window_s"] * 1000.0 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": round(nat["value"] / base["value"], 4) if base and base["value"] > 0 else None,
        "dtype": "bf16" if args.device == "cuda" else "fp32",
        "data": (f"synthetic: {args.backlog} requests per instance queued at t=0 (a burst in progress), then "
                 f"Gamma(CV={args.cv}) arrivals at {args.rate}x{args.burst_factor} req/s per GPU; prompt lengths "
                 f"uniform in {args.prompt_range}, output lengths uniform in {args.output_range}; random-init "
                 "N(0,0.02) weights"),
        "config": {"model": args.model, "global_batch": args.max_batch * ninst, "seq_len": args.prompt_range[1] +
                   args.output_range[1], "parallelism": par, "tp": tp, "instances": ninst, "balloon_groups": ngroups
                   if gs > 1 else 0, "balloon_mode": args.balloon_mode, "kv_budget_gb_per_gpu": args.kv_gb,
                   "block_size": args.block_size, "chunked_prefill_budget": args.budget,
                   "slo": {"ttft_s": args.ttft_slo, "tpot_s": args.tpot_slo},
                   "l2": f"inputs larger than L2: every step streams the weights ({weight_gb_per_gpu(args.model, tp):.0f} "
                         f"GB per TP{tp} GPU) and the KV pages",
                   "policy": "mixed prefill+decode batches, recompute preemption"},
        "p99_ttft_s": round(pct(nat["ttft"], 99), 4), "p99_tpot_s": round(pct(nat["tpot"], 99), 5),
        "p50_ttft_s": round(pct(nat["ttft"], 50), 4), "p50_tpot_s": round(pct(nat["tpot"], 50), 5),
        "finished": nat["finished"], "good": nat["good"], "finished_goodput": round(nat["finished_goodput"], 4),
        "window_s": round(nat["window_s"], 4),
        "running_at_start": nat["running_at_start"], "queued_at_start": nat["queued_at_start"],
        "kv_used_at_start": nat["kv_used_at_start"], "fill_steps": nat["fill_steps"],
        "preemptions": nat["preemptions"], "tpot_samples": nat["tpot_samples"],
        "transitions_in_window": nat["transitions_in_window"], "transitions": nat["transitions"],
        "restored_gb": nat["restored_gb"], "restore_gbps": nat["restore_gbps"],
        "restore_device": nat["restore_device"], "drain_s": nat["drain_s"],
        "gpu_launches": int(nat["launches"]), "forward_busy_frac": round(nat["fwd_busy"], 3),
        "clocks": nat["clocks"], "host_profile": nat["host_profile"],
        # device-time share of the W warm steps before the window spent in
        # the tensor-parallel collective (fused push GEMM + reduce; NCCL
        # all-reduce in the baseline), all GPUs
        "tp_collective_share": nat["tp_collective_share"],
    }
    if base is not None:
        line["baseline"] = {"impl": "library baseline: ATen/cuBLAS GEMMs, NCCL all-reduce and NCCL KV/weight moves",
                            "value": round(base["value"], 4),
                            "finished_goodput": round(base["finished_goodput"], 4),
                            "ms_per_step": round(base["window_s"] * 1000.0 /
                                                                                  args.steps, 3),
                            "p99_ttft_s": round(pct(base["ttft"], 99), 4),
                            "p99_tpot_s": round(pct(base["tpot"], 99), 5), "finished": base["finished"],
                            "preemptions": base["preemptions"], "transitions_in_window":
                            base["transitions_in_window"], "restore_gbps": base["restore_gbps"],
                            "tp_collective_share": base["tp_collective_share"], "clocks": base["clocks"]}
    if e2e is not None:
        line["e2e"] = {"value": round(e2e["value"], 4), "unit": "req/s", "api": "AsyncLLM.generate",
                       "finished_goodput": round(e2e["finished_goodput"], 4),
                       "p99_ttft_s": round(pct(e2e["ttft"], 99), 4), "p99_tpot_s": round(pct(e2e["tpot"], 99), 5),
                       "h2d_bytes_per_step": int(e2e["h2d_per_step"]), "d2h_bytes_per_step": int(e2e["d2h_per_step"]),
                       "window_s": round(e2e["host_window_s"], 4), "finished": e2e["finished"],
                       "transitions": e2e.get("transitions")}
    return line


if __name__ == "__main__":
    sys.exit(main())
