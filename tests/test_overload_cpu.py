"""Automatic overload handling on CPU, as the benchmark configuration's
config 1 specifies: tiny Llama (2 layers, hidden 256, 4 heads, 2 KV heads,
FFN 688, vocab 32000), two instances on gloo worker processes, 16-token KV
blocks and a 64-block budget per instance, 200 seeded Poisson requests at
4 req/s with prompts uniform in [16, 128] and outputs uniform in [8, 64].

Nothing triggers a transition by hand: the coordinator's votes must drive
INITIAL -> BALLOON -> RESTORE -> INITIAL.  The trace is replayed 20x faster
than its timestamps so that a fast CPU still overloads 64 blocks (the order
and the relative spacing of arrivals are the trace's).  Block accounting is
checked after every transition, and every request's tokens must equal an
unfused greedy run of the same weights.

Also unit tests of the votes (reference ``flash_backend.py:611-672``): the
balloon vote needs demand >= 95 % and pending >= free pages; the restore
vote needs no pending request, demand <= 50 % and a falling trend; the init
vote needs no pipeline request left."""
import asyncio

import pytest

from kunserve_b200.config import BalloonConfig, BenchConfig, CacheConfig, KunServeConfig, ModelConfig, \
    ParallelConfig, SchedConfig
from kunserve_b200.engine.instance import InstanceEngine
from kunserve_b200.evaluation.trace import build_trace
from kunserve_b200.request import Request, SamplingParams
from kunserve_b200.utils.misc import EngineState, Event

SPEEDUP = 20.0


def _trace():
    return build_trace(1000.0, 4.0, "poisson", seed=1, lengths="uniform", prompt_range=(16, 128),
                       output_range=(8, 64), vocab=32000)[:200]


def _cfg():
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.pp, e.tp, e.block_size = 1, 2, 1, 1, 16
    e.dtype = "fp32"
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 256
    cfg.balloon_config.enable_balloon = True
    cfg.balloon_config.balloon_mode = "reshard"
    cfg.bench_config.enable_restore = True
    return cfg


async def _serve(trace, overloaded: bool):
    from kunserve_b200.llm import AsyncLLM
    cfg = _cfg()
    if not overloaded:
        cfg.engine_config.group_size = 1
        cfg.balloon_config.enable_balloon = False
    mc = ModelConfig("tiny-llama", dtype="fp32")
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="torch",
                                actor_kind="process" if overloaded else "local",
                                devices=["cpu", "cpu"] if overloaded else ["cpu"],
                                num_gpu_blocks=64 if overloaded else 4096, seed=0)
    group = llm.groups[0]
    co = llm.coordinator
    co.load_interval, co.fsm_interval = 0.05, 0.02
    for inst in group.instances:
        inst.set_vote_window(10)
    checked = []

    # check block accounting right after every transition the state machine makes
    orig = group.handle_event

    async def handle_and_check(event):
        await orig(event)
        for inst in group.instances:
            for bm in inst.block_managers:
                bm.check_invariants()
        checked.append(group.state)

    group.handle_event = handle_and_check
    loop = asyncio.get_running_loop()
    try:
        t0 = loop.time()
        tasks = []
        for i, r in enumerate(trace):
            delay = t0 + r.arrival / SPEEDUP - loop.time()
            if delay > 0:
                await asyncio.sleep(delay)
            sp = SamplingParams(temperature=0.0, max_tokens=r.output_len, ignore_eos=True)
            tasks.append(asyncio.create_task(llm.generate(prompt_token_ids=r.prompt, sampling_params=sp,
                                                          request_id=i)))
        results = await asyncio.wait_for(asyncio.gather(*tasks), 600)
        # the burst is over: wait for the state machine to restore and split
        t1 = loop.time()
        while overloaded and group.state != EngineState.INITIAL and loop.time() - t1 < 120:
            await asyncio.sleep(0.05)
        names = [name for _, name, _ in group.transitions]
        for inst in group.instances:
            for bm in inst.block_managers:
                bm.check_invariants()
        return {r["request_id"]: r["outputs"] for r in results}, names, checked
    finally:
        await llm.terminate()


@pytest.fixture
def few_threads(monkeypatch):
    """Two worker processes and the front end share the CPU: two threads
    each (more only oversubscribes the cores and slows every step)."""
    import torch
    monkeypatch.setenv("OMP_NUM_THREADS", "2")
    n = torch.get_num_threads()
    torch.set_num_threads(2)
    yield
    torch.set_num_threads(n)


@pytest.mark.slow
def test_config1_votes_drive_a_full_balloon_cycle_token_exact(few_threads):
    trace = _trace()
    assert len(trace) == 200
    got, names, checked = asyncio.run(_serve(trace, overloaded=True))
    want, _, _ = asyncio.run(_serve(trace, overloaded=False))
    assert "INITIAL->BALLOON" in names, names
    i = names.index("INITIAL->BALLOON")
    assert names[i:i + 3] == ["INITIAL->BALLOON", "BALLOON->RESTORE", "RESTORE->INITIAL"], names
    assert len(checked) == len(names)
    assert set(got) == set(range(200))
    bad = [k for k in range(200) if got[k] != want[k]]
    assert not bad, f"{len(bad)} requests differ from the unfused run, e.g. {bad[:5]}"


# ----------------------------------------------------------------- votes
def _instance():
    mc = ModelConfig("tiny-llama", dtype="fp32")
    pc = ParallelConfig()
    cc = CacheConfig(block_size=16)
    sc = SchedConfig()
    bench = BenchConfig()
    bench.enable_restore = True
    inst = InstanceEngine(0, 0, mc, pc, cc, sc, BalloonConfig(), bench, [[None]])
    from kunserve_b200.kv.block_manager import BlockManager
    inst.block_managers.append(BlockManager(100, 0, 16))
    inst.scheduler = [inst._new_scheduler()]
    inst.set_vote_window(4)
    return inst


def _queue(inst, n, tokens=32):
    for i in range(n):
        inst.unaccepted_queue.append(Request(0.0, 1000 + i, None, list(range(tokens)),
                                             SamplingParams(max_tokens=4)))


def test_balloon_vote_needs_high_demand_and_pending_over_free():
    inst = _instance()
    inst.sliding_window.append(96.0)
    assert not inst.vote_for(Event.BALLOON)            # nothing pending
    _queue(inst, 10)                                   # 20 pages pending < 100 free
    assert not inst.vote_for(Event.BALLOON)
    _queue(inst, 45)                                   # 110 pages pending >= 100 free
    assert inst.vote_for(Event.BALLOON)
    inst.sliding_window.append(90.0)                   # demand below 95 %
    assert not inst.vote_for(Event.BALLOON)


def test_restore_vote_needs_no_pending_low_demand_and_falling_trend():
    inst = _instance()
    for d in (90.0, 90.0, 90.0, 90.0, 80.0, 70.0, 60.0, 40.0):
        inst.sliding_window.append(d)
        inst.rate_window.append((d - inst.sliding_window[0]) / len(inst.sliding_window))
    assert inst.vote_for(Event.RESTORE)
    _queue(inst, 1)
    assert not inst.vote_for(Event.RESTORE)            # a pending request blocks it
    inst.unaccepted_queue.clear()
    inst.sliding_window.append(55.0)                   # demand above 50 %
    assert not inst.vote_for(Event.RESTORE)
    inst.sliding_window.append(45.0)
    inst.rate_window.extend([5.0] * 4)                 # rising
    assert not inst.vote_for(Event.RESTORE)
    inst.bench_config.enable_restore = False
    inst.rate_window.extend([-5.0] * 4)
    assert not inst.vote_for(Event.RESTORE)


def test_init_vote_waits_for_pipeline_requests():
    inst = _instance()
    assert inst.vote_for(Event.INIT)
    r = Request(0.0, 1, None, list(range(8)), SamplingParams(max_tokens=4))
    r.fusion_exec = True
    inst.scheduler[0].running_queue.requests.append(r)
    assert not inst.vote_for(Event.INIT)
