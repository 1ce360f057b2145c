"""The balloon cycle on two CPU instances (gloo worker processes):
INITIAL -> BALLOON (drop parameters, fuse into PP=2, reshard live KV) ->
RESTORE (pull parameters back from the peer, live-restore pipeline KV) ->
INITIAL, with every generated token checked against an unfused reference."""
import asyncio

import pytest

from kunserve_b200.config import KunServeConfig, ModelConfig, ParallelConfig
from kunserve_b200.models.weights import LlamaWeights
from kunserve_b200.request import SamplingParams
from kunserve_b200.utils.misc import EngineState

from helpers import hf_from_weights, hf_greedy, make_requests

pytestmark = pytest.mark.slow


def _cfg(mode):
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.pp, e.tp, e.block_size = 1, 2, 1, 1, 16
    e.dtype = "fp32"
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 96
    cfg.balloon_config.enable_balloon = False      # transitions are driven by the test
    cfg.balloon_config.balloon_mode = mode
    cfg.balloon_config.exchange_batch_size = 4
    cfg.bench_config.enable_restore = True
    return cfg


def _gen(llm, r):
    sp = SamplingParams(temperature=0.0, max_tokens=r.sampling_params.max_tokens, ignore_eos=True)
    return asyncio.create_task(llm.generate(prompt_token_ids=r.prompt_token_ids, sampling_params=sp,
                                            request_id=r.request_id))


async def _run(mode):
    from kunserve_b200.llm import AsyncLLM
    cfg = _cfg(mode)
    mc = ModelConfig("tiny-llama", dtype="fp32")
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="torch", actor_kind="process",
                                devices=["cpu", "cpu"], num_gpu_blocks=64, seed=0)
    group = llm.groups[0]
    loop = asyncio.get_running_loop()
    try:
        reqs = make_requests(12, seed=21, plen=(20, 60), olen=(30, 45))
        tasks = [_gen(llm, r) for r in reqs]
        leader = group.leader
        t0 = loop.time()
        while sum(len(s.running_queue.get_decode_requests()) for i in group.instances for s in i.scheduler) < 6:
            assert loop.time() - t0 < 120
            await asyncio.sleep(0.01)
        await group.trigger_balloon()
        assert group.state == EngineState.BALLOON
        assert leader.num_instances == 2 and leader.is_fusion_state
        assert all(bm.num_extend_gpu_blocks > 0 for bm in leader.block_managers)
        for bm in leader.block_managers:
            bm.check_invariants()
        # a second wave arrives while fused: these become pipeline requests
        more = make_requests(6, seed=22, plen=(20, 50), olen=(10, 20))
        for r in more:
            r.request_id += 100
        tasks += [_gen(llm, r) for r in more]
        await asyncio.sleep(1.0)
        await group.trigger_restore()
        assert group.state == EngineState.RESTORE and not leader.is_fusion_state
        for bm in leader.block_managers:
            bm.check_invariants()
        t0 = loop.time()
        while leader.get_num_fusion_requests() and loop.time() - t0 < 120:
            await asyncio.sleep(0.05)
        assert leader.get_num_fusion_requests() == 0
        await group.trigger_init()
        assert group.state == EngineState.INITIAL and leader.num_instances == 1
        try:
            results = await asyncio.wait_for(asyncio.gather(*tasks), 300)
        except asyncio.TimeoutError:
            # name where every unfinished request sits, so a stall is debuggable
            where = []
            for inst in group.instances:
                where.append(f"instance {inst.instance_id} state={inst.state} stopped={inst.stopped} "
                             f"unaccepted={[r.request_id for r in inst.unaccepted_queue]}")
                for k, s in enumerate(inst.scheduler):
                    where.append(f"  ve{k} running={[r.request_id for r in s.running_queue.requests]} "
                                 f"waiting={[r.request_id for r in s.waiting_queue]} "
                                 f"swapped={[r.request_id for r in s.swapped_queue]} "
                                 f"unaccepted={[r.request_id for r in s.unaccepted_queue]} "
                                 f"long={[r.request_id for r in s.long_unaccepted_queue]}")
            raise AssertionError("requests did not finish after the balloon cycle:\n" + "\n".join(where))
        for inst in group.instances:
            for bm in inst.block_managers:
                bm.check_invariants()
                assert not bm.block_table
        return mc, reqs + more, results
    finally:
        await llm.terminate()


@pytest.mark.parametrize("mode", ["reshard", "livereshard", "recompute"])
def test_balloon_cycle_is_token_exact(mode):
    mc, reqs, results = asyncio.run(_run(mode))
    w = LlamaWeights.random(mc, ParallelConfig(), seed=0)
    hf = hf_from_weights(mc, w)
    by_id = {r["request_id"]: r for r in results}
    for r in reqs:
        got = by_id[r.request_id]["outputs"]
        assert got == hf_greedy(hf, r.prompt_token_ids, r.sampling_params.max_tokens), r.request_id
