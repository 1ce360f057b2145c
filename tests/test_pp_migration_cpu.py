"""Static pipeline parallelism and intra-group queue migration, served
through the public API on CPU worker processes (gloo).

* ``pp=2`` instances (reference ``--pp``, ``flash_backend.py:313-331``):
  each stage holds half of the layers, activations move over the ``pp``
  communicator and the instance runs two virtual engines; every request's
  greedy tokens must equal the unsplit model's (a PyTorch reference).
* ``enable_migration`` (reference ``flash_backend.py:2299-2339``): when an
  instance's queue holds more pages than it has free, VE 0 moves its
  shortest queued requests to the least loaded member of its group; the
  moved requests finish there with the same tokens.
"""
import asyncio

import pytest

from kunserve_b200.config import KunServeConfig, ModelConfig, ParallelConfig
from kunserve_b200.models.weights import LlamaWeights
from kunserve_b200.request import SamplingParams

from helpers import hf_from_weights, hf_greedy, make_requests

pytestmark = pytest.mark.slow


def _gen(llm, r):
    sp = SamplingParams(temperature=0.0, max_tokens=r.sampling_params.max_tokens, ignore_eos=True)
    return asyncio.create_task(llm.generate(prompt_token_ids=r.prompt_token_ids, sampling_params=sp,
                                            request_id=r.request_id))


def _reference(mc, reqs):
    w = LlamaWeights.random(mc, ParallelConfig(), seed=0)
    hf = hf_from_weights(mc, w)
    return {r.request_id: hf_greedy(hf, r.prompt_token_ids, r.sampling_params.max_tokens) for r in reqs}


async def _serve(cfg, reqs, devices, num_pages, check=None):
    from kunserve_b200.llm import AsyncLLM
    mc = ModelConfig("tiny-llama", dtype="fp32")
    llm = await AsyncLLM.create(cfg, model_config=mc, backend="torch", actor_kind="process", devices=devices,
                                num_gpu_blocks=num_pages, seed=0)
    try:
        tasks = [_gen(llm, r) for r in reqs]
        results = await asyncio.wait_for(asyncio.gather(*tasks), 300)
        extra = check(llm) if check else None
        for g in llm.groups:
            for inst in g.instances:
                for bm in inst.block_managers:
                    bm.check_invariants()
        return mc, {r["request_id"]: r["outputs"] for r in results}, extra
    finally:
        await llm.terminate()


def test_static_pipeline_two_stages_token_exact(monkeypatch):
    monkeypatch.setenv("OMP_NUM_THREADS", "2")
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.pp, e.tp, e.block_size = 1, 1, 2, 1, 16
    e.dtype = "fp32"
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 64
    reqs = make_requests(10, seed=31, plen=(10, 50), olen=(5, 20))

    def shape(llm):
        inst = llm.groups[0].instances[0]
        return inst.pp_size, len(inst.scheduler), len(inst.workers)

    mc, got, (pp, ves, stages) = asyncio.run(_serve(cfg, reqs, ["cpu", "cpu"], 64, shape))
    assert (pp, ves, stages) == (2, 2, 2)
    want = _reference(mc, reqs)
    assert got == want


def test_queue_migration_moves_requests_to_the_idle_member(monkeypatch):
    monkeypatch.setenv("OMP_NUM_THREADS", "2")
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.pp, e.tp, e.block_size = 1, 2, 1, 1, 16
    e.dtype = "fp32"
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 64
    cfg.bench_config.enable_migration = True
    # migration moves requests of the instance-wide queue, which requests
    # enter with look-ahead scheduling (as in the reference)
    cfg.bench_config.enable_look_ahead = True
    # every request goes to instance 0 (dispatch by memory load sees two
    # idle instances and picks the first); its 12-page pool overflows
    cfg.dispatch_config.dispatch_strategy = "memory"
    reqs = make_requests(12, seed=33, plen=(30, 60), olen=(10, 16))

    def where(llm):
        g = llm.groups[0]
        return [inst.finished_requests for inst in g.instances]

    import kunserve_b200.control.coordinator as co
    monkeypatch.setattr(co.Coordinator, "get_next_assign", lambda self: (0, 0))
    mc, got, finished = asyncio.run(_serve(cfg, reqs, ["cpu", "cpu"], 12, where))
    assert finished[1] > 0, f"nothing migrated: {finished}"
    want = _reference(mc, reqs)
    assert got == want


def test_cross_group_transfer_moves_running_requests(monkeypatch):
    """Two balloon groups of one instance each: requests all land on
    instance 0; the coordinator moves running requests with their KV pages
    to instance 1 (pairs of send/recv_blocks on the ``global`` communicator
    on CPU ranks; over NVLink pulls on GPUs), and they finish there with the
    same tokens."""
    monkeypatch.setenv("OMP_NUM_THREADS", "2")
    cfg = KunServeConfig()
    e = cfg.engine_config
    e.ngroups, e.group_size, e.pp, e.tp, e.block_size = 2, 1, 1, 1, 16
    e.dtype = "fp32"
    e.enable_chunked_prefill, e.chunked_prefill_budget = True, 128
    reqs = make_requests(10, seed=35, plen=(20, 50), olen=(24, 32))
    import kunserve_b200.control.coordinator as co
    monkeypatch.setattr(co.Coordinator, "get_next_assign", lambda self: (0, 0))

    async def run():
        from kunserve_b200.llm import AsyncLLM
        mc = ModelConfig("tiny-llama", dtype="fp32")
        llm = await AsyncLLM.create(cfg, model_config=mc, backend="torch", actor_kind="process",
                                    devices=["cpu", "cpu"], num_gpu_blocks=64, seed=0)
        try:
            tasks = [_gen(llm, r) for r in reqs]
            src, dst = llm.groups[0].instances[0], llm.groups[1].instances[0]
            loop = asyncio.get_running_loop()
            t0 = loop.time()
            while sum(len(s.running_queue.get_decode_requests()) for s in src.scheduler) < 6:
                assert loop.time() - t0 < 120
                await asyncio.sleep(0.01)
            moved = await llm.coordinator.transfer_requests(src, dst, 20)
            results = await asyncio.wait_for(asyncio.gather(*tasks), 300)
            for inst in (src, dst):
                for bm in inst.block_managers:
                    bm.check_invariants()
                    assert not bm.block_table
            return mc, {r["request_id"]: r["outputs"] for r in results}, moved, dst.finished_requests
        finally:
            await llm.terminate()

    mc, got, moved, dst_done = asyncio.run(run())
    assert 0 < moved <= 20 and dst_done > 0
    assert got == _reference(mc, reqs)
