"""Front end: ``AsyncLLM``, the call a user makes.

Parity: ``kunserve/llm.py`` ``AsyncLLM`` (:41-400): ``create`` /
``from_engine_args``, ``initialize``, ``generate`` (returns ``{request_id,
prompt, prompt_len, outputs, metrics}``), ``batch_generate``, per-epoch
``report_server_metrics``, ``pop_metrics``, ``get_unfinished_num``,
``check_pending_num``, ``abort`` and ``terminate`` (which, unlike the
reference's no-op, stops every loop and worker).
"""
import asyncio
import gc
import itertools
import os
import time
from typing import Dict, List, Optional, Sequence

from .config.kunserve_config import KunServeConfig
from .config.runtime import CacheConfig, ModelConfig, SchedConfig
from .control.coordinator import Coordinator
from .control.group import GroupEngine
from .request import SamplingParams, create_request
from .runtime.streams import StreamRouter
from .utils.logger import init_logger
from .utils.metrics import calculate_metrics

logger = init_logger(__name__)


def runtime_configs(cfg: KunServeConfig, model_config: Optional[ModelConfig] = None):
    ec = cfg.engine_config
    mc = model_config or ModelConfig(cfg.bench_config.model or "tiny-llama", dtype=ec.dtype)
    cc = CacheConfig(block_size=ec.block_size, gpu_memory_utilization=ec.gpu_util)
    sc = SchedConfig(policy=ec.schedule_policy, preempt_method=ec.preempt_method,
                     max_batch_size=ec.max_batch_size, max_tokens_per_batch=ec.max_batch_tokens,
                     enable_chunked_prefill=ec.enable_chunked_prefill,
                     chunked_prefill_size=ec.chunked_prefill_size,
                     chunked_prefill_budget=ec.chunked_prefill_budget, use_tensor_cores=ec.use_tensor_cores)
    return mc, cc, sc


def tune_gc() -> None:
    """The front end's event loop drives every step: a full garbage
    collection over thousands of live requests pauses it (and the GPUs
    waiting for their next step) for up to seconds.  The objects built at
    start-up go to the permanent generation and full collections run ten
    times less often (the youngest generations, where per-step garbage
    dies, keep their defaults)."""
    gc.collect()
    gc.freeze()
    g0, g1, g2 = gc.get_threshold()
    gc.set_threshold(g0, g1, max(g2, 100))


class AsyncLLM:
    def __init__(self, cfg: KunServeConfig, model_config: ModelConfig, groups: List[GroupEngine],
                 router: StreamRouter, server_id: int = 0, tokenizer=None):
        self.cfg = cfg
        self.model_config = model_config
        self.groups = groups
        self.router = router
        self.server_id = server_id
        self.tokenizer = tokenizer
        self.coordinator = Coordinator(groups, cfg.dispatch_config.dispatch_strategy,
                                       cfg.balloon_config.enable_balloon,
                                       enable_transfer=cfg.balloon_config.enable_transfer,
                                       transfer_low=cfg.balloon_config.restore_memory_threshold)
        self._ids = itertools.count()
        self._tasks: List[asyncio.Task] = []
        self._epoch_t = time.time()
        self.started = False

    @classmethod
    async def create(cls, cfg: KunServeConfig, model_config: Optional[ModelConfig] = None, server_id: int = 0,
                     backend: str = "auto", actor_kind: str = "auto", devices=None, seed: int = 0,
                     num_gpu_blocks: Optional[int] = None, cache_config: Optional[CacheConfig] = None,
                     tokenizer=None, weights_path: str = "") -> "AsyncLLM":
        from .bootstrap import build_instances

        mc, cc, sc = runtime_configs(cfg, model_config)
        if cache_config is not None:
            cc = cache_config
        router = StreamRouter(asyncio.get_running_loop())
        inst_groups = await asyncio.get_running_loop().run_in_executor(
            None, lambda: build_instances(cfg, mc, cc, sc, server_id, backend, actor_kind, devices, seed,
                                          tokenizer, router))
        groups = [GroupEngine(gi, insts, cfg.balloon_config.effective_mode,
                              cfg.balloon_config.max_balloon_memory_ratio)
                  for gi, insts in enumerate(inst_groups)]
        for g in groups:
            await asyncio.gather(*[i.initialize(num_gpu_blocks=num_gpu_blocks, weights_path=weights_path)
                                   for i in g.instances])
            if os.environ.get("KUNSERVE_P2P", "1") != "0":
                await g.setup_peer_memory()
        llm = cls(cfg, mc, groups, router, server_id, tokenizer)
        if cfg.balloon_config.enable_transfer and os.environ.get("KUNSERVE_P2P", "1") != "0":
            await llm.coordinator.setup_global_peer_memory()
        tune_gc()
        llm.start()
        return llm

    from_engine_args = create

    def start(self) -> None:
        if self.started:
            return
        for g in self.groups:
            g.start()
            self._tasks.append(asyncio.create_task(g.monitor_engines()))
        self.coordinator.start()
        self.started = True

    async def initialize(self) -> None:
        self.start()

    def _check_alive(self) -> None:
        for g in self.groups:
            if g.failed is not None:
                raise RuntimeError(f"group {g.group_id} failed") from g.failed

    async def generate(self, prompt: Optional[str] = None, prompt_token_ids: Optional[List[int]] = None,
                       sampling_params: Optional[SamplingParams] = None, request_id: Optional[int] = None,
                       arrival_time: Optional[float] = None) -> Dict:
        self._check_alive()
        sp = sampling_params or SamplingParams()
        rid = next(self._ids) if request_id is None else request_id
        req = create_request(prompt, prompt_token_ids, sp, None, tokenizer=self.tokenizer,
                             max_model_len=self.cfg.bench_config.max_model_len,
                             arrival_time=arrival_time, request_id=rid)
        gi, ii = self.coordinator.get_next_assign()
        stream = self.router.register(rid)
        self.groups[gi].add_request(ii, req)
        final = None
        async for out in stream:
            final = out
        ids = [t.new_token_id for t in final.outputs] if final else []
        times = [t.new_token_time for t in final.outputs] if final else []
        text = self.tokenizer.decode(ids) if (self.tokenizer is not None and ids) else None
        return {"request_id": rid, "prompt": prompt, "prompt_len": len(req.prompt_token_ids), "outputs": ids,
                "text": text, "metrics": calculate_metrics(times, req.arrival_time, req.start_time, rid)}

    async def batch_generate(self, requests: Sequence[Dict]) -> List[Dict]:
        return await asyncio.gather(*[self.generate(**r) for r in requests])

    def abort(self, request_id: int) -> None:
        for g in self.groups:
            for inst in g.instances:
                inst.abort_request([request_id])
        self.router.abort(request_id)

    def get_unfinised_num(self) -> int:
        return sum(g.get_unfinished() for g in self.groups)

    get_unfinished_num = get_unfinised_num

    def check_pending_num(self) -> int:
        return sum(i.check_pending_num() for g in self.groups for i in g.instances if i.scheduler)

    def report_server_metrics(self) -> Dict:
        """One epoch of aggregate counters (throughput, demand, state)."""
        now = time.time()
        dt = max(now - self._epoch_t, 1e-6)
        self._epoch_t = now
        out = {"time": now, "tokens": 0, "finished": 0, "demand": [], "state": []}
        for g in self.groups:
            state, usages = g.get_gpu_blocks_usage()
            out["state"].append(state.name)
            for demand, _, _, tok, fin in usages:
                out["tokens"] += tok
                out["finished"] += fin
                out["demand"].append(demand)
        out["throughput_tok_s"] = out["tokens"] / dt
        return out

    def pop_metrics(self):
        ttft, tbt = [], []
        for g in self.groups:
            for i in g.instances:
                a, b = i.pop_metrics()
                ttft += a
                tbt += b
        return ttft, tbt

    async def terminate(self) -> None:
        self.coordinator.stop()
        for t in self._tasks:
            t.cancel()
        for g in self.groups:
            g.terminate()
        for g in self.groups:
            for t in g.tasks.values():
                try:
                    await asyncio.wait_for(t, 10)
                except (asyncio.TimeoutError, asyncio.CancelledError):
                    pass
        for g in self.groups:
            for inst in g.instances:
                for stage in inst.workers:
                    for w in stage:
                        w.kill()
