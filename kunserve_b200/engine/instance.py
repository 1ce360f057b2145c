"""Instance engine: scheduling loop and balloon/restore of one DP instance.

Parity: ``kunserve/flash_backend.py`` ``FlashBackend`` (:93-2732).  One
instance owns ``pp x tp`` workers, one block manager and ``pp`` virtual
engines (VEs).  When its balloon group fuses, the leader instance adopts the
members' workers, block managers and VEs (``merge_engine``) and drives the
whole group as one pipeline; ``split_engine`` hands them back.

Differences by design:

* Instances live in the front-end process (asyncio); only workers are
  separate processes (or Ray actors).  Merging and splitting therefore move
  Python objects instead of serialised property bundles.
* The fused pipeline runs stages in layer order: for every static stage
  ``s``, instance 0's slice, then instance 1's, ...  (the reference walks
  instance-major, which is only layer-ordered when ``pp == 1``).
* A request that cannot grow because the pool is exhausted and has no other
  victim to preempt is itself recomputed (or aborted if it can never fit),
  so a step never runs a request whose page table is short.
* Extend pages packed into the base region before a restore are really
  copied (the reference only rewrote the table, ``flash_backend.py:1116-1125``).
"""
import asyncio
import time
from collections import deque
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

from ..config.kunserve_config import BalloonConfig, BenchConfig
from ..config.runtime import CacheConfig, ModelConfig, ParallelConfig, SchedConfig
from ..kv.block_manager import BlockManager, NoFreeBlocksError
from ..request import BatchedRequests, Request, RequestOutput
from ..runtime.actors import aw
from ..sched.admission import AdmissionMixin
from ..sched.scheduler import ColocatedScheduler
from ..utils.lifetime import LifetimeEventType, now_event
from ..utils.logger import init_logger
from ..utils.misc import Event, cdiv
from .step import StepInput

logger = init_logger(__name__)

SLEEP_IN_EACH_EVENT_LOOP = 0.0005
OOM_RATE = 95.0
VALLEY_RATE = 50.0


class LifetimeRecorder:
    def __init__(self):
        self.events = []

    def scheduled(self, r: Request):
        self.events.append(now_event(LifetimeEventType.SCHEDULED, r.request_id))

    def add(self, kind, rid):
        self.events.append(now_event(kind, rid))


class InstanceEngine(AdmissionMixin):
    def __init__(self, server_id: int, instance_id: int, model_config: ModelConfig,
                 parallel_config: ParallelConfig, cache_config: CacheConfig,
                 sched_config: SchedConfig, balloon_config: BalloonConfig, bench_config: BenchConfig,
                 workers: List[List[object]], tokenizer=None,
                 output_callback: Optional[Callable[[List[RequestOutput]], None]] = None,
                 record_lifetime: bool = False):
        self.server_id = server_id
        self.instance_id = instance_id
        self.model_config = model_config
        self.parallel_config = parallel_config
        self.cache_config = cache_config
        self.sched_config = sched_config
        self.balloon_config = balloon_config
        self.bench_config = bench_config
        self.block_size = cache_config.block_size
        self.pp_size = parallel_config.pipeline_parallel_size
        self.tp_size = parallel_config.tensor_parallel_size
        self.workers = workers                     # [instance*pp + stage][tp]
        self.tokenizer = tokenizer
        self.output_callback = output_callback
        self.lifetime = LifetimeRecorder() if record_lifetime else None

        self.block_managers: List[BlockManager] = []
        self.scheduler: List[ColocatedScheduler] = []
        self.scheduler_running: List[bool] = []
        self.unaccepted_queue: Deque[Request] = deque()
        self.num_instances = 1
        self.member_ids: List[int] = [instance_id]
        self.is_fusion_state = False
        self.stopped = False
        self.state = "initial"
        self.is_resharding: List[bool] = []
        self.is_restoring = False
        self.is_reclaiming_ex_blocks = False
        self.allocate_lock = asyncio.Lock()
        self.p2p_kv = False         # KV moves as in-kernel pulls over mapped peer memory
        # micro-batches per virtual-engine step in the fused pipeline
        # (KUNSERVE_PIPE_MICROBATCHES; 1: the reference's one batch per VE)
        import os
        self.pipe_microbatches = max(1, int(os.environ.get("KUNSERVE_PIPE_MICROBATCHES", "1")))
        # host seconds by phase (scheduling between steps, building step
        # inputs, waiting for the workers' forward), for profiling the loop
        self.host_time = {"schedule": 0.0, "build": 0.0, "forward": 0.0, "post": 0.0}
        self.num_gpu_blocks = 0
        self.block_size_in_bytes = 0
        self.step_counter = 0

        # metrics
        self.finished_tokens = 0
        self.finished_requests = 0
        self._last_tokens = 0
        self._last_requests = 0
        self.ttfts: List[float] = []
        self.tbts: List[float] = []
        self.set_vote_window(30)
        self.step_log: List[Tuple[float, int, int]] = []   # (seconds, tokens, requests)
        self.event_log: List[Tuple[float, str, float]] = []  # (time, event, seconds)
        self.restore_log: List[Tuple[float, float]] = []     # (bytes pulled by all workers, seconds)
        self._loop_task: Optional[asyncio.Task] = None
        # per VE scheduler: was its next batch prepared after its last step?

    def set_vote_window(self, n: int) -> None:
        """Samples of KV demand (one per load collection) behind the balloon
        and restore votes; the reference keeps 30."""
        self.sliding_window: Deque[float] = deque([0.0] * n, maxlen=n)
        self.rate_window: Deque[float] = deque([0.0] * n, maxlen=n)

    # ------------------------------------------------------------ set-up
    def _new_scheduler(self) -> ColocatedScheduler:
        s = ColocatedScheduler(self.sched_config, self.block_managers, self.block_size)
        s.is_fusion_state = self.is_fusion_state
        return s

    def _all_workers(self):
        return [w for stage in self.workers for w in stage]

    def _call_all(self, name: str, *args):
        return [getattr(w, name).remote(*args) for w in self._all_workers()]

    def _call_instance(self, inst: int, name: str, *args, **kwargs):
        out = []
        for stage in self.workers[inst * self.pp_size:(inst + 1) * self.pp_size]:
            for w in stage:
                out.append(getattr(w, name).remote(*args, **kwargs))
        return out

    async def initialize(self, num_gpu_blocks: Optional[int] = None, weights_path: str = "") -> None:
        w00 = self.workers[0][0]
        prof = await aw(w00._profile_num_available_blocks.remote(
            self.block_size, self.cache_config.gpu_memory_utilization,
            self.cache_config.cpu_swap_space, self.cache_config.kv_cache_ratio))
        n_gpu, n_cpu, bb = prof
        if self.bench_config.num_gpu_blocks is not None:
            n_gpu = self.bench_config.num_gpu_blocks
        if num_gpu_blocks is not None:
            n_gpu = num_gpu_blocks
        self.num_gpu_blocks, self.block_size_in_bytes = n_gpu, bb
        await asyncio.gather(*[aw(f) for f in self._call_all(
            "init_model", n_gpu, weights_path, self.sched_config.max_tokens_per_batch,
            self.sched_config.max_batch_size, n_cpu)])
        self.block_managers.append(BlockManager(n_gpu, n_cpu, self.block_size, rank=0,
                                                reserved_blocks_ratio=self.cache_config.reserved_blocks_ratio))
        self.scheduler = [self._new_scheduler() for _ in range(self.pp_size)]
        self.scheduler_running = [False] * self.pp_size
        self.is_resharding = [False] * self.pp_size
        logger.info(f"instance {self.instance_id}: {n_gpu} KV pages of {self.block_size} tokens")

    # ---------------------------------------------------------- event loop
    async def start_event_loop(self) -> None:
        tasks: Dict[int, asyncio.Task] = {}
        while True:
            n = len(self.scheduler)
            for ve in range(n):
                t = tasks.get(ve)
                if (t is None or t.done()) and not self.stopped:
                    if t is not None and t.exception() is not None:
                        raise t.exception()
                    tasks[ve] = asyncio.create_task(self._step(ve))
            for ve in [v for v in tasks if v >= n]:
                tasks.pop(ve)
            if self.stopped and all(t.done() for t in tasks.values()):
                for t in tasks.values():
                    if t.exception() is not None:
                        raise t.exception()
                tasks.clear()
                await asyncio.sleep(SLEEP_IN_EACH_EVENT_LOOP)
                if getattr(self, "_terminate", False):
                    return
                continue
            busy = any(s.running_queue.requests for s in self.scheduler)
            pending = [t for t in tasks.values() if not t.done()]
            if busy and pending:
                # wake when a VE step finishes (or after the idle interval, so
                # that a VE without work looks for new requests) instead of
                # spinning: a spinning loop holds the interpreter lock that the
                # actor reader threads need to hand back step results
                await asyncio.wait(pending, timeout=SLEEP_IN_EACH_EVENT_LOOP, return_when=asyncio.FIRST_COMPLETED)
            else:
                await asyncio.sleep(0 if busy else SLEEP_IN_EACH_EVENT_LOOP)

    def launch(self) -> asyncio.Task:
        self._loop_task = asyncio.create_task(self.start_event_loop())
        return self._loop_task

    def terminate(self) -> None:
        self._terminate = True
        self.stopped = True

    def reset(self) -> None:
        """Drop every request and its pages and clear the counters, so the
        instance can serve a fresh workload (the loop must not be running)."""
        for s in self.scheduler:
            for r in s.all_requests():
                self._free_blocks(r)
            s.unaccepted_queue.clear()
            s.long_unaccepted_queue.clear()
            s.waiting_queue.clear()
            s.swapped_queue.clear()
            s.running_queue.requests.clear()
            s.num_preemption = 0
        self.unaccepted_queue.clear()
        for bm in self.block_managers:
            assert not bm.block_table, "pages still held after reset"
        self._terminate = False
        self.stopped = False
        self.ttfts, self.tbts, self.step_log = [], [], []
        self.finished_tokens = self.finished_requests = 0
        self.set_vote_window(len(self.sliding_window))

    async def stop_and_wait(self) -> None:
        self.stopped = True
        while any(self.scheduler_running):
            # a short sleep, not a spin: the steps in flight finish only once
            # the actor reader threads get the interpreter lock back
            await asyncio.sleep(SLEEP_IN_EACH_EVENT_LOOP)
        self.release_finished()

    def release_finished(self) -> None:
        """Free the pages of requests that finished in the last step before a
        stop (the step's batch preparation, which normally frees them, is
        skipped once the engine is stopped), so a transition starts from
        exact page accounting."""
        for s in self.scheduler:
            for r in s.pop_finished_requests():
                self._free_blocks(r)

    def set_engine_stopped(self, stopped: bool) -> None:
        self.stopped = stopped

    # ------------------------------------------------------------- stepping
    def _chain(self, fusion_exec: bool, kv_rank: int) -> List[Tuple[int, int]]:
        """(instance, stage) in layer order for one batch."""
        if fusion_exec and self.num_instances > 1:
            return [(i, s) for s in range(self.pp_size) for i in range(self.num_instances)]
        return [(kv_rank, s) for s in range(self.pp_size)]

    def _build_step(self, requests: Sequence[Request], inst: int, stage_layers: int,
                    fusion_exec: bool) -> StepInput:
        bm = self.block_managers[inst]
        n = self.num_instances if fusion_exec else 1
        ls = stage_layers // n
        lstart = inst * ls if fusion_exec and n > 1 else 0
        sp = [r.sampling_params for r in requests]
        tables = bm.get_block_table(requests)
        for r, t in zip(requests, tables):
            if len(t) * self.block_size < r.context_len_after_step():
                raise AssertionError(
                    f"instance {self.instance_id} (state {self.state}, member {inst}): request {r.request_id} "
                    f"needs {r.context_len_after_step()} KV slots but holds {len(t)} pages ({r!r}, "
                    f"kind={bm._kind.get(r.request_id)})")
        return StepInput(
            request_ids=[r.request_id for r in requests],
            input_tokens=[r.get_input_tokens_ids() for r in requests],
            start_positions=[r.start_position() for r in requests],
            page_tables=tables,
            is_prefill=[int(r.is_context_stage()) for r in requests],
            layer_start=lstart, layer_end=lstart + ls,
            fusion_size=bm.fusion_size if fusion_exec else 1,
            temperature=[p.temperature if not p.is_greedy else 0.0 for p in sp],
            top_k=[p.top_k for p in sp], top_p=[p.top_p for p in sp],
            seeds=[(p.seed if p.seed is not None else r.request_id) for p, r in zip(sp, requests)],
            step_id=self.step_counter)

    async def _forward(self, requests: List[Request], fusion_exec: bool, kv_rank: int,
                       restore: Optional[tuple] = None) -> List[int]:
        tb = time.perf_counter()
        stage_layers = self.model_config.get_num_layers(self.parallel_config)
        chain = self._chain(fusion_exec, kv_rank)
        comm = "gp" if (fusion_exec and self.num_instances > 1) else "pp"
        steps = {inst: self._build_step(requests, inst, stage_layers, fusion_exec)
                 for inst in {c[0] for c in chain}}
        if restore is not None:
            home, n, tables, dp = restore
            for inst, st in steps.items():
                st.restore = (home, n, inst, tables, dp)
        self.step_counter += 1
        futs = []
        for k, (inst, stage) in enumerate(chain):
            def idx(c):
                i, s = c
                return i * self.pp_size + s if comm == "gp" else s
            recv_from = (comm, idx(chain[k - 1])) if k > 0 else None
            send_to = (comm, idx(chain[k + 1])) if k + 1 < len(chain) else None
            last = k + 1 == len(chain)
            for w in self.workers[inst * self.pp_size + stage]:
                futs.append((last, w.step.remote(steps[inst], recv_from, send_to, last)))
        tf = time.perf_counter()
        self.host_time["build"] += tf - tb
        result = None
        for last, f in futs:
            out = await aw(f)
            if last and result is None:
                result = out
        self.host_time["forward"] += time.perf_counter() - tf
        return result

    async def _step(self, ve: int) -> None:
        if self.stopped:
            return
        self.scheduler_running[ve] = True
        try:
            resharding: List[Request] = []
            if ve < len(self.is_resharding) and self.is_resharding[ve]:
                resharding = await self._live_reshard_prepare(ve)
            if not self.scheduler[ve].next_batch_prepared:
                # a transition stopped the previous step before it prepared
                # this VE's next batch (page growth, admission): do it now
                async with self.allocate_lock:
                    await self._get_next_batch(ve)
            self.scheduler[ve].next_batch_prepared = False
            batch, _ = self.scheduler[ve].schedule(prefill_only_chunk=True)
            batch.set_sched_time()
            pipe, replica = batch.get_fusion_requests()
            if pipe:
                k = self.pipe_microbatches
                if k > 1 and self.num_instances > 1 and len(pipe) >= 2 * k:
                    # several micro-batches of this VE in flight at once, so a
                    # stage computes the next one while the later stages work
                    # on this one (disjoint requests: no token depends on
                    # another micro-batch of the same step)
                    parts = [pipe[i::k] for i in range(k)]
                    await asyncio.gather(*[self._step_inner(ve, p, fusion_exec=True) for p in parts if p])
                else:
                    await self._step_inner(ve, pipe, fusion_exec=True)
            if resharding:
                await self._reshard_blocks_batched(resharding)
            if not self.is_fusion_state and replica:
                await self._step_inner(ve, replica, fusion_exec=False)
            if self.is_reclaiming_ex_blocks:
                await self.pack_blocks_into_base_region(pipe)
            async with self.allocate_lock:
                t0 = time.perf_counter()
                await self._get_next_batch(ve)
                self.host_time["schedule"] += time.perf_counter() - t0
        finally:
            self.scheduler_running[ve] = False

    async def _step_inner(self, ve: int, requests: List[Request], fusion_exec: bool) -> None:
        if self.stopped or not requests:
            return
        kv_rank = ve // self.pp_size
        # live restore: move up to exchange_batch_size pipeline requests home
        restore_reqs, restore_pages = [], []
        if self.state == "restore" and fusion_exec and self.num_instances > 1:
            home = self.block_managers[kv_rank]
            for r in requests:
                if r.is_context_stage():
                    continue
                k = len(home.get_single_block_table(r.request_id))
                pages = home.get_free_gpu_blocks(k)
                if not pages:
                    break
                restore_reqs.append(r)
                restore_pages.append(pages)
                if len(restore_reqs) >= self.balloon_config.exchange_batch_size:
                    break
        batch = BatchedRequests(requests)
        t0 = time.time()
        batch.start_one_iteration(t0)
        restore = None
        if restore_reqs:
            n = self.num_instances
            tables = [[p for r, dp in zip(restore_reqs, restore_pages)
                       for p in self.block_managers[i].get_single_block_table(r.request_id)[:len(dp)]]
                      for i in range(n)]
            restore = (kv_rank, n, tables, [p for dp in restore_pages for p in dp])
        tokens = await self._forward(requests, fusion_exec, kv_rank, restore)
        t1 = time.time()
        tp0 = time.perf_counter()
        if restore_reqs:
            self._finish_live_restore(kv_rank, restore_reqs, restore_pages)
        self.step_log.append((t1 - t0, batch.get_num_input_tokens(), len(requests)))
        texts = self._detok(tokens[:len(requests)])
        batch.finish_one_iteration(texts, tokens[:len(requests)], t1)
        outs = []
        for r in requests:
            if r.is_context_stage():
                continue
            self.finished_tokens += 1
            if len(r.outputs) == 1:
                self.ttfts.append(r.outputs[0].new_token_time - r.arrival_time)
                if self.lifetime:
                    self.lifetime.add(LifetimeEventType.FIRST_TOKEN, r.request_id)
            elif len(r.outputs) >= min(20, r.sampling_params.max_tokens):
                self.tbts.append((r.outputs[-1].new_token_time - r.outputs[0].new_token_time)
                                 / (len(r.outputs) - 1))
            if r.is_finished:
                self.finished_requests += 1
                if self.lifetime:
                    self.lifetime.add(LifetimeEventType.FINISHED, r.request_id)
                outs.append(RequestOutput(r.request_id, r.prompt_token_ids, r.outputs, r.start_time,
                                          r.server_info, True, arrival_time=r.arrival_time))
        if outs and self.output_callback is not None:
            self.output_callback(outs)
        self.host_time["post"] += time.perf_counter() - tp0

    def _detok(self, ids: Sequence[int]) -> List[str]:
        if self.tokenizer is None:
            return [""] * len(ids)
        out = []
        for i in ids:
            try:
                out.append(self.tokenizer.decode([i]))
            except Exception:  # noqa: BLE001 - unknown ids decode to empty text
                out.append("")
        return out

    async def _get_next_batch(self, ve: int) -> None:
        if self.stopped:
            return
        s = self.scheduler[ve]
        s.next_batch_prepared = True
        for r in s.pop_finished_requests():
            self._free_blocks(r)
        # 1. grow the running requests; preempt on shortage
        for r in list(s.running_queue.requests):
            if r not in s.running_queue.requests:
                continue
            while True:
                try:
                    self._allocate_blocks(r)
                    break
                except NoFreeBlocksError:
                    if self.sched_config.preempt_method == "swap" and not r.fusion_exec:
                        res = s.trigger_swap(r.kv_fusion_rank)
                        if res is not None:
                            await self._do_swap(res[1], False, r.kv_fusion_rank)
                            continue
                    victim = s.trigger_recompute(r.fusion_exec, r.kv_fusion_rank)
                    if victim is None or victim is r:
                        if victim is None:
                            self._preempt_self(s, r)
                        break
        # 2. waiting queue (KV ready) back into the batch
        while (r := s.fetch_waiting_queue()) is not None:
            if self.check_add(ve, r, is_waiting=True) == (0, 0, 0):
                s.swap_in_from_waiting_queue(r)
            else:
                break
        # 3. swapped queue
        if self.sched_config.preempt_method == "swap":
            while s.swapped_queue:
                r = s.swapped_queue[0]
                if self.check_add(ve, r)[1:] != (0, 0):
                    break
                res = s.swap_in_request()
                if res is None:
                    break
                await self._do_swap(res[1], True, r.kv_fusion_rank)
        # 4. queue-level migration to the least-loaded peer instance
        if ve == 0 and self.bench_config.enable_migration and self.peers:
            await self._maybe_migrate()
        # 5. admission
        if len(self.scheduler) > 1 and self.state != "restore":
            if self.bench_config.enable_look_ahead:
                self.balance_prefill(ve)
            if self.bench_config.enable_packing:
                self.schedule_packed_prefill(ve)
            else:
                self.schedule_prefill(ve)
        else:
            self.schedule_prefill(ve)

    def _preempt_self(self, s: ColocatedScheduler, r: Request) -> None:
        """No other victim: give ``r``'s pages back and requeue it, or abort it
        if it cannot fit even in an empty pool."""
        cap = min(bm.P * (bm.fusion_size if r.fusion_exec else 1) + bm.num_free_extend()
                  for bm in self._bms_for(r))
        if cdiv(r.get_num_tokens(), self.block_size) > cap:
            logger.warning(f"request {r.request_id} needs more KV than the pool holds; aborting it")
            s.running_queue.requests.remove(r)
            self._free_blocks(r)
            r.is_finished = True
            if self.output_callback is not None:
                self.output_callback([RequestOutput(r.request_id, r.prompt_token_ids, r.outputs,
                                                    r.start_time, r.server_info, True,
                                                    arrival_time=r.arrival_time)])
            return
        s.recompute_requests([r], in_running_queue=True)

    async def _do_swap(self, pairs, is_swap_in: bool, inst: int) -> None:
        await asyncio.gather(*[aw(f) for f in self._call_instance(inst, "swap_blocks", pairs, is_swap_in)])

    # --------------------------------------------------------------- intake
    def abort_request(self, request_ids) -> None:
        for rid in request_ids:
            for q in (self.unaccepted_queue,):
                for r in list(q):
                    if r.request_id == rid:
                        q.remove(r)
            for s in self.scheduler:
                s.abort_request(rid)

    peers: List["InstanceEngine"] = []

    async def _maybe_migrate(self) -> None:
        pending = sum(cdiv(r.get_num_tokens(), self.block_size) for r in self.unaccepted_queue)
        if pending < self.get_free_gpu_blocks():
            return
        local = self.get_used_gpu_blocks()
        loads = [(p.get_used_gpu_blocks(), p) for p in self.peers if p is not self and not p.stopped]
        if not loads:
            return
        min_load, dst = min(loads, key=lambda x: x[0])
        if min_load >= local:
            return
        budget = (local - min_load) // 2
        moved, used = [], 0
        for r in sorted(self.unaccepted_queue, key=lambda r: r.get_num_tokens()):
            b = cdiv(r.get_num_tokens(), self.block_size)
            if used + b > budget:
                break
            used += b
            moved.append(r)
        for r in moved:
            self.unaccepted_queue.remove(r)
        if moved:
            dst.add_requests(moved)
            logger.info(f"instance {self.instance_id}: migrated {len(moved)} queued requests "
                        f"to instance {dst.instance_id}")

    # ----------------------------------------------------------- accounting
    def get_unfinished_requests(self) -> int:
        return len(self.unaccepted_queue) + sum(
            len(s.running_queue) + len(s.waiting_queue) + len(s.swapped_queue) +
            len(s.unaccepted_queue) + len(s.long_unaccepted_queue) for s in self.scheduler)

    def get_used_gpu_blocks(self) -> int:
        tot = 0
        for s in self.scheduler:
            for r in list(s.waiting_queue) + list(s.swapped_queue) + s.running_queue.requests:
                tot += cdiv(r.get_num_tokens(), self.block_size)
        return tot

    def get_free_gpu_blocks(self) -> int:
        if self.is_fusion_state:
            return min(bm.get_num_avail_gpu_blocks() for bm in self.block_managers)
        return sum(bm.num_free_whole() for bm in self.block_managers)

    def get_gpu_blocks_usage(self):
        """(demand %, unfinished requests, -free pages, tokens this epoch,
        finished requests this epoch).  Also feeds the vote windows."""
        used = self.get_used_gpu_blocks()
        cap = max(self.get_capacity_units(), 1)
        demand = used / cap * 100.0
        self.sliding_window.append(demand)
        self.rate_window.append((demand - self.sliding_window[0]) / len(self.sliding_window))
        tok = self.finished_tokens - self._last_tokens
        req = self.finished_requests - self._last_requests
        self._last_tokens, self._last_requests = self.finished_tokens, self.finished_requests
        return demand, self.get_unfinished_requests(), -self.get_free_gpu_blocks(), tok, req

    def get_capacity_units(self) -> float:
        """Pages a request of the current state can use: whole pages when
        unfused; slices (+extend) of one member when fused."""
        if self.is_fusion_state:
            return min(bm.P * bm.fusion_size + bm.num_extend_gpu_blocks for bm in self.block_managers)
        return sum(bm.P for bm in self.block_managers)

    def get_num_fusion_requests(self) -> int:
        return sum(s.get_num_fusion_requests() for s in self.scheduler)

    def get_num_preemption(self) -> int:
        return sum(s.num_preemption for s in self.scheduler)

    def pop_metrics(self):
        t, b = self.ttfts, self.tbts
        self.ttfts, self.tbts = [], []
        return t, b

    # ------------------------------------------------------------------ votes
    def vote_for(self, event: Event) -> bool:
        if event == Event.BALLOON:
            pending = sum(cdiv(r.get_num_tokens(), self.block_size) for r in self.unaccepted_queue)
            for s in self.scheduler:
                pending += sum(cdiv(r.get_num_tokens(), self.block_size)
                               for r in list(s.unaccepted_queue) + list(s.long_unaccepted_queue))
            usage = self.sliding_window[-1]
            return usage >= OOM_RATE and pending >= self.get_free_gpu_blocks() and pending > 0
        if event == Event.RESTORE:
            if not self.bench_config.enable_restore or self.check_pending_num():
                return False
            return self.sliding_window[-1] <= VALLEY_RATE and sum(self.rate_window) < 0
        if event == Event.INIT:
            return self.get_num_fusion_requests() == 0
        return False

    # ------------------------------------------------------- merge / split
    def merge_engine(self, rank: int, other: "InstanceEngine") -> None:
        """Adopt a group member's workers, block manager and VEs."""
        assert rank == self.num_instances
        self.workers.extend(other.workers)
        bm = other.block_managers[0]
        bm.rank = rank
        self.block_managers.append(bm)
        for s in other.scheduler:
            for r in s.running_queue.requests + list(s.swapped_queue) + list(s.waiting_queue):
                r.kv_fusion_rank = rank
            s.block_managers = self.block_managers
            s.next_batch_prepared = False
            self.scheduler.append(s)
            self.scheduler_running.append(False)
            self.is_resharding.append(False)
        for s in self.scheduler:
            s.block_managers = self.block_managers
        self.unaccepted_queue.extend(other.unaccepted_queue)
        other.unaccepted_queue.clear()
        self.num_instances += 1
        self.member_ids.append(other.instance_id)
        other.workers, other.block_managers, other.scheduler = [], [], []
        other.scheduler_running, other.is_resharding = [], []
        other.stopped = True
        other.state = "merged"

    def split_engine(self, members: Sequence["InstanceEngine"]) -> None:
        """Give every member back its workers, block manager and VEs."""
        pp = self.pp_size
        for bm in self.block_managers:
            bm.restore_from_fusion()
        for k, other in enumerate(members, start=1):
            other.workers = self.workers[k * pp:(k + 1) * pp]
            bm = self.block_managers[k]
            bm.rank = 0
            other.block_managers = [bm]
            other.scheduler = self.scheduler[k * pp:(k + 1) * pp]
            for s in other.scheduler:
                s.block_managers = other.block_managers
                s.is_fusion_state = False
                s.next_batch_prepared = False
                for r in s.all_requests():
                    r.kv_fusion_rank = 0
                    r.fusion_exec = False
            other.scheduler_running = [False] * pp
            other.is_resharding = [False] * pp
            other.num_instances = 1
            other.member_ids = [other.instance_id]
            other.is_fusion_state = False
            other.state = "initial"
        self.workers = self.workers[:pp]
        self.block_managers = self.block_managers[:1]
        self.scheduler = self.scheduler[:pp]
        for s in self.scheduler:
            s.block_managers = self.block_managers
            s.is_fusion_state = False
            s.next_batch_prepared = False
            for r in s.all_requests():
                r.fusion_exec = False
                r.kv_fusion_rank = 0
        self.scheduler_running = [False] * pp
        self.is_resharding = [False] * pp
        self.num_instances = 1
        self.member_ids = [self.instance_id]

    def set_fusion_state(self, value: bool) -> None:
        self.is_fusion_state = value
        for s in self.scheduler:
            s.is_fusion_state = value

    # --------------------------------------------------------------- balloon
    async def trigger_balloon(self, balloon_mode: str, from_restore: bool,
                              members: Sequence["InstanceEngine"]) -> int:
        """Fuse this instance and ``members`` into one pipeline (leader side)."""
        t0 = time.perf_counter()
        await self.stop_and_wait()
        for m in members:
            await m.stop_and_wait()
        t_stop = time.perf_counter() - t0   # in-flight steps finishing
        if not from_restore:
            for k, m in enumerate(members, start=1):
                self.merge_engine(k, m)
        n = self.num_instances
        self.set_fusion_state(True)
        for bm in self.block_managers:
            bm.convert_to_pipeline_format(n)
        t_merge = time.perf_counter() - t0 - t_stop
        # drop parameters; their memory becomes extend pages
        drops = [self._call_instance(i, "pmm_drop", i, n) for i in range(n)]
        for i, futs in enumerate(drops):
            res = [await aw(f) for f in futs]
            self.block_managers[i].add_ex_fusion_blocks(min(res))
        t_drop = time.perf_counter() - t0 - t_stop - t_merge
        # stale (pre-balloon) requests
        self.is_resharding = [False] * len(self.scheduler)
        mode = self.balloon_config.effective_mode
        if mode == "recompute":
            for s in self.scheduler:
                s.trigger_recompute_for_stale_requests()
        elif mode == "reshard":
            stale: List[Request] = []
            for s in self.scheduler:
                stale.extend(s.trigger_reshard_for_stale_requests(live_reshard=False))
            await self.reshard_blocks(stale)
        elif mode == "livereshard":
            self.is_resharding = [True] * len(self.scheduler)
        t_kv = time.perf_counter() - t0 - t_stop - t_merge - t_drop
        for bm in self.block_managers:
            bm.convert_all_reserved_blocks_into_fusion()
        # even out VE loads, then admit again
        loads = [len(s.running_queue) for s in self.scheduler]
        hi, lo = loads.index(max(loads)), loads.index(min(loads))
        if hi != lo:
            k = (loads[hi] - loads[lo]) // 2
            moving = [r for r in self.scheduler[hi].running_queue.requests if r.fusion_exec][:k]
            for r in moving:
                self.scheduler[hi].running_queue.requests.remove(r)
                self.scheduler[lo].running_queue.requests.append(r)
        self.state = "balloon"
        self.stopped = False
        self.sched_config.enable_chunked_prefill = True
        async with self.allocate_lock:
            for ve in range(len(self.scheduler)):
                await self._get_next_batch(ve)
        dt = time.perf_counter() - t0
        self.event_log.append((time.time(), "balloon", dt))
        logger.info(f"instance {self.instance_id}: balloon with {n} instances in {dt:.3f}s "
                    f"(in-flight steps {t_stop:.3f}s, merge {t_merge:.3f}s, parameter drop {t_drop:.3f}s, "
                    f"stale KV {t_kv:.3f}s), free pages now {self.get_free_gpu_blocks()}")
        return self.get_free_gpu_blocks()

    def prepare_reshard_blocks(self, requests: Sequence[Request]) -> Tuple[List[Request], List[Request]]:
        """Allocate slices on every other member for each stale request."""
        ok, fail = [], []
        for r in requests:
            done = []
            try:
                for i, bm in enumerate(self.block_managers):
                    if i == r.kv_fusion_rank:
                        continue
                    bm.allocate_blocks(r, only_new_blocks=True)
                    done.append(bm)
                ok.append(r)
            except NoFreeBlocksError:
                for bm in done:
                    bm.free_request(r.request_id)
                fail.append(r)
        return ok, fail

    async def _reshard_blocks_batched(self, requests: Sequence[Request]) -> None:
        """Move each stale request's other layer slices to the members that
        run them (reference ``_reshard_blocks_batched``, ``kv_exchange``)."""
        n = self.num_instances
        by_home: List[List[Request]] = [[] for _ in range(n)]
        for r in sorted(requests, key=lambda r: r.request_id):
            by_home[r.kv_fusion_rank].append(r)
        if n > 1 and requests:
            t0 = time.perf_counter()
            futs = []
            for i in range(n):
                bm = self.block_managers[i]
                pages = []
                for j in range(n):
                    lst = []
                    for r in by_home[j]:
                        home_len = len(self.block_managers[j].get_single_block_table(r.request_id))
                        lst.extend(bm.get_single_block_table(r.request_id)[:home_len])
                    pages.append(lst)
                home = [[p for r in by_home[j] for p in self.block_managers[j].get_single_block_table(r.request_id)]
                        for j in range(n)]
                for st in range(self.pp_size):
                    for w in self.workers[i * self.pp_size + st]:
                        futs.append(w.kv_exchange.remote(pages, i, n, home))
            try:
                moved = await asyncio.gather(*[aw(f) for f in futs])
            except Exception:
                logger.error("kv_exchange failed on a worker; the group's exchange state is unknown")
                raise
            dt = time.perf_counter() - t0
            self.event_log.append((time.time(), "reshard", dt))
            logger.info(f"resharded {len(requests)} requests ({sum(moved) / 2**20:.1f} MiB) in {dt:.3f}s")
        for i in range(n):
            for r in by_home[i]:
                self.block_managers[i].free_blocks_into_fusion_except(r.request_id, n, i)
        for r in requests:
            r.fusion_exec = True
            r.once_fusion_exec = True
            r.kvcache_ready = True

    async def reshard_blocks(self, requests: Sequence[Request]) -> None:
        """Bulk reshard in batches of ``exchange_batch_size`` requests.  The
        requests keep their place in their VE's running queue; what cannot be
        placed on the other members is recomputed instead."""
        remaining = list(requests)
        # the NCCL exchange stages each batch in a scratch buffer, so batches
        # are bounded; the P2P pulls copy page to page and take all at once
        cap = (len(remaining) if self.p2p_kv else self.balloon_config.exchange_batch_size) or len(remaining) or 1
        while remaining:
            head, remaining = remaining[:cap], remaining[cap:]
            ok, fail = self.prepare_reshard_blocks(head)
            if ok:
                await self._reshard_blocks_batched(ok)
            if fail and not ok:
                for r in fail + remaining:
                    for s in self.scheduler:
                        if r in s.running_queue.requests:
                            s.running_queue.requests.remove(r)
                    self._free_blocks(r)
                    r.prepare_for_recompute()
                    r.fusion_exec = True
                    self.unaccepted_queue.appendleft(r)
                break
            remaining = fail + remaining

    async def _live_reshard_prepare(self, ve: int) -> List[Request]:
        s = self.scheduler[ve]
        stale = s.trigger_reshard_for_stale_requests(
            live_reshard=True, live_reshard_batch_size=self.balloon_config.exchange_batch_size)
        if not stale:
            self.is_resharding[ve] = False
            return []
        ok, fail = self.prepare_reshard_blocks(stale)
        s.running_queue.add_requests(fail)
        for r in ok:
            r.kvcache_ready = False
            s.waiting_queue.append(r)
        return ok

    # ---------------------------------------------------------------- restore
    async def pack_blocks_into_base_region(self, requests: Sequence[Request]) -> None:
        for i, bm in enumerate(self.block_managers):
            moves = bm.pack_blocks_into_base_region(requests)
            if moves:
                await asyncio.gather(*[aw(f) for f in self._call_instance(
                    i, "local_copy_blocks", moves, bm.fusion_size)])

    async def reclaim_extra_blocks(self, timeout_s: float = 600.0) -> None:
        """Stop using extend pages and wait until every one is back."""
        self.is_reclaiming_ex_blocks = True
        for bm in self.block_managers:
            bm.start_extend_reclaim()
        t0 = time.time()
        while not all(bm.extend_reclaimed() for bm in self.block_managers):
            if time.time() - t0 > timeout_s:
                raise TimeoutError("extend pages were not returned in time")
            await asyncio.sleep(0.001)
        self.is_reclaiming_ex_blocks = False

    async def pmm_restore(self) -> None:
        """Restore every member's dropped parameters (reference
        ``pmm_restore``, called before the engines stop,
        ``kunserve/llm_engine.py:546-570``): the pulls run on side streams
        while this instance's fused pipeline keeps serving, and this returns
        once every byte landed."""
        n = self.num_instances
        t0 = time.perf_counter()
        futs = []
        for i in range(n):
            futs.extend(self._call_instance(i, "pmm_restore_start", n, None, i))
        moved = await asyncio.gather(*[aw(f) for f in futs])
        while True:
            done = await asyncio.gather(*[aw(f) for i in range(n) for f in self._call_instance(i, "pmm_restore_done")])
            if all(done):
                break
            await asyncio.sleep(0.0005)
        await asyncio.gather(*[aw(f) for i in range(n) for f in self._call_instance(i, "pmm_restore_finish")])
        dt = time.perf_counter() - t0
        self.event_log.append((time.time(), "pmm_restore", dt))
        self.restore_log.append((float(sum(moved)), dt))
        logger.info(f"parameters restored ({sum(moved) / 2**30:.2f} GiB pulled) in {dt:.3f}s")

    def restore_instance(self) -> None:
        self.set_fusion_state(False)
        for bm in self.block_managers:
            bm.restore_kvblocks()
        self.state = "restore"
        self.stopped = False

    def _finish_live_restore(self, home: int, reqs: List[Request], pages: List[List[int]]) -> None:
        """Bookkeeping after a step that moved ``reqs`` home: their KV now
        lives in ``pages`` on the home instance (every member copied its
        layer slice inside the step)."""
        for r, dp in zip(reqs, pages):
            for bm in self.block_managers:
                if bm.is_allocated(r.request_id):
                    bm.free_request(r.request_id)
            self.block_managers[home].attach_blocks(r.request_id, dp)
            r.fusion_exec = False
            r.kv_fusion_rank = home

    # ------------------------------------------------- cross-group transfer
    def pop_transferable(self, max_pages: int) -> List[Tuple[Request, List[int]]]:
        """Running decode requests to hand to an instance of another group,
        latest first, up to ``max_pages`` pages: they leave this instance's
        running queues with their pages still allocated (the instance must be
        stopped and unfused)."""
        assert self.num_instances == 1 and not self.is_fusion_state
        bm = self.block_managers[0]
        out, used = [], 0
        for s in self.scheduler:
            for r in list(reversed(s.running_queue.requests)):
                if r.fusion_exec or r.is_context_stage() or r.is_finished or not bm.is_allocated(r.request_id):
                    continue
                pages = list(bm.get_single_block_table(r.request_id))
                if used + len(pages) > max_pages:
                    continue
                s.running_queue.requests.remove(r)
                out.append((r, pages))
                used += len(pages)
        return out

    def take_pages_for(self, items: Sequence[Tuple[Request, List[int]]]):
        """Free pages of this pool for transferred requests, in order, until
        one does not fit: ``[(request, source pages, destination pages)]``."""
        bm = self.block_managers[0]
        out = []
        for r, pages in items:
            got = bm.get_free_gpu_blocks(len(pages))
            if not got:
                break
            out.append((r, pages, got))
        return out

    def adopt_transferred(self, moved) -> None:
        """Requests whose KV now sits in this pool join the least loaded VE."""
        bm = self.block_managers[0]
        for r, _, dst in moved:
            bm.attach_blocks(r.request_id, dst)
            r.fusion_exec = False
            r.kv_fusion_rank = 0
            s = min(self.scheduler, key=lambda x: len(x.running_queue))
            s.running_queue.requests.append(r)
            s.next_batch_prepared = False

    def return_transferable(self, items) -> None:
        """Requests that did not move go back to a running queue here."""
        for r, _ in items:
            s = min(self.scheduler, key=lambda x: len(x.running_queue))
            s.running_queue.requests.append(r)
            s.next_batch_prepared = False

    def trigger_init(self) -> None:
        self.num_instances = 1
        self.state = "initial"
        self.stopped = False
