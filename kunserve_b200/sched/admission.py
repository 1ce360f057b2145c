"""Admission of new requests into a virtual engine's running batch.

Parity with ``kunserve/flash_backend.py``:

* ``check_add`` ≙ ``_check_add_to_cur_batch`` (:1441-1492): overflow in KV
  pages, batch size and token budget.  A request admitted while the instance
  is fused becomes a pipeline request.
* ``schedule_prefill`` ≙ :1870-1950 — Sarathi-style chunked prefill: fill the
  step's token budget, chunking the request that does not fit.
* ``balance_prefill`` ≙ :1543-1868 — look-ahead stage 1: route the global
  queue longest-first to the VE with the fewest queued prefill tokens; with
  packing, long prompts (``> long_threshold * budget``) go to a separate queue.
* ``schedule_packed_prefill`` ≙ :1952-2137 — stage 2: at most one long prompt
  per step, chunked to the mean short-prompt length, then shorts.
* ``balance_decode`` ≙ :1495-1541 — decode rebalancing between VEs; only
  valid when VEs share KV (fused state), which is enforced here.

This is a mixin: the instance engine provides ``scheduler``,
``block_managers``, ``unaccepted_queue``, ``sched_config``, ``bench_config``,
``is_fusion_state`` and ``pp_size``.
"""
from collections import deque
from typing import Optional, Tuple

from ..kv.block_manager import NoFreeBlocksError
from ..request import Request
from ..utils.logger import init_logger
from ..utils.misc import cdiv

logger = init_logger(__name__)


class AdmissionMixin:
    # ------------------------------------------------------------ helpers
    def _blocks(self, n_tokens: int) -> int:
        return cdiv(n_tokens, self.block_size)

    def _bms_for(self, request: Request):
        if request.fusion_exec:
            return list(self.block_managers)
        return [self.block_managers[request.kv_fusion_rank]]

    def _allocate_blocks(self, request: Request) -> None:
        """All-or-nothing across every block manager the request needs."""
        if not request.fusion_exec:
            # most steps a request's pages already cover its next token
            bm = self.block_managers[request.kv_fusion_rank]
            table = bm.block_table.get(request.request_id)
            if table is not None and len(table) * bm.block_size >= request.get_num_tokens():
                return
        done = []
        try:
            for bm in self._bms_for(request):
                new = bm.allocate_blocks(request)
                done.append((bm, new))
        except NoFreeBlocksError:
            for bm, new in done:
                self._rollback(bm, request, new)
            raise

    @staticmethod
    def _rollback(bm, request: Request, new_ids) -> None:
        if not new_ids:
            return
        table = bm.block_table[request.request_id]
        if len(table) == len(new_ids):
            bm.free_request(request.request_id)
            return
        del table[len(table) - len(new_ids):]
        for f in new_ids:
            if bm._kind[request.request_id] == "whole":
                bm._release_whole(f)
            else:
                bm._release_id(f)

    def _free_blocks(self, request: Request) -> None:
        for bm in self._bms_for(request):
            if bm.is_allocated(request.request_id):
                bm.free_blocks(request)

    def free_blocks_batched(self, requests) -> None:
        for r in requests:
            self._free_blocks(r)

    def get_min_cost_scheduler(self):
        costs = [s.get_num_unfinished_requests() for s in self.scheduler]
        return self.scheduler[costs.index(min(costs))]

    def add_request(self, request: Request) -> None:
        n = request.get_input_len()
        request.output_capacity = self._blocks(n) * self.block_size - n
        if self.bench_config.enable_look_ahead:
            self.unaccepted_queue.append(request)
        else:
            self.get_min_cost_scheduler().unaccepted_queue.append(request)

    def add_requests(self, requests) -> None:
        for r in requests:
            n = r.get_input_len()
            r.output_capacity = self._blocks(n) * self.block_size - n
        self.unaccepted_queue.extend(requests)

    def check_pending_num(self) -> int:
        return len(self.unaccepted_queue) + sum(
            len(s.unaccepted_queue) + len(s.long_unaccepted_queue) for s in self.scheduler)

    def _fetch_unaccepted(self, ve: int, use_global: bool = True):
        s = self.scheduler[ve]
        if s.unaccepted_queue:
            return s.unaccepted_queue[0]
        if use_global and self.unaccepted_queue:
            return self.unaccepted_queue[0]
        return None

    def _pop_unaccepted(self, ve: int, request: Request, is_long: bool = False) -> None:
        s = self.scheduler[ve]
        for q in ((s.long_unaccepted_queue,) if is_long else (s.unaccepted_queue, self.unaccepted_queue)):
            if q and q[0] is request:
                q.popleft()
                return
        raise AssertionError("request is not at a queue head")

    def _free_units(self, request: Request, kv_rank: int) -> int:
        if self.is_fusion_state:
            return min(bm.get_num_avail_gpu_blocks() for bm in self.block_managers)
        return self.block_managers[kv_rank].num_free_whole()

    # ---------------------------------------------------------- admission
    def check_add(self, ve: int, request: Request, is_waiting: bool = False,
                  batch_tokens: Optional[int] = None) -> Tuple[int, int, int]:
        """(overflow pages, overflow requests, overflow tokens) if ``request``
        joined VE ``ve`` now; all zero means it fits.  ``batch_tokens``: the
        input tokens of VE ``ve``'s running batch, when the caller keeps that
        sum (chunked or mixed batching only)."""
        kv_rank = ve // self.pp_size
        if not is_waiting:
            request.fusion_exec = self.is_fusion_state
            request.kv_fusion_rank = kv_rank
        need = self._blocks(request.get_num_tokens())
        over_blocks = 0 if is_waiting else max(0, need - self._free_units(request, kv_rank))
        s = self.scheduler[ve]
        mixed = self.sched_config.policy == "mixed"
        whole_batch = not (request.is_context_stage() and not self.sched_config.enable_chunked_prefill and not mixed)
        cur = s.running_queue.requests if whole_batch else s.running_queue.get_context_requests()
        over_reqs = max(0, len(cur) + 1 - self.sched_config.max_batch_size)
        limit = (self.sched_config.chunked_prefill_budget if self.sched_config.enable_chunked_prefill
                 else self.sched_config.max_tokens_per_batch)
        if whole_batch and batch_tokens is not None:
            used = batch_tokens
        else:
            used = sum(r.get_num_input_tokens() for r in cur)
        over_tokens = max(0, used + request.get_num_input_tokens() - limit)
        return over_blocks, over_reqs, over_tokens

    _check_add_to_cur_batch = check_add

    def _admit(self, ve: int, request: Request, is_long: bool = False) -> bool:
        try:
            self._allocate_blocks(request)
        except NoFreeBlocksError:
            return False
        self._pop_unaccepted(ve, request, is_long)
        self.scheduler[ve].add_to_cur_batch(request)
        if self.lifetime is not None:
            self.lifetime.scheduled(request)
        return True

    def _advance_chunks(self, ve: int) -> int:
        """Give every partly-prefilled request its next chunk; returns the
        remaining token budget."""
        batch = self.scheduler[ve].running_queue
        budget = self.sched_config.chunked_prefill_budget
        used = sum(r.get_num_input_tokens() for r in batch.requests if not r.have_follow_up_chunk())
        free = budget - used
        for r in batch.requests:
            if r.have_follow_up_chunk():
                free = r.set_chunk(max(free, 1)) if free > 0 else r.set_chunk(1)
        return free

    def schedule_prefill(self, ve: int, use_global: bool = True) -> bool:
        """Admit FCFS until pages, batch size or the token budget run out.
        Returns True if admission stopped on KV pages (queueing)."""
        if self.sched_config.enable_chunked_prefill:
            self._advance_chunks(ve)
        # the running batch's input tokens, kept up to date as requests join
        # (chunked or mixed batching: every running request counts)
        keep = self.sched_config.enable_chunked_prefill or self.sched_config.policy == "mixed"
        batch = self.scheduler[ve].running_queue.requests
        used = sum(q.get_num_input_tokens() for q in batch) if keep else None
        while (r := self._fetch_unaccepted(ve, use_global)) is not None:
            ob, oreq, otok = self.check_add(ve, r, batch_tokens=used)
            if (ob, oreq, otok) == (0, 0, 0):
                if not self._admit(ve, r):
                    return True
                if keep:
                    used += r.get_num_input_tokens()
            elif self.sched_config.enable_chunked_prefill and ob == 0 and oreq == 0:
                avail = r.get_num_input_tokens() - otok
                if avail <= 0:
                    break
                r.set_chunk(avail)
                if not self._admit(ve, r):
                    return True
                if keep:
                    used += r.get_num_input_tokens()
                if r.have_follow_up_chunk():
                    break
            else:
                self._update_pending(ve)
                return ob > 0
        self._update_pending(ve)
        return False

    def _update_pending(self, ve: int) -> None:
        s = self.scheduler[ve]
        s.num_pending_prefill_tokens = (sum(r.get_num_tokens() for r in s.unaccepted_queue) +
                                        s.running_queue.get_unfinished_prefill_tokens())

    def balance_prefill(self, ve: int) -> None:
        bc = self.bench_config
        long_thr = self.sched_config.chunked_prefill_budget * bc.long_threshold
        pending = sorted(self.unaccepted_queue, key=lambda r: r.get_input_len(), reverse=True)
        self.unaccepted_queue.clear()
        if bc.enable_decode_balance:
            self.balance_decode(ve)
        if not pending:
            return
        load = [s.num_pending_prefill_tokens + s.running_queue.get_num_input_tokens()
                for s in self.scheduler]
        was_empty = all(not s.unaccepted_queue for s in self.scheduler)
        for r in pending:
            i = load.index(min(load))
            load[i] += r.get_input_len()
            if bc.enable_packing and r.get_input_len() > long_thr:
                self.scheduler[i].long_unaccepted_queue.append(r)
            else:
                self.scheduler[i].unaccepted_queue.append(r)
        for s in self.scheduler:
            key = (lambda r: r.get_input_len()) if (bc.enable_reorder and was_empty) else (lambda r: r.arrival_time)
            s.unaccepted_queue = deque(sorted(s.unaccepted_queue, key=key))

    def balance_decode(self, ve: int) -> None:
        if not self.is_fusion_state:
            return   # moving a replica request between VEs would strand its KV
        decodes = [s.running_queue.get_decode_requests() for s in self.scheduler]
        loads = [len(d) for d in decodes]
        hi, lo = loads.index(max(loads)), loads.index(min(loads))
        if hi != ve or hi == lo:
            return
        k = (loads[hi] - loads[lo]) // 2
        move = decodes[hi][:k]
        s = self.scheduler[hi]
        s.running_queue.requests = [r for r in s.running_queue.requests if r not in move]
        self.scheduler[lo].running_queue.requests.extend(move)

    def schedule_packed_prefill(self, ve: int, use_global: bool = True) -> bool:
        s = self.scheduler[ve]
        budget = self.sched_config.chunked_prefill_budget
        long_thr = budget * self.bench_config.long_threshold
        shorts = [r.get_num_input_tokens() for r in s.running_queue.get_context_requests() + list(s.unaccepted_queue)
                  if r.get_num_input_tokens() <= long_thr]
        mean_short = sum(shorts) // len(shorts) if shorts else int(long_thr)
        free = self._advance_chunks(ve) if self.sched_config.enable_chunked_prefill else budget
        overflow = False
        if s.long_unaccepted_queue:
            r = s.long_unaccepted_queue[0]
            ob, oreq, _ = self.check_add(ve, r)
            if ob == 0 and oreq == 0:
                n = min(free, max(mean_short, 1))
                if n > 0:
                    r.set_chunk(n)
                    self._admit(ve, r, is_long=True)
            elif ob:
                overflow = True
        return self.schedule_prefill(ve, use_global) or overflow
