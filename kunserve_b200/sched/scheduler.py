"""Per-virtual-engine request queues and preemption.

Parity: ``kunserve/colocated_scheduler.py:18-538``.  One scheduler exists per
*virtual engine* (VE): a micro-batch slot of an instance.  An instance has
``pp`` VEs; when a balloon group fuses, the leader adopts every member's VEs
(``kv_rank = ve // pp`` is the member that owned it).

Queues: ``unaccepted`` (admitted to this VE, no KV yet), ``long_unaccepted``
(packed prefill's long requests), ``waiting`` (KV being moved, e.g. live
reshard), ``swapped`` (KV on the host) and ``running``.

Preemption victims are the newest decode-stage requests of the requested
kind (pipeline vs replica on a given rank), as in the reference.  Recompute
folds generated tokens into the prompt and puts the request back at the head
of ``unaccepted``.
"""
from collections import deque
from typing import Callable, Deque, List, Optional, Sequence, Tuple

from ..config.runtime import SchedConfig
from ..kv.block_manager import BlockManager
from ..request import BatchedRequests, Request
from ..utils.logger import init_logger
from ..utils.misc import cdiv

logger = init_logger(__name__)


class ColocatedScheduler:
    def __init__(self, sched_config: SchedConfig, block_managers: List[BlockManager],
                 block_size: int, on_release: Optional[Callable[[Sequence[Request]], None]] = None):
        self.sched_config = sched_config
        self.block_managers = block_managers      # shared list, owned by the instance
        self.block_size = block_size
        self.on_release = on_release
        self.unaccepted_queue: Deque[Request] = deque()
        self.long_unaccepted_queue: Deque[Request] = deque()
        self.waiting_queue: Deque[Request] = deque()
        self.swapped_queue: Deque[Request] = deque()
        self.running_queue = BatchedRequests([])
        self.num_pending_prefill_tokens = 0
        self.num_preemption = 0
        self.is_fusion_state = False
        # the owning instance grew this VE's running requests for the next
        # step (page growth, admission); travels with the VE across
        # merge/split so a new owner never trusts another's bookkeeping
        self.next_batch_prepared = False

    # ------------------------------------------------------------- queues
    def _blocks(self, n_tokens: int) -> int:
        return cdiv(n_tokens, self.block_size)

    def add_request(self, request: Request) -> None:
        n = request.get_input_len()
        request.output_capacity = self._blocks(n) * self.block_size - n
        self.unaccepted_queue.append(request)

    def abort_request(self, request_id: int) -> bool:
        for r in self.running_queue.requests:
            if r.request_id == request_id:
                r.is_finished = True      # released at the next batch boundary
                return True
        for q in (self.unaccepted_queue, self.long_unaccepted_queue, self.waiting_queue,
                  self.swapped_queue):
            for r in list(q):
                if r.request_id == request_id:
                    q.remove(r)
                    return True
        return False

    def all_requests(self) -> List[Request]:
        return (list(self.running_queue.requests) + list(self.waiting_queue) +
                list(self.swapped_queue) + list(self.unaccepted_queue) +
                list(self.long_unaccepted_queue))

    def get_num_fusion_requests(self) -> int:
        return sum(1 for r in self.all_requests() if r.fusion_exec and not r.is_finished)

    def get_num_unfinished_requests(self) -> int:
        return (len(self.unaccepted_queue) + len(self.long_unaccepted_queue) +
                len(self.swapped_queue) + len(self.running_queue) + len(self.waiting_queue))

    def get_num_decode_requests(self) -> int:
        return len(self.running_queue.get_decode_requests())

    def fetch_unaccepted_queue(self) -> Optional[Request]:
        return self.unaccepted_queue[0] if self.unaccepted_queue else None

    def pop_unaccepted_queue(self) -> Optional[Request]:
        return self.unaccepted_queue.popleft() if self.unaccepted_queue else None

    def fetch_waiting_queue(self) -> Optional[Request]:
        for r in self.waiting_queue:
            if r.kvcache_ready:
                return r
        return None

    def swap_in_from_waiting_queue(self, request: Request) -> None:
        self.waiting_queue.remove(request)
        self.running_queue.add_request(request)

    def fetch_swapped_queue(self) -> Optional[Request]:
        return self.swapped_queue[0] if self.swapped_queue else None

    def add_to_cur_batch(self, request: Request) -> None:
        self.running_queue.add_request(request)

    # ------------------------------------------------------------- schedule
    def schedule(self, prefill_only_chunk: bool = True) -> Tuple[BatchedRequests, bool]:
        """The next step's batch.  ``policy == "mixed"`` (or chunked prefill
        with ``prefill_only_chunk=False``) runs prefill chunks and decodes
        together; otherwise prefills run first and decodes wait."""
        prefills, decodes = self.running_queue.split_requests()
        prefills = [r for r in prefills if r.kvcache_ready and r.get_num_input_tokens() > 0]
        decodes = [r for r in decodes if r.kvcache_ready]
        mixed = self.sched_config.policy == "mixed" or (
            self.sched_config.enable_chunked_prefill and not prefill_only_chunk)
        if mixed:
            return BatchedRequests(prefills + decodes), bool(prefills)
        if prefills:
            return BatchedRequests(prefills), True
        return BatchedRequests(decodes), False

    def pop_finished_requests(self) -> List[Request]:
        return self.running_queue.pop_finished_requests()

    # ----------------------------------------------------------- preemption
    def _bms_of(self, request: Request) -> List[BlockManager]:
        if request.fusion_exec:
            return list(self.block_managers)
        return [self.block_managers[request.kv_fusion_rank]]

    def _release(self, request: Request) -> None:
        for bm in self._bms_of(request):
            if bm.is_allocated(request.request_id):
                bm.free_blocks(request)

    def get_latest_running_request(self, is_fusion: bool, rank: int = 0) -> Optional[Request]:
        for r in reversed(self.running_queue.requests):
            if r.is_migrating_out or r.is_resharding or r.is_context_stage():
                continue
            if is_fusion and r.fusion_exec:
                self.running_queue.requests.remove(r)
                return r
            if not is_fusion and not r.fusion_exec and r.kv_fusion_rank == rank:
                self.running_queue.requests.remove(r)
                return r
        return None

    def preempt_request(self, request: Request, in_running_queue: bool) -> None:
        if in_running_queue and request in self.running_queue.requests:
            self.running_queue.requests.remove(request)
        request.preempted_times += 1
        request.preempting = False
        self.num_preemption += 1

    def recompute_requests(self, requests: Sequence[Request], in_running_queue: bool = True,
                           abort: bool = False) -> bool:
        for r in requests:
            self.preempt_request(r, in_running_queue)
            self._release(r)
        if self.on_release is not None:
            self.on_release(requests)
        for r in requests:
            r.prepare_for_recompute()
            r.fusion_exec = self.is_fusion_state
        if not abort:
            for r in reversed(list(requests)):
                self.unaccepted_queue.appendleft(r)
        return True

    def trigger_recompute(self, is_fusion: bool, rank: int = 0, abort: bool = False) -> Optional[Request]:
        victim = self.get_latest_running_request(is_fusion, rank)
        if victim is None:
            return None
        self.recompute_requests([victim], in_running_queue=False, abort=abort)
        return victim

    def trigger_recompute_for_stale_requests(self) -> List[Request]:
        stale = [r for r in reversed(self.running_queue.requests) if not r.fusion_exec]
        for r in stale:
            r.once_fusion_exec = True
        self.recompute_requests(stale, in_running_queue=True)
        return stale

    def trigger_reshard_for_stale_requests(self, live_reshard: bool,
                                           live_reshard_batch_size: int = -1) -> List[Request]:
        """Stale (pre-balloon, replica) running requests to reshard now.  With
        ``live_reshard`` only up to ``live_reshard_batch_size`` leave the
        running queue per call; the rest keep their place."""
        valid, stale = self.running_queue.get_fusion_requests()
        if live_reshard:
            if live_reshard_batch_size > 0:
                valid.extend(stale[live_reshard_batch_size:])
                stale = stale[:live_reshard_batch_size]
            self.running_queue = BatchedRequests(valid)
        for r in stale:
            r.preempted_times += 1
            self.num_preemption += 1
        return stale

    def trigger_abort(self, budget_blocks: int = 1) -> List[Request]:
        aborted, freed = [], 0
        while freed < budget_blocks and self.running_queue.requests:
            r = self.running_queue.requests.pop(0)
            aborted.append(r)
            freed += self._blocks(r.get_num_tokens())
        self.recompute_requests(aborted, in_running_queue=False, abort=True)
        return aborted

    def try_get_victim_request(self, preempt_limit: int, is_fusion: Optional[bool] = None) -> Optional[Request]:
        def ok(r: Request) -> bool:
            if r.is_context_stage():
                return False
            if self.is_fusion_state:
                return r.fusion_exec
            return is_fusion is None or r.fusion_exec == is_fusion
        cands = sorted((r for r in self.running_queue.requests if ok(r)),
                       key=lambda r: r.arrival_time, reverse=True)
        for v in cands:
            if not v.preempting and (preempt_limit < 0 or v.preempted_times < preempt_limit):
                v.preempting = True
                return v
        return None

    # ----------------------------------------------------------------- swap
    def trigger_swap(self, rank: int = 0) -> Optional[Tuple[Request, list]]:
        """Swap the newest replica decode request of ``rank`` to host memory.
        Returns ``(victim, [(gpu_page, cpu_page)...])`` for the engine to copy."""
        victim = self.get_latest_running_request(False, rank)
        if victim is None:
            return None
        pairs = self.block_managers[rank].swap_out_requests([victim])
        if pairs is None:
            self.running_queue.requests.append(victim)
            return None
        self.swapped_queue.append(victim)
        self.preempt_request(victim, in_running_queue=False)
        return victim, pairs

    def swap_in_request(self) -> Optional[Tuple[Request, list]]:
        if not self.swapped_queue:
            return None
        r = self.swapped_queue[0]
        pairs = self.block_managers[r.kv_fusion_rank].swap_in_requests([r])
        if pairs is None:
            return None
        self.swapped_queue.popleft()
        self.running_queue.add_request(r)
        return r, pairs

    # ----------------------------------------------------------- accounting
    def get_total_gpu_blocks_needed(self) -> int:
        return sum(self._blocks(r.get_num_tokens()) for r in self.all_requests())

    def pop_running_requests_transfer(self, is_pp: bool, num_blocks_limit: int) -> List[Request]:
        total, out, keep = 0, [], []
        for r in self.running_queue.requests:
            b = self._blocks(r.get_num_tokens())
            if r.fusion_exec == is_pp and total + b <= num_blocks_limit:
                out.append(r)
                total += b
            else:
                keep.append(r)
        self.running_queue.requests = keep
        return out

    def __repr__(self) -> str:
        return (f"ColocatedScheduler(unaccepted={len(self.unaccepted_queue)}, "
                f"running={len(self.running_queue)}, waiting={len(self.waiting_queue)}, "
                f"swapped={len(self.swapped_queue)})")
