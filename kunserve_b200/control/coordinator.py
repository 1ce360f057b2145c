"""Server-level coordinator: request dispatch, load collection and the
balloon state-machine driver.

Parity: ``kunserve/coordinator.py:21-330``.  Dispatch is round-robin over
``group x instance`` or least-load (``memory``/``load``) from the last
collected usage; load is collected every 0.5 s and the state machine polled
every 0.1 s (the reference's intervals).  A dispatch never targets a member
that is merged into its group leader: it goes to the leader.
"""
import asyncio
from typing import List, Optional, Tuple

from ..utils.logger import init_logger
from ..utils.misc import EngineState
from .group import GroupEngine

logger = init_logger(__name__)

LOAD_INTERVAL_S = 0.5
FSM_INTERVAL_S = 0.1


class Coordinator:
    def __init__(self, groups: List[GroupEngine], strategy: str = "round-robin", enable_balloon: bool = False,
                 load_interval: float = LOAD_INTERVAL_S, fsm_interval: float = FSM_INTERVAL_S,
                 enable_transfer: bool = False, transfer_high: float = 0.95, transfer_low: float = 0.5):
        self.groups = groups
        # cross-group transfer of running requests (reference
        # ``coordinator.py:39-147``): from an unfused instance whose KV demand
        # is at least transfer_high to one of another group below transfer_low
        self.enable_transfer = enable_transfer
        self.transfer_high, self.transfer_low = transfer_high, transfer_low
        self.global_p2p = False
        self.transfers: List[Tuple[int, int, int, float]] = []   # (src, dst, pages, seconds)
        self.load_interval = load_interval
        self.fsm_interval = fsm_interval
        self.strategy = strategy
        self.enable_balloon = enable_balloon
        self._rr = 0
        self.loads: List[List[float]] = [[0.0] * len(g.instances) for g in groups]
        self._tasks: List[asyncio.Task] = []

    def _targets(self) -> List[Tuple[int, int]]:
        out = []
        for gi, g in enumerate(self.groups):
            for ii, inst in enumerate(g.instances):
                out.append((gi, ii))
        return out

    def get_next_assign(self) -> Tuple[int, int]:
        targets = self._targets()
        if self.strategy == "round-robin":
            t = targets[self._rr % len(targets)]
            self._rr += 1
            return t
        best, best_load = targets[0], None
        for gi, ii in targets:
            load = self.loads[gi][ii] if ii < len(self.loads[gi]) else 0.0
            if best_load is None or load < best_load:
                best, best_load = (gi, ii), load
        return best

    def collect_instance_loads(self) -> None:
        for gi, g in enumerate(self.groups):
            state, usages = g.get_gpu_blocks_usage()
            if state == EngineState.INITIAL:
                self.loads[gi] = [u[0] for u in usages]
            else:
                # a fused group shares one pool: every member sees the leader's load
                self.loads[gi] = [usages[0][0]] * len(g.instances)

    async def collect_loop(self) -> None:
        while True:
            self.collect_instance_loads()
            await asyncio.sleep(self.load_interval)

    async def monitor_engine_events(self) -> None:
        while True:
            for g in self.groups:
                if g.state == EngineState.STOP:
                    continue
                _, event = await g.get_event()
                if event is not None:
                    await g.handle_event(event)
            if self.enable_transfer:
                await self.balance_groups()
            await asyncio.sleep(self.fsm_interval)

    # ------------------------------------------------- cross-group transfer
    def _unfused_instances(self):
        out = []
        for gi, g in enumerate(self.groups):
            if g.state != EngineState.INITIAL:
                continue
            for inst in g.instances:
                if inst.state == "initial" and inst.num_instances == 1 and inst.scheduler:
                    out.append((gi, inst))
        return out

    async def setup_global_peer_memory(self) -> bool:
        """Map every instance's KV pool into every instance of the server
        (same pipeline stage and TP rank), so cross-group page transfers
        pull over NVLink; False when the workers have no native engine."""
        from ..runtime.actors import aw
        insts = [inst for g in self.groups for inst in g.instances]
        if len(insts) < 2:
            return False
        pp, tp = insts[0].pp_size, insts[0].tp_size
        for st in range(pp):
            for t in range(tp):
                ws = [inst.workers[st][t] for inst in insts]
                infos = [await aw(w.export_memory.remote()) for w in ws]
                if not all(infos):
                    return False
                await asyncio.gather(*[aw(w.import_peers.remote(
                    {insts[j].instance_id: infos[j] for j in range(len(ws)) if j != i}, "global"))
                    for i, w in enumerate(ws)])
        self.global_p2p = True
        return True

    async def transfer_requests(self, src, dst, max_pages: int) -> int:
        """Move running requests (and their KV pages) from instance ``src``
        to instance ``dst`` of another group: both stop briefly; every
        destination worker pulls the pages from its source counterpart over
        NVLink (or the pair exchanges them over the ``global`` NCCL
        communicator).  Returns the pages moved."""
        import time
        from ..runtime.actors import aw
        t0 = time.perf_counter()
        await src.stop_and_wait()
        await dst.stop_and_wait()
        try:
            items = src.pop_transferable(max_pages)
            moved = dst.take_pages_for(items)
            src.return_transferable(items[len(moved):])
            if not moved:
                return 0
            src_pages = [p for _, sp, _ in moved for p in sp]
            dst_pages = [p for _, _, dp in moved for p in dp]
            pp = src.pp_size
            futs = []
            for st in range(pp):
                for t in range(src.tp_size):
                    ws, wd = src.workers[st][t], dst.workers[st][t]
                    if self.global_p2p:
                        futs.append(wd.pull_blocks.remote(src.instance_id, src_pages, dst_pages))
                    else:
                        # global comm index: instance * pp + stage (same TP rank)
                        futs.append(ws.send_blocks.remote(dst.instance_id * pp + st, src_pages))
                        futs.append(wd.recv_blocks.remote(src.instance_id * pp + st, dst_pages))
            await asyncio.gather(*[aw(f) for f in futs])
            bm = src.block_managers[0]
            for r, _, _ in moved:
                bm.free_request(r.request_id)
            dst.adopt_transferred(moved)
            self.transfers.append((src.instance_id, dst.instance_id, len(dst_pages), time.perf_counter() - t0))
            logger.info(f"moved {len(moved)} requests ({len(dst_pages)} pages) from instance {src.instance_id} "
                        f"to instance {dst.instance_id} in {time.perf_counter() - t0:.3f}s")
            return len(dst_pages)
        finally:
            src.stopped = False
            dst.stopped = False

    async def balance_groups(self) -> int:
        """One step of cross-group load balancing: when an unfused instance's
        KV demand reaches ``transfer_high`` and an unfused instance of another
        group is below ``transfer_low``, move half the page difference."""
        cands = self._unfused_instances()
        if len({gi for gi, _ in cands}) < 2:
            return 0
        loads = [(inst.get_used_gpu_blocks() / max(inst.get_capacity_units(), 1), gi, inst) for gi, inst in cands]
        hi = max(loads, key=lambda x: x[0])
        lo = min((x for x in loads if x[1] != hi[1]), key=lambda x: x[0], default=None)
        if lo is None or hi[0] < self.transfer_high or lo[0] >= self.transfer_low:
            return 0
        pages = int((hi[2].get_used_gpu_blocks() - lo[2].get_used_gpu_blocks()) // 2)
        return await self.transfer_requests(hi[2], lo[2], pages) if pages > 0 else 0

    def start(self) -> None:
        self._tasks.append(asyncio.create_task(self.collect_loop()))
        if self.enable_balloon:
            self._tasks.append(asyncio.create_task(self.monitor_engine_events()))

    def stop(self) -> None:
        for t in self._tasks:
            t.cancel()
        self._tasks.clear()
