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
                 load_interval: float = LOAD_INTERVAL_S, fsm_interval: float = FSM_INTERVAL_S):
        self.groups = groups
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
            await asyncio.sleep(self.fsm_interval)

    def start(self) -> None:
        self._tasks.append(asyncio.create_task(self.collect_loop()))
        if self.enable_balloon:
            self._tasks.append(asyncio.create_task(self.monitor_engine_events()))

    def stop(self) -> None:
        for t in self._tasks:
            t.cancel()
        self._tasks.clear()
