"""Balloon group controller: ``group_size`` DP instances that fuse into one
pipeline under KV overload and split back afterwards.

Parity: ``kunserve/llm_engine.py`` ``ColocatedEngine`` (:327-837): state
machine ``INITIAL -> BALLOON -> RESTORE -> INITIAL`` (every transition via
``STOP``), voting (``make_decision_for``: INIT needs every vote, the others a
majority of at least one), ``trigger_balloon`` / ``trigger_restore`` /
``trigger_init``, ``get_event`` and engine monitoring.  The group owns its
instances directly (one controller per group instead of the reference's
leader/follower property shuffling).  Unlike the reference
(``coordinator.py:152-160``) a transition only ever acts on the group that
voted for it.
"""
import asyncio
import time
from typing import Dict, List, Optional, Tuple

from ..engine.instance import InstanceEngine
from ..request import Request
from ..utils.logger import init_logger
from ..utils.misc import EngineState, Event
from ..utils.trace import nvtx_range

logger = init_logger(__name__)


class GroupEngine:
    def __init__(self, group_id: int, instances: List[InstanceEngine], balloon_mode: str = "reshard",
                 max_balloon_memory_ratio: float = 0.5):
        self.group_id = group_id
        self.instances = instances
        self.balloon_mode = balloon_mode
        self.max_balloon_memory_ratio = max_balloon_memory_ratio
        self.state = EngineState.INITIAL
        self.tasks: Dict[int, asyncio.Task] = {}
        self.transitions: List[Tuple[float, str, float]] = []
        self.failed: Optional[BaseException] = None
        self.p2p = False
        for inst in instances:
            inst.peers = instances

    @property
    def leader(self) -> InstanceEngine:
        return self.instances[0]

    def active_instances(self) -> List[InstanceEngine]:
        return self.instances if self.state == EngineState.INITIAL else self.instances[:1]

    # ------------------------------------------------------------ loops
    def start(self) -> None:
        for i, inst in enumerate(self.instances):
            if i not in self.tasks or self.tasks[i].done():
                if inst.state != "merged":
                    self.tasks[i] = asyncio.create_task(inst.start_event_loop())

    async def monitor_engines(self, interval: float = 0.05) -> None:
        """Restart an instance loop that ended while it was not stopped (the
        reference's monitor, ``llm_engine.py:649-672``); surface crashes."""
        while True:
            for i, t in list(self.tasks.items()):
                if t.done():
                    exc = t.exception()
                    if exc is not None:
                        self.failed = exc
                        logger.error(f"group {self.group_id}: instance {i} crashed: {exc!r}")
                        raise exc
                    inst = self.instances[i]
                    if not getattr(inst, "_terminate", False) and inst.state != "merged":
                        self.tasks[i] = asyncio.create_task(inst.start_event_loop())
            await asyncio.sleep(interval)

    async def stop_all_engines(self) -> None:
        for inst in self.instances:
            await inst.stop_and_wait()

    def terminate(self) -> None:
        for inst in self.instances:
            inst.terminate()

    async def setup_peer_memory(self) -> bool:
        """Map every member's KV pool and weight segments into its peers
        (same pipeline stage and TP rank), so reshard, live restore and
        parameter restore pull over NVLink inside the copy kernel.  Returns
        False when the workers have no native engine."""
        from ..runtime.actors import aw
        if len(self.instances) < 2:
            return False
        pp, tp = self.leader.pp_size, self.leader.tp_size
        for st in range(pp):
            for t in range(tp):
                members = [inst.workers[st][t] for inst in self.instances]
                infos = [await aw(w.export_memory.remote()) for w in members]
                if not all(infos):
                    return False
                await asyncio.gather(*[aw(w.import_peers.remote({j: infos[j] for j in range(len(members))
                                                                 if j != i}))
                                       for i, w in enumerate(members)])
        self.p2p = True
        for inst in self.instances:
            inst.p2p_kv = True
        return True

    # ------------------------------------------------------------ votes
    async def make_decision_for(self, engines: List[InstanceEngine], event: Event) -> bool:
        votes = [e.vote_for(event) for e in engines if e.state != "merged" or e is self.leader]
        if event == Event.INIT:
            return all(votes)
        return sum(votes) > 0 and sum(votes) >= len(votes) // 2

    async def get_event(self) -> Tuple[EngineState, Optional[Event]]:
        if len(self.instances) < 2:
            return self.state, None
        if self.state == EngineState.INITIAL:
            if await self.make_decision_for(self.instances, Event.BALLOON):
                return self.state, Event.BALLOON
        elif self.state == EngineState.BALLOON:
            if await self.make_decision_for(self.instances[:1], Event.RESTORE):
                return self.state, Event.RESTORE
        elif self.state == EngineState.RESTORE:
            if await self.make_decision_for(self.instances[:1], Event.INIT):
                return self.state, Event.INIT
        return self.state, None

    # ------------------------------------------------------- transitions
    async def trigger_balloon(self, from_restore: bool = False) -> int:
        with nvtx_range(f"kunserve.group{self.group_id}.balloon"):
            return await self._trigger_balloon(from_restore)

    async def _trigger_balloon(self, from_restore: bool) -> int:
        t0 = time.perf_counter()
        prev = self.state
        self.state = EngineState.STOP
        free = await self.leader.trigger_balloon(self.balloon_mode, from_restore, self.instances[1:])
        self.state = EngineState.BALLOON
        self.start()
        dt = time.perf_counter() - t0
        self.transitions.append((time.time(), f"{prev.name}->BALLOON", dt))
        logger.info(f"group {self.group_id}: {prev.name} -> BALLOON in {dt:.3f}s")
        return int(free * self.max_balloon_memory_ratio)

    async def trigger_restore(self) -> None:
        with nvtx_range(f"kunserve.group{self.group_id}.restore"):
            await self._trigger_restore()

    async def _trigger_restore(self) -> None:
        """Reclaim the extend pages, pull the dropped parameters back while
        the fused pipeline keeps serving (the reference restores before it
        stops the engines, ``kunserve/llm_engine.py:546-570``), then stop
        briefly to switch the block managers back to whole pages."""
        t0 = time.perf_counter()
        leader = self.leader
        await leader.reclaim_extra_blocks()
        await leader.pmm_restore()
        self.state = EngineState.STOP
        await self.stop_all_engines()
        leader.restore_instance()
        self.state = EngineState.RESTORE
        self.start()
        dt = time.perf_counter() - t0
        self.transitions.append((time.time(), "BALLOON->RESTORE", dt))
        logger.info(f"group {self.group_id}: BALLOON -> RESTORE in {dt:.3f}s")

    async def trigger_init(self) -> None:
        with nvtx_range(f"kunserve.group{self.group_id}.init"):
            await self._trigger_init()

    async def _trigger_init(self) -> None:
        t0 = time.perf_counter()
        self.state = EngineState.STOP
        await self.stop_all_engines()
        leader = self.leader
        leader.split_engine(self.instances[1:])
        for inst in self.instances:
            inst.trigger_init()
        self.state = EngineState.INITIAL
        self.start()
        dt = time.perf_counter() - t0
        self.transitions.append((time.time(), "RESTORE->INITIAL", dt))
        logger.info(f"group {self.group_id}: RESTORE -> INITIAL in {dt:.3f}s")

    async def handle_event(self, event: Optional[Event]) -> None:
        if event == Event.BALLOON:
            await self.trigger_balloon(from_restore=self.state == EngineState.RESTORE)
        elif event == Event.RESTORE:
            await self.trigger_restore()
        elif event == Event.INIT:
            await self.trigger_init()

    # ------------------------------------------------------------ load
    def get_gpu_blocks_usage(self):
        return self.state, [inst.get_gpu_blocks_usage() for inst in self.active_instances()]

    def add_request(self, instance_idx: int, request: Request) -> None:
        """Requests for a merged member go to the leader, which owns its VEs."""
        inst = self.instances[instance_idx]
        if inst.state == "merged":
            inst = self.leader
        inst.add_request(request)

    def get_unfinished(self) -> int:
        return sum(i.get_unfinished_requests() for i in self.instances)
