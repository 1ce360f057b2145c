"""Global dispatcher across servers (parity: the reference's deprecated
``kunserve/global_dispatcher.py:22-250``).

Round-robin or least-load dispatch over a list of front ends, plus the
Llumnix-style rebalance the reference sketched: when one server queues
requests it cannot admit while another has spare KV, its queued (not yet
admitted) requests move to the least-loaded server.  The coordinator inside
each ``AsyncLLM`` handles dispatch within a server; this layer is only
needed with several front ends.
"""
from typing import List, Sequence


class GlobalDispatcher:
    def __init__(self, servers: Sequence, strategy: str = "round-robin"):
        self.servers = list(servers)
        self.strategy = strategy
        self._rr = 0

    def pick(self):
        if self.strategy == "round-robin":
            s = self.servers[self._rr % len(self.servers)]
            self._rr += 1
            return s
        return min(self.servers, key=lambda s: s.get_unfinised_num())

    async def generate(self, **kw):
        return await self.pick().generate(**kw)

    def redispatch(self, min_gap: int = 4) -> int:
        """Move queued requests from the most to the least loaded server's
        instances; returns how many moved."""
        if len(self.servers) < 2:
            return 0
        loads = [(s.check_pending_num(), s) for s in self.servers]
        (hi_n, hi), (lo_n, lo) = max(loads, key=lambda x: x[0]), min(loads, key=lambda x: x[0])
        if hi_n - lo_n < min_gap:
            return 0
        moved: List = []
        budget = (hi_n - lo_n) // 2
        for g in hi.groups:
            for inst in g.instances:
                while inst.unaccepted_queue and len(moved) < budget:
                    moved.append(inst.unaccepted_queue.pop())
        target = lo.groups[0].leader
        target.add_requests(moved)
        # outputs still flow to the original server's streams
        target.output_callback = _Tee(target.output_callback, hi.router)
        return len(moved)


class _Tee:
    def __init__(self, a, b):
        self.a, self.b = a, b

    def __call__(self, outs):
        if self.a is not None:
            self.a(outs)
        self.b(outs)
