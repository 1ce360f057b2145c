"""Rank layout of a serving job and the members of its five communicators.

Global rank = ((((server * ngroups + group) * group_size + instance) * pp
+ stage) * tp + tp_rank).  The communicators follow the reference's
(``kunserve/flash_backend.py:323-376``, ``llm_engine.py:437-439``,
``llm.py:165-167``):

* ``tp``     — TP ranks of one pipeline stage of one instance;
* ``pp``     — stages of one instance (same TP rank);
* ``gp``     — the fused pipeline of a balloon group: every stage of every
  instance of the group (same TP rank), ordered ``instance * pp + stage``;
* ``kvex``   — same members as ``gp``; carries KV reshard and parameter restore;
* ``global`` — every stage of every instance of a server (same TP rank),
  ordered ``(group * group_size + instance) * pp + stage``; carries
  cross-group block transfer.
"""
from dataclasses import dataclass
from typing import Dict, List, Tuple

COMMS = ("tp", "pp", "gp", "kvex", "global")


@dataclass(frozen=True)
class Topology:
    nservers: int = 1
    ngroups: int = 1
    group_size: int = 1
    pp: int = 1
    tp: int = 1

    @property
    def world_size(self) -> int:
        return self.nservers * self.ngroups * self.group_size * self.pp * self.tp

    def rank_of(self, server: int, group: int, inst: int, stage: int, tp_rank: int) -> int:
        return ((((server * self.ngroups + group) * self.group_size + inst) * self.pp + stage)
                * self.tp + tp_rank)

    def coords(self, rank: int) -> Tuple[int, int, int, int, int]:
        tp_rank = rank % self.tp
        rank //= self.tp
        stage = rank % self.pp
        rank //= self.pp
        inst = rank % self.group_size
        rank //= self.group_size
        group = rank % self.ngroups
        server = rank // self.ngroups
        return server, group, inst, stage, tp_rank

    def members(self, comm: str, rank: int) -> List[int]:
        s, g, i, st, t = self.coords(rank)
        if comm == "tp":
            return [self.rank_of(s, g, i, st, r) for r in range(self.tp)]
        if comm == "pp":
            return [self.rank_of(s, g, i, x, t) for x in range(self.pp)]
        if comm in ("gp", "kvex"):
            return [self.rank_of(s, g, ii, x, t) for ii in range(self.group_size) for x in range(self.pp)]
        if comm == "global":
            return [self.rank_of(s, gg, ii, x, t) for gg in range(self.ngroups)
                    for ii in range(self.group_size) for x in range(self.pp)]
        raise KeyError(comm)

    def all_groups(self, comm: str) -> List[Tuple[int, ...]]:
        """Every distinct member list of ``comm`` in a fixed order (every rank
        must create process groups in the same order)."""
        seen: Dict[Tuple[int, ...], None] = {}
        for r in range(self.world_size):
            seen.setdefault(tuple(self.members(comm, r)), None)
        return list(seen)

    def instance_ranks(self, server: int, group: int, inst: int) -> List[List[int]]:
        """``[stage][tp_rank]`` global ranks of one instance."""
        return [[self.rank_of(server, group, inst, st, t) for t in range(self.tp)] for st in range(self.pp)]
