"""Communicators over ``torch.distributed`` (gloo on CPU, NCCL on GPU).

Creates the five communicators of ``topology.py`` as process groups and
offers the few operations the engine needs: TP all-reduce, point-to-point
activation transfer on ``pp``/``gp``, and chunked KV / parameter transfer on
``kvex``/``global``.  The fused TP GEMM+all-reduce and the P2P copy kernels of
the native engine replace the TP and KV paths on GPU; this module is their
baseline and the CPU implementation.
"""
import os
from datetime import timedelta
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .topology import COMMS, Topology


def init_default_group(backend: str, rank: int, world_size: int, timeout_s: float = 120.0,
                       master_addr: str = "127.0.0.1", master_port: Optional[int] = None,
                       init_file: Optional[str] = None) -> None:
    """Join the job's default process group: through a shared file when
    ``init_file`` is given (processes on one node; no port to race for),
    else through ``master_addr:master_port``."""
    if dist.is_initialized():
        return
    if init_file is not None:
        dist.init_process_group(backend, init_method=f"file://{init_file}", rank=rank, world_size=world_size,
                                timeout=timedelta(seconds=timeout_s))
        return
    os.environ.setdefault("MASTER_ADDR", master_addr)
    if master_port is not None:
        os.environ["MASTER_PORT"] = str(master_port)
    os.environ.setdefault("MASTER_PORT", "29511")
    dist.init_process_group(backend, rank=rank, world_size=world_size,
                            timeout=timedelta(seconds=timeout_s))


class Communicator:
    """The five communicators of one rank."""

    def __init__(self, topo: Topology, rank: int, backend: Optional[str] = None):
        self.topo = topo
        self.rank = rank
        self.backend = backend or dist.get_backend()
        self.groups: Dict[str, object] = {}
        self.members: Dict[str, List[int]] = {}
        for comm in COMMS:
            for ranks in topo.all_groups(comm):
                if len(ranks) == 1:
                    g = None
                else:
                    g = dist.new_group(list(ranks), backend=self.backend)
                if rank in ranks:
                    self.groups[comm] = g
                    self.members[comm] = list(ranks)
        if os.environ.get("KUNSERVE_WARM_LINKS", "1") != "0":
            self.warm_links()

    def warm_links(self) -> None:
        """Set up every communicator's collective and point-to-point links
        now: NCCL creates them at their first use, and the first use of the
        fused pipeline's activation sends (or of a KV or parameter exchange)
        would otherwise pay that set-up inside serving, right after a balloon
        transition.  Every rank calls this at the same point (groups of one
        comm type are disjoint, and each group's sends and receives go in one
        batch), so no rank waits on another's order."""
        dev = torch.device("cuda", torch.cuda.current_device()) if self.backend == "nccl" else torch.device("cpu")
        for comm in COMMS:
            g, members = self.groups.get(comm), self.members.get(comm, [])
            if g is None or len(members) < 2:
                continue
            x = torch.zeros(1, device=dev)
            dist.all_reduce(x, group=g)
            ops, bufs = [], []
            for peer in members:
                if peer == self.rank:
                    continue
                b = torch.zeros(1, device=dev)
                bufs.append(b)
                ops.append(dist.P2POp(dist.isend, torch.ones(1, device=dev), peer, group=g))
                ops.append(dist.P2POp(dist.irecv, b, peer, group=g))
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        if self.backend == "nccl":
            torch.cuda.synchronize()

    def size(self, comm: str) -> int:
        return len(self.members[comm])

    def index(self, comm: str) -> int:
        return self.members[comm].index(self.rank)

    def peer(self, comm: str, idx: int) -> int:
        return self.members[comm][idx]

    def tp_all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size("tp") == 1:
            return x
        y = x.contiguous()
        dist.all_reduce(y, group=self.groups["tp"])
        return y

    def send(self, x: torch.Tensor, comm: str, idx: int) -> None:
        dist.send(x.contiguous(), self.peer(comm, idx), group=self.groups[comm])

    def isend(self, x: torch.Tensor, comm: str, idx: int):
        """Start a point-to-point send; returns the work handle (the caller
        keeps ``x`` alive until it completes)."""
        return dist.isend(x, self.peer(comm, idx), group=self.groups[comm])

    def recv(self, shape, dtype, device, comm: str, idx: int) -> torch.Tensor:
        out = torch.empty(shape, dtype=dtype, device=device)
        dist.recv(out, self.peer(comm, idx), group=self.groups[comm])
        return out

    def exchange(self, comm: str, sends: Dict[int, torch.Tensor],
                 recv_shapes: Dict[int, Tuple[Tuple[int, ...], torch.dtype]], device) -> Dict[int, torch.Tensor]:
        """Pairwise exchange with every peer in one batch of isend/irecv."""
        ops, outs = [], {}
        for idx, (shape, dtype) in recv_shapes.items():
            outs[idx] = torch.empty(shape, dtype=dtype, device=device)
        g = self.groups[comm]
        if self.backend == "gloo":
            reqs = []
            for idx, t in sends.items():
                reqs.append(dist.isend(t.contiguous(), self.peer(comm, idx), group=g))
            for idx, t in outs.items():
                reqs.append(dist.irecv(t, self.peer(comm, idx), group=g))
            for r in reqs:
                r.wait()
            return outs
        for idx, t in sends.items():
            ops.append(dist.P2POp(dist.isend, t.contiguous(), self.peer(comm, idx), g))
        for idx, t in outs.items():
            ops.append(dist.P2POp(dist.irecv, t, self.peer(comm, idx), g))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
        return outs

    def barrier(self, comm: Optional[str] = None) -> None:
        if comm is None:
            dist.barrier()
        elif self.size(comm) > 1:
            dist.barrier(group=self.groups[comm])
