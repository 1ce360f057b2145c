"""Communicators of the largest single-node layout (two balloon groups of two
TP2 instances, eight ranks) on gloo processes: every rank builds the five
communicators, sets up their links at start-up without any rank waiting on
another's order, and each communicator then carries data between exactly
its members."""
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kunserve_b200.parallel.topology import COMMS, Topology

TOPO = Topology(nservers=1, ngroups=2, group_size=2, pp=1, tp=2)


def _rank(rank, world, init_file, q):
    try:
        torch.set_num_threads(1)
        from kunserve_b200.parallel.comm import Communicator, init_default_group
        init_default_group("gloo", rank, world, timeout_s=60, init_file=init_file)
        comm = Communicator(TOPO, rank, "gloo")
        sums = {}
        for c in COMMS:
            members = comm.members[c]
            x = torch.tensor([float(rank)])
            if comm.groups[c] is not None:
                dist.all_reduce(x, group=comm.groups[c])
            sums[c] = (x.item(), float(sum(members)))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, sums, None))
    except Exception as e:  # noqa: BLE001 - reported to the test
        q.put((rank, None, repr(e)))


@pytest.mark.slow
def test_eight_rank_communicators_warm_and_carry_their_members():
    world = TOPO.world_size
    assert world == 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "rdv")
        procs = [ctx.Process(target=_rank, args=(r, world, init_file, q)) for r in range(world)]
        for p in procs:
            p.start()
        results = [q.get(timeout=240) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
    for rank, sums, err in results:
        assert err is None, (rank, err)
        for c, (got, want) in sums.items():
            assert got == want, (rank, c, got, want)
