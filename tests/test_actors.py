"""Actor runtime, including host-side failure injection: a method that
raises, a worker process that dies mid-call, and a rank that never joins."""
import os
import time

import pytest

from kunserve_b200.runtime import ActorDiedError, RemoteError, get, make_actor


class Echo:
    def __init__(self, base=0):
        self.base = base

    def add(self, x):
        return self.base + x

    def boom(self):
        raise ValueError("injected")

    def die(self):
        os._exit(3)

    def getpid(self):
        return os.getpid()


@pytest.mark.parametrize("kind", ["local", "thread", "process"])
def test_calls_and_errors(kind):
    a = make_actor(kind, Echo, 10)
    assert get(a.add.remote(5)) == 15
    with pytest.raises((ValueError, RemoteError)) as e:
        get(a.boom.remote())
    assert "injected" in str(e.value)
    assert get([a.add.remote(i) for i in range(3)]) == [10, 11, 12]
    a.kill()


def test_dead_process_fails_pending_calls():
    a = make_actor("process", Echo)
    assert get(a.getpid.remote()) != os.getpid()
    f = a.die.remote()
    with pytest.raises(ActorDiedError):
        get(f, timeout=30)
    with pytest.raises(ActorDiedError):
        get(a.add.remote(1), timeout=30)


def _join(rank, world, port, timeout):
    from kunserve_b200.parallel.comm import init_default_group
    init_default_group("gloo", rank, world, timeout_s=timeout, master_port=port)
    return rank


def test_rank_that_never_joins_times_out():
    from kunserve_b200.bootstrap import free_port
    from kunserve_b200.runtime import ProcessActor
    t0 = time.time()
    a = ProcessActor(_join, 0, 2, free_port(), 3.0, wait_ready=False)   # rank 1 never starts
    with pytest.raises(RemoteError):
        a.wait_ready(timeout=60)
    assert time.time() - t0 < 60
    a.kill()
