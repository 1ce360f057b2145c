from kunserve_b200.config import SchedConfig
from kunserve_b200.kv import BlockManager
from kunserve_b200.request import Request, SamplingParams
from kunserve_b200.sched import ColocatedScheduler


def R(rid, n, gen=0, t=0.0):
    r = Request(t, rid, None, list(range(n)), SamplingParams(max_tokens=50))
    for i in range(gen):
        r.add_generated_token("", i)
    return r


def _sched(policy="prefill-first", chunked=False):
    bm = BlockManager(32, block_size=16)
    return ColocatedScheduler(SchedConfig(policy=policy, enable_chunked_prefill=chunked), [bm], 16), bm


def test_prefill_first_vs_mixed():
    s, _ = _sched()
    p, d = R(1, 10), R(2, 10, gen=2)
    s.running_queue.requests = [d, p]
    b, has = s.schedule()
    assert [r.request_id for r in b] == [1] and has
    s2, _ = _sched("mixed")
    s2.running_queue.requests = [d, p]
    b, _ = s2.schedule()
    assert sorted(r.request_id for r in b) == [1, 2]


def test_recompute_victim_is_newest_decode_and_requeued_first():
    s, bm = _sched()
    old, new = R(1, 20, gen=3, t=1.0), R(2, 20, gen=3, t=2.0)
    for r in (old, new):
        bm.allocate_blocks(r)
        s.running_queue.add_request(r)
    v = s.trigger_recompute(False, 0)
    assert v is new and v.get_input_len() == 23 and v.get_output_len() == 0
    assert s.unaccepted_queue[0] is new and not bm.is_allocated(2)
    assert s.num_preemption == 1 and new.preempted_times == 1
    bm.check_invariants()


def test_abort_and_queue_accounting():
    s, _ = _sched()
    s.add_request(R(1, 5))
    s.add_request(R(2, 5))
    assert s.get_num_unfinished_requests() == 2
    assert s.abort_request(1)
    assert s.get_num_unfinished_requests() == 1
    r = R(3, 5)
    s.running_queue.add_request(r)
    s.abort_request(3)
    assert r.is_finished


def test_chunk_sizing():
    r = R(1, 100)
    assert r.set_chunk(30) == 0 and r.get_num_input_tokens() == 30 and r.have_follow_up_chunk()
    assert r.get_optimal_chunk_size(10_000, floor=16) >= 16
