"""Block-manager accounting: unit cases of every transition and a randomized
(hypothesis) sequence of operations with invariants checked after each."""
import pytest
from hypothesis import given, settings, strategies as st

from kunserve_b200.kv import BlockManager, KVLayout, NoFreeBlocksError
from kunserve_b200.kv import copy_plan
from kunserve_b200.request import Request, SamplingParams


def R(rid, n_tokens, fusion=False, rank=0):
    r = Request(0.0, rid, None, [1] * n_tokens, SamplingParams(max_tokens=100))
    r.fusion_exec, r.kv_fusion_rank = fusion, rank
    return r


def test_dp_allocate_grow_free():
    bm = BlockManager(8, block_size=16)
    r = R(1, 20)
    assert len(bm.allocate_blocks(r)) == 2
    r.prompt_token_ids += [1] * 20
    assert len(bm.allocate_blocks(r)) == 1
    bm.check_invariants()
    with pytest.raises(NoFreeBlocksError):
        bm.allocate_blocks(R(2, 16 * 6))
    bm.check_invariants()          # failed allocation left nothing behind
    bm.free_blocks(r)
    assert bm.num_free_whole() == 8
    bm.check_invariants()


def test_balloon_transitions_and_ids():
    P, N = 8, 2
    bm = BlockManager(P, block_size=16)
    stale = R(1, 40)               # 3 whole pages
    bm.allocate_blocks(stale)
    bm.convert_to_pipeline_format(N)
    ext = bm.add_ex_fusion_blocks(5)
    assert ext == list(range(N * P, N * P + 5))
    new = R(2, 16 * 12, fusion=True)     # needs 12 slices: 10 from 5 free pages + 2 extend
    got = bm.allocate_blocks(new)
    assert sum(1 for f in got if f >= N * P) == 2
    bm.check_invariants()
    pages = list(bm.get_single_block_table(1))
    bm.free_blocks_into_fusion_except(1, N, 1)
    assert bm.get_single_block_table(1) == [1 * P + b for b in pages]
    bm.check_invariants()
    # restore: stop extend, pack extend pages of `new` into base slices
    bm.start_extend_reclaim()
    bm.free_blocks(stale)
    moves = bm.pack_blocks_into_base_region([new])
    assert len(moves) == 2 and all(s >= N * P and d < N * P for s, d in moves)
    assert bm.extend_reclaimed()
    bm.restore_kvblocks()
    assert not bm.is_fusion_state
    bm.check_invariants()
    dp = R(3, 16)                  # unfused allocation takes a whole free page
    bm.allocate_blocks(dp)
    assert bm._kind[3] == "whole"
    bm.free_blocks(new)
    bm.free_blocks(dp)
    bm.restore_from_fusion()
    assert bm.fusion_size == 1 and bm.num_free_whole() == P
    bm.check_invariants()


def test_swap_round_trip():
    bm = BlockManager(4, num_cpu_blocks=4, block_size=16)
    r = R(1, 40)
    bm.allocate_blocks(r)
    pairs = bm.swap_out_requests([r])
    assert len(pairs) == 3 and bm.num_free_whole() == 4
    back = bm.swap_in_requests([r])
    assert [c for c, _ in back] == [c for _, c in pairs]
    bm.check_invariants()


def test_copy_plan_offsets_match_layout():
    lay = KVLayout(num_pages=8, num_layers=4, block_size=16, num_kv_heads=2, head_dim=8)
    # slice k of whole page b is where layers [k*Ls, (k+1)*Ls) of page b live
    for b in range(8):
        for k in range(2):
            assert copy_plan.whole_page_slice_offset(lay, b, k, 2) == lay.kv_offset(b, k * 2, 1)
    send, recv = copy_plan.reshard_plan(lay, 2, 0, [[3, 5], [9, 17]])
    assert send[1] == [lay.kv_offset(3, 2, 1), lay.kv_offset(5, 2, 1)]
    assert recv[1] == [lay.kv_offset(9, 0, 2), lay.kv_offset(17, 0, 2)]


ops = st.lists(st.tuples(st.sampled_from(["alloc", "grow", "free", "fuse", "ext", "except", "reclaim"]),
                         st.integers(0, 7), st.integers(1, 70)), min_size=5, max_size=60)


@settings(max_examples=60, deadline=None)
@given(ops)
def test_random_operations_keep_invariants(seq):
    P = 12
    bm = BlockManager(P, block_size=16)
    live = {}
    for op, rid, n in seq:
        if op == "alloc" and rid not in live:
            r = R(rid, n, fusion=bm.is_fusion_state)
            try:
                bm.allocate_blocks(r)
                live[rid] = r
            except NoFreeBlocksError:
                pass
        elif op == "grow" and rid in live:
            live[rid].prompt_token_ids += [1] * (n % 20)
            try:
                bm.allocate_blocks(live[rid])
            except NoFreeBlocksError:
                pass
        elif op == "free" and rid in live:
            bm.free_blocks(live.pop(rid))
        elif op == "fuse" and not bm.is_fusion_state and bm.fusion_size == 1:
            bm.convert_to_pipeline_format(2)
        elif op == "ext" and bm.is_fusion_state and not bm._ext_reclaiming:
            bm.add_ex_fusion_blocks(n % 5)
        elif op == "except" and rid in live and bm.fusion_size == 2 and bm._kind.get(rid) == "whole":
            bm.free_blocks_into_fusion_except(rid, 2, rid % 2)
            live[rid].fusion_exec = True
        elif op == "reclaim" and bm.is_fusion_state:
            bm.start_extend_reclaim()
        bm.check_invariants()
        used = bm.used_pages()
        assert 0 <= used <= bm.capacity_pages() + 1e-9
