"""Host-side attention work lists (no GPU): decode work units, prefill item
order and split counts, as packed by ``native_runner.pack_meta``."""
import numpy as np
import pytest

from kunserve_b200.engine.native_runner import (DEC_UNIT_SLOTS, Q_TILE_ROWS, decode_units, pack_meta,
                                                prefill_splits)
from kunserve_b200.engine.step import StepInput


def _check_cover(units, ctx):
    """Every request's units are consecutive and cover its key blocks once."""
    blocks = (np.asarray(ctx) + 63) // 64
    u = 0
    for i, b in enumerate(blocks):
        first, count = units[u, 3] >> 8, units[u, 3] & 255
        assert first == u and 1 <= count <= 32
        nxt = 0
        for j in range(count):
            di, blk0, nb, w = units[u + j]
            assert di == i and w == units[u, 3] and blk0 == nxt and nb > 0
            nxt += nb
        assert nxt == b
        u += count
    assert u == len(units) <= DEC_UNIT_SLOTS


def test_uniform_batches_keep_about_one_wave():
    # 64 requests x 8 heads already fill two CTAs per SM: no cutting
    u = decode_units(np.full(64, 512), 8, 148)
    assert len(u) == 64
    _check_cover(u, np.full(64, 512))
    # 16 requests: two units each
    assert len(decode_units(np.full(16, 2048), 8, 148)) == 32
    # one request: 128-key units, at most 32
    assert len(decode_units(np.array([2048]), 8, 148)) == 16
    assert len(decode_units(np.array([8192]), 8, 148)) == 32


def test_skewed_batch_cuts_only_the_long_context():
    ctx = np.array([8192] + [700] * 29)
    u = decode_units(ctx, 8, 148)
    _check_cover(u, ctx)
    counts = np.bincount(u[:, 0], minlength=len(ctx))
    assert counts[0] >= 8 and (counts[1:] == 1).all()
    # the long request's units are no larger than a short request
    assert u[u[:, 0] == 0, 2].max() <= 16
    assert len(u) * 8 <= 1.1 * 2 * 148


@pytest.mark.parametrize("seed", range(5))
def test_random_batches_cover_every_block(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 300))
    ctx = rng.integers(1, 20000, size=n)
    u = decode_units(ctx, int(rng.choice([1, 2, 8])), 148)
    _check_cover(u, ctx)


def test_many_requests_stay_within_the_unit_scratch():
    ctx = np.full(DEC_UNIT_SLOTS, 100000)
    u = decode_units(ctx, 8, 148)
    assert len(u) == DEC_UNIT_SLOTS
    _check_cover(u, ctx)
    with pytest.raises(ValueError):
        decode_units(np.ones(DEC_UNIT_SLOTS + 1, dtype=np.int64), 8, 148)


def test_pack_meta_orders_items_longest_first_and_lists_units():
    G, bs = 4, 16
    starts, qlens = [0, 1000, 300, 5000], [600, 100, 1, 1]
    tables = [list(range(k * 400, k * 400 + (s + n + bs - 1) // bs)) for k, (s, n) in enumerate(zip(starts, qlens))]
    step = StepInput(list(range(4)), [[0] * n for n in qlens], starts, tables, [1, 1, 0, 0], 0, 1)
    buf = np.zeros(20000, dtype=np.int32)
    width = max(len(t) for t in tables)
    n, T, B, n_items, pre_ctx, n_dec, n_units, hg = pack_meta(step, bs, G, width, buf, 8, 148)
    assert hg == 1
    assert (T, B, n_dec) == (702, 4, 2)
    assert pre_ctx == 1100   # decode contexts do not count for prefill splits
    items = buf[:2 * n_items].reshape(n_items, 2)
    assert n_items == -(-600 * G // Q_TILE_ROWS) + -(-100 * G // Q_TILE_ROWS)
    # keys seen by each item's last row, non-increasing
    ends = [starts[r] + min(row0 + Q_TILE_ROWS, qlens[r] * G) // G for r, row0 in items]
    assert ends == sorted(ends, reverse=True)
    o_dec = n - 8 * n_units - n_dec
    assert buf[o_dec:o_dec + n_dec].tolist() == [2, 3]
    rec = buf[o_dec + n_dec:n].reshape(n_units, 8)
    _check_cover(rec[:, [6, 3, 4, 5]], [301, 5001])
    # token row, context and request of each unit's decode request
    q_start = np.cumsum([0] + qlens)
    for r in rec:
        req = [2, 3][r[6]]
        assert (r[0], r[1], r[2], r[7]) == (q_start[req], starts[req] + 1, req, 0)


def test_wide_decode_ctas_only_for_large_batches():
    bs, G = 16, 4
    for n, ctx, want in ((2, 300, 1), (64, 2048, 4)):
        tables = [list(range(k * 200, k * 200 + (ctx + bs - 1) // bs)) for k in range(n)]
        step = StepInput(list(range(n)), [[0]] * n, [ctx - 1] * n, tables, [0] * n, 0, 1)
        buf = np.zeros(40000, dtype=np.int32)
        *_, n_units, hg = pack_meta(step, bs, G, max(len(t) for t in tables), buf, 8, 148, hg_max=4)
        assert hg == want
        units = decode_units(np.full(n, ctx), 8 // hg, 148)
        assert n_units == len(units)


def test_prefill_splits_stay_within_one_wave():
    assert prefill_splits(512, 8, 512, 8, 148) == 1
    assert prefill_splits(512, 8, 4096, 8, 148) == 2
    assert prefill_splits(128, 2, 4096, 8, 148) == 9
    assert prefill_splits(600, 8, 8192, 8, 148) == 1   # large steps never split
