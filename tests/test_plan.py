"""Host-side schedule builder: tiles cover every token once, items are balanced."""
from __future__ import annotations

import numpy as np
import pytest

from asterq import _lib
from asterq.plan import COLD_TILE, COLD_TILE_INT8, HOT_TILE, SequenceLayout, build_plan


def _layout(cold, hot, q_start=0, q_len=1):
    return SequenceLayout(cold=cold, hot=hot, q_start=q_start, q_len=q_len)


def test_tiles_cover_each_token_once():
    seqs = [
        _layout([(0, 0, 512), (1, 0, 300)], [(0, 0, 512), (1, 0, 7)], 0, 1),
        _layout([], [(2, 10, 40)], 1, 3),
        _layout([], [], 4, 2),
    ]
    plan = build_plan(seqs, 16, n_sms=4)
    t = plan.tiles
    cold = t[t[:, 0] == _lib.TILE_COLD]
    hot = t[t[:, 0] == _lib.TILE_HOT]
    new = t[t[:, 0] == _lib.TILE_NEW]
    assert cold[:, 3].sum() == 812 and (cold[:, 3] <= COLD_TILE).all()
    assert hot[:, 3].sum() == 512 + 7 + 40 and (hot[:, 3] <= HOT_TILE).all()
    assert sorted(new[:, 1].tolist()) == [0, 1, 4] and sorted(new[:, 3].tolist()) == [1, 2, 3]
    assert plan.total_q == 6


def test_items_partition_tiles_per_row_block():
    seqs = [_layout([(i, 0, 512) for i in range(40)], [(0, 0, 512)], 0, 3)]
    plan = build_plan(seqs, 16, n_sms=8, ctas_per_sm=1, waves=1)
    items = plan.items
    # 3 q tokens x 16 heads = 48 rows = 3 row blocks, each split into several items
    for rb in range(3):
        mine = items[items[:, 1] == rb]
        ranges = sorted((int(a), int(b)) for a, b in mine[:, 2:4])
        assert ranges[0][0] == 0 and ranges[-1][1] == plan.tiles.shape[0]
        assert all(r0[1] == r1[0] for r0, r1 in zip(ranges[:-1], ranges[1:]))
        assert (mine[:, 4] >= 0).all()
    assert plan.combine.shape[0] == 3
    assert plan.n_slots == items.shape[0]
    assert set(plan.combine[:, 2].tolist()) == {0, 16, 32}


def test_single_item_sequences_write_output_directly():
    seqs = [_layout([], [(0, 0, 40)], i, 1) for i in range(10)]
    plan = build_plan(seqs, 16)
    assert (plan.items[:, 4] == -1).all() and plan.n_slots == 0 and plan.combine.shape[0] == 0


def test_items_sorted_longest_first():
    seqs = [_layout([(i, 0, 512)] * (i + 1), [], i, 1) for i in range(6)]
    plan = build_plan(seqs, 16, n_sms=1000, persistent=False)
    sizes = plan.items[:, 3] - plan.items[:, 2]
    assert (np.diff(sizes) <= 0).all()
    assert plan.workers is None


def _ragged_batch(n=64, seed=0):
    """C3-like: lengths U[1024, 32768], hot window 2048, cold chunks of 512, q_len 1."""
    rng = np.random.default_rng(seed)
    seqs, cp, hp = [], 0, 0
    for i, length in enumerate(rng.integers(1024, 32769, n)):
        hot = min(int(length), 2048)
        cold = int(length) - hot
        chunks = [(cp + k, 0, min(512, cold - s)) for k, s in enumerate(range(0, cold, 512))]
        cp += len(chunks)
        hots = [(hp + k, 0, min(512, hot - s)) for k, s in enumerate(range(0, hot, 512))]
        hp += len(hots)
        seqs.append(_layout(chunks, hots, i, 1))
    return seqs


def _item_ns(plan):
    from asterq.plan import _ITEM_NS, _tile_ns

    tns = np.array([_tile_ns(k, n) for k, _, _, n in plan.tiles])
    P = np.concatenate(([0], np.cumsum(tns)))
    return P[plan.items[:, 3]] - P[plan.items[:, 2]] + _ITEM_NS


@pytest.mark.parametrize("n_sms", [148, 37, 8])
def test_persistent_workers_cover_every_tile_once_and_balance(n_sms):
    from asterq.plan import _ITEM_NS, _MIN_PIECE_NS

    seqs = _ragged_batch()
    plan = build_plan(seqs, 16, n_sms=n_sms)
    w = plan.workers
    assert w is not None and w[0] == 0 and w[-1] == plan.items.shape[0] and (np.diff(w) >= 1).all()
    assert plan.n_workers <= n_sms
    # every unit's items tile its visible range exactly once, in order
    for unit in range(plan.n_units):
        mine = plan.items[plan.items[:, 0] == unit]
        ranges = sorted((int(a), int(b)) for a, b in mine[:, 2:4])
        assert all(r0[1] == r1[0] for r0, r1 in zip(ranges[:-1], ranges[1:]))
        assert ranges[-1][1] - ranges[0][0] == sum(b - a for a, b in ranges)
        if len(mine) == 1:
            assert mine[0, 4] == -1
        else:
            assert (mine[:, 4] >= 0).all()
    assert sorted(plan.items[plan.items[:, 4] >= 0, 4].tolist()) == list(range(plan.n_slots))
    # workers' estimated times within a few tiles of each other; pieces never tiny
    cost = _item_ns(plan)
    loads = np.array([cost[w[k]:w[k + 1]].sum() for k in range(plan.n_workers)])
    assert loads.max() <= loads.mean() + 2 * _MIN_PIECE_NS
    split = plan.items[:, 4] >= 0
    assert (cost[split] - _ITEM_NS >= 0.5 * _MIN_PIECE_NS).all()


def test_persistent_schedule_does_not_split_small_blocks():
    # blocks under two full cold tiles of work are never cut
    seqs = [_layout([], [(i, 0, 40)], i, 1) for i in range(10)]
    plan = build_plan(seqs, 16)
    assert plan.items.shape[0] == 10 and plan.n_slots == 0 and plan.n_workers == 10


def test_small_batch_cuts_finer_but_not_below_one_cold_tile():
    from asterq.plan import _COLD_TILE_NS, _ITEM_NS

    seqs = [_layout([(i, 0, 512) for i in range(14)], [(0, 0, 512), (1, 0, 512)], 0, 1)]  # one 8k sequence
    plan = build_plan(seqs, 16)
    assert plan.items.shape[0] > 40  # far more pieces than the 4-cold-tile minimum of a full batch allows
    cost = _item_ns(plan) - _ITEM_NS
    single_tile = (plan.items[:, 3] - plan.items[:, 2]) == 1
    assert ((cost >= sum(_COLD_TILE_NS) - 1) | single_tile).all()
    # a full batch keeps the larger minimum piece
    big = build_plan(_ragged_batch(), 16)
    from asterq.plan import _MIN_PIECE_NS

    split = big.items[:, 4] >= 0
    assert ((_item_ns(big) - _ITEM_NS)[split] >= 0.5 * _MIN_PIECE_NS).all()


def test_max_items_per_seq_deals_whole_blocks_to_workers():
    seqs = _ragged_batch(n=20, seed=1)
    plan = build_plan(seqs, 16, n_sms=8, max_items_per_seq=1)
    assert plan.items.shape[0] == 20 and plan.n_slots == 0 and plan.n_workers == 8
    cost = _item_ns(plan)
    w = plan.workers
    loads = np.array([cost[w[k]:w[k + 1]].sum() for k in range(8)])
    assert loads.max() - loads.min() <= cost.max()


@pytest.mark.parametrize("bad", [dict(q_len=0), dict(q_len=2049)])
def test_rejects_bad_q_len(bad):
    with pytest.raises(ValueError):
        build_plan([_layout([], [], 0, **bad)], 16)


def test_prefill_chunk_row_blocks_see_only_their_causal_prefix():
    """q_len 100 new tokens, 16 heads: 32-token new tiles; row block rb (token rb)
    keeps the cache plus the new tiles up to its own token."""
    from asterq.plan import HOT_TILE

    lay = _layout([(0, 0, 512)], [(1, 0, 64)], 0, q_len=100)
    plan = build_plan([lay], 16, max_items_per_seq=1)
    new = plan.tiles[plan.tiles[:, 0] == 2]
    assert [int(n) for n in new[:, 3]] == [32, 32, 32, 4]
    assert [int(o) for o in new[:, 2]] == [0, 32, 64, 96]
    n_cache = 512 // 128 + 64 // HOT_TILE
    for it in plan.items:
        rb, t0, t1 = int(it[1]), int(it[2]), int(it[3])
        assert t1 - t0 == n_cache + rb // HOT_TILE + 1


def test_rejects_bad_chunks():
    with pytest.raises(ValueError):
        build_plan([_layout([(0, 0, 0)], [])], 16)


@pytest.mark.parametrize("n_sms", [148, 16, 3])
def test_fused_combine_jobs(n_sms):
    """Blocks cut into at most FUSED_COMBINE_MAX_PARTS pieces are merged by the decode kernel:
    their jobs follow the separate ones and unit_jobs points at them."""
    from asterq.plan import FUSED_COMBINE_MAX_PARTS

    seqs = _ragged_batch(n=24, seed=2)
    seqs.append(_layout([(9000 + k, 0, 512) for k in range(400)], [], 24, 1))  # one very long block
    plan = build_plan(seqs, 16, n_sms=n_sms)
    n_sep = plan.n_separate
    parts = plan.combine[:, 1] - plan.combine[:, 0]
    assert (parts[:n_sep] > FUSED_COMBINE_MAX_PARTS).all()
    assert (parts[n_sep:] <= FUSED_COMBINE_MAX_PARTS).all() and (parts[n_sep:] >= 2).all()
    jobs = plan.unit_jobs if plan.unit_jobs is not None else np.full(plan.n_units, -1)
    assert sorted(j for j in jobs.tolist() if j >= 0) == list(range(n_sep, plan.combine.shape[0]))
    for unit, job in enumerate(jobs.tolist()):
        mine = plan.items[plan.items[:, 0] == unit]
        if job >= 0:  # the job covers exactly this unit's slots
            a, b = plan.combine[job, :2]
            assert sorted(mine[:, 4].tolist()) == list(range(a, b))
    # a worker runs its pieces of cut blocks first
    w = plan.workers
    for k in range(plan.n_workers):
        whole = plan.items[w[k]:w[k + 1], 4] < 0
        assert not (whole[:-1] & ~whole[1:]).any()


def test_force_partial_fuses_nothing():
    seqs = _ragged_batch(n=8, seed=3)
    plan = build_plan(seqs, 16, n_sms=8, force_partial=True)
    assert plan.unit_jobs is None and plan.n_separate == plan.combine.shape[0] == plan.n_units
    assert (plan.items[:, 4] >= 0).all()


def test_vectorized_tile_table_matches_the_per_sequence_walk():
    from asterq.plan import _tile_table, _tiles_of

    rng = np.random.default_rng(5)
    seqs = []
    for i in range(40):
        cold = [(int(rng.integers(0, 99)), int(rng.integers(0, 64)), int(rng.integers(1, 513))) for _ in range(rng.integers(0, 5))]
        hot = [(int(rng.integers(0, 99)), int(rng.integers(0, 64)), int(rng.integers(1, 600))) for _ in range(rng.integers(0, 4))]
        seqs.append(SequenceLayout(cold=cold, hot=hot, q_start=3 * i, q_len=int(rng.integers(1, 70)),
                                   attend_new=bool(rng.integers(0, 4))))
    for cold_tile in (COLD_TILE, COLD_TILE_INT8):
        tiles, off = _tile_table(seqs, cold_tile)
        want = []
        for k, seq in enumerate(seqs):
            mine = _tiles_of(seq, cold_tile)
            assert off[k + 1] - off[k] == len(mine)
            want.extend(mine)
        assert np.array_equal(tiles, np.asarray(want, dtype=np.int32).reshape(-1, 4))


def test_one_byte_schemes_plan_64_token_cold_tiles():
    """cold_tile=64 (int8 / float8 codes): every cold tile at most 64 tokens, each token once, and the
    same estimated time per full tile as a 128-token INT4 tile (an equal split of the work)."""
    seqs = [SequenceLayout(cold=[(0, 0, 512), (1, 0, 300)], hot=[(0, 0, 100)], q_start=0, q_len=1),
            SequenceLayout(cold=[(2, 0, 512)] * 6, hot=[(1, 0, 2048)], q_start=1, q_len=1)]
    p128 = build_plan(seqs, 16, n_sms=16)
    p64 = build_plan(seqs, 16, n_sms=16, cold_tile=COLD_TILE_INT8)
    assert p128.cold_tile == COLD_TILE and p64.cold_tile == COLD_TILE_INT8
    cold64 = p64.tiles[p64.tiles[:, 0] == _lib.TILE_COLD]
    cold128 = p128.tiles[p128.tiles[:, 0] == _lib.TILE_COLD]
    assert cold64[:, 3].max() == 64 and cold64[:, 3].sum() == cold128[:, 3].sum() == 512 + 300 + 6 * 512
    pages = [512, 300] + [512] * 6
    assert len(cold64) == sum(-(-n // 64) for n in pages) and len(cold128) == sum(-(-n // 128) for n in pages)
    with pytest.raises(ValueError, match="cold_tile"):
        build_plan(seqs, 16, cold_tile=32)
