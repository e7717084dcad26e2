"""Split-KV schedule for the ragged / paged decode batch.

A batch is a list of sequences, each with its cold chunks (pages of INT4
codes), its hot pages (BF16) and ``q_len`` new tokens.  The reference walks one
sequence's chunks serially (cache.py:139-159, latent_attention.py:222-227);
here every sequence's token list is cut into tiles (128 cold tokens or 32 hot /
new tokens).  The default (persistent) schedule gives every SM one worker CTA
and cuts the concatenated tile lists of all 16-row query blocks into one
contiguous share per worker of equal estimated time (measured per-tile costs
plus a fixed cost per item); a worker runs its items one after another, so a
ragged batch ends on all SMs at about the same time.  Items that do not cover
a whole query block write partial (m, l, o) records merged by the combine step.

Tables (int32, see include/asterq.h):
  tiles   [n_tiles, 4]  {kind, page, offset, n_tokens}
  items   [n_items, 8]  {unit, row_block, tile_begin, tile_end, slot, out_row0, n_rows, q_len}
  combine [n_combine, 4] {slot_begin, slot_end, out_row0, n_rows}
  workers [n_workers + 1] item offsets: worker w runs items workers[w] .. workers[w + 1] - 1
"""
from __future__ import annotations

import bisect
import heapq
from dataclasses import dataclass, field

import numpy as np

from . import _lib

COLD_TILE = 128
COLD_TILE_INT8 = 64  # int8 codes: a 64-token cold tile holds the code bytes of a 128-token INT4 tile
HOT_TILE = 32
ROWS_PER_BLOCK = 16
MAX_Q_LEN = 2048  # new tokens per sequence and step (the reference prefills in chunks of 2048)

# bytes one tile streams from HBM (cost model for balancing)
_COLD_TOKEN_BYTES = 256 + 16 + 128
_HOT_TOKEN_BYTES = 1024 + 128
_ITEM_OVERHEAD_BYTES = 48 * 1024  # query load + rotation + output/partial write

# time model of the persistent schedule (ns, one B200 SM; least-squares fit to the measured end
# times of every worker of the C3 batch and of one C5 shard under five schedules, rms 4 us):
# a full cold tile 2.75 us, a full hot tile 1.66 us, an item's fixed cost (query copy, barrier
# reset, output write) 1.8 us, and 5.7 us more for a piece of a cut block (its partial record
# written and, for one piece per block, the merge of the block's records)
_COLD_TILE_NS = (1000, 1750)  # fixed + per full tile
_HOT_TILE_NS = (560, 1100)
_ITEM_NS = 1800
_PIECE_NS = 5700
_MIN_PIECE_NS = 4 * sum(_COLD_TILE_NS)  # a worker does not start a piece of a block below this
# a block cut into at most this many pieces is merged by the decode kernel itself (the CTA
# that writes the last piece reads them all back from L2); more pieces go to the combine launch
# (measured: a 9-piece merge inside the kernel saves ~2 us, a 20-piece one costs ~6 us)
FUSED_COMBINE_MAX_PARTS = 16


@dataclass
class SequenceLayout:
    """Where one sequence's cache lives and where its new tokens sit.

    ``cold``: (page, offset, n_tokens) chunks, oldest first.
    ``hot``: (page, offset, n_tokens) runs of the hot window, oldest first.
    ``q_start``: index of the first new token in the batch's q / new-token arrays.
    """

    cold: list[tuple[int, int, int]] = field(default_factory=list)
    hot: list[tuple[int, int, int]] = field(default_factory=list)
    q_start: int = 0
    q_len: int = 1
    attend_new: bool = True  # False: the query rows attend to the cache only (a context-parallel rank without them)

    @property
    def cold_tokens(self) -> int:
        return sum(n for _, _, n in self.cold)

    @property
    def hot_tokens(self) -> int:
        return sum(n for _, _, n in self.hot)

    @property
    def cache_bytes(self) -> int:
        return self.cold_tokens * _COLD_TOKEN_BYTES + (self.hot_tokens + self.q_len * self.attend_new) * _HOT_TOKEN_BYTES


QPREP_BYTES = 37376  # prepared query operands of one 16-row block (int8 limbs, bf16 fragments, scalars,
                     # int8 limbs of the RoPE query for quantized cold RoPE keys)


@dataclass
class DecodePlan:
    tiles: np.ndarray
    items: np.ndarray
    combine: np.ndarray
    n_slots: int
    total_q: int
    n_heads: int
    units: np.ndarray = field(default_factory=lambda: np.zeros((0, 2), np.int32))  # [n_units][2] {out_row0, n_rows}
    workers: np.ndarray | None = None  # [n_workers + 1] item offsets, or None: one CTA per item
    # combine jobs [0, n_separate_combine) run in the combine launch; the others are run by
    # the decode kernel itself (unit_jobs[u] = the unit's job, or -1)
    n_separate_combine: int | None = None
    unit_jobs: np.ndarray | None = None
    cold_tile: int = COLD_TILE  # tokens of a cold tile (COLD_TILE_INT8 for int8 codes)

    @property
    def n_workers(self) -> int:
        return 0 if self.workers is None else int(self.workers.shape[0]) - 1

    @property
    def n_units(self) -> int:
        return int(self.units.shape[0])

    @property
    def n_separate(self) -> int:
        return int(self.combine.shape[0]) if self.n_separate_combine is None else self.n_separate_combine

    @property
    def workspace_bytes(self) -> int:
        counters = (self.n_units * 4 + 15) // 16 * 16  # one int32 per unit (fused combine jobs)
        return self.n_slots * ROWS_PER_BLOCK * (512 + 2) * 4 + self.n_units * QPREP_BYTES + counters


def _tiles_of(seq: SequenceLayout, cold_tile: int = COLD_TILE) -> list[tuple[int, int, int, int]]:
    out = []
    for page, off, n in seq.cold:
        for s in range(0, n, cold_tile):
            out.append((_lib.TILE_COLD, page, off + s, min(cold_tile, n - s)))
    for page, off, n in seq.hot:
        for s in range(0, n, HOT_TILE):
            out.append((_lib.TILE_HOT, page, off + s, min(HOT_TILE, n - s)))
    if seq.q_len > 0 and seq.attend_new:
        for s in range(0, seq.q_len, HOT_TILE):
            out.append((_lib.TILE_NEW, seq.q_start, s, min(HOT_TILE, seq.q_len - s)))
    return out


def _tile_table(seqs: list[SequenceLayout], cold_tile: int = COLD_TILE) -> tuple[np.ndarray, np.ndarray]:
    """All sequences' tiles at once (numpy, no per-tile Python): [n_tiles, 4] int32 in the
    order of _tiles_of per sequence, and [n_seqs + 1] offsets of each sequence's tiles."""
    rows, seg_kind, seg_len, per_seq = [], [], [], []
    cold_k, hot_k, new_k = _lib.TILE_COLD, _lib.TILE_HOT, _lib.TILE_NEW
    for seq in seqs:
        r0 = len(rows)
        rows.extend(seq.cold)
        rows.extend(seq.hot)
        seg_kind += [cold_k, hot_k]
        seg_len += [len(seq.cold), len(seq.hot)]
        if seq.q_len > 0 and seq.attend_new:  # the new tokens: "page" = first row in the batch
            rows.append((seq.q_start, 0, seq.q_len))
            seg_kind.append(new_k)
            seg_len.append(1)
        per_seq.append(len(rows) - r0)
    A = np.asarray(rows, dtype=np.int64).reshape(-1, 3)
    K = np.repeat(np.asarray(seg_kind, dtype=np.int64), np.asarray(seg_len, dtype=np.int64))
    Pg, Of, N = A[:, 0], A[:, 1], A[:, 2]
    bad = (N <= 0) | (Of < 0) | (Pg < 0)
    if bad.any():
        i = int(np.argmax(bad))
        raise ValueError(f"bad chunk (page={int(Pg[i])}, offset={int(Of[i])}, n={int(N[i])})")
    T = np.where(K == cold_k, cold_tile, HOT_TILE)
    cnt = (N + T - 1) // T
    rep = np.repeat(np.arange(K.shape[0]), cnt)
    first = np.cumsum(cnt) - cnt
    j = np.arange(int(cnt.sum())) - first[rep]
    Tr = T[rep]
    tiles = np.stack([K[rep], Pg[rep], Of[rep] + j * Tr, np.minimum(Tr, N[rep] - j * Tr)], axis=1).astype(np.int32)
    chunk_off = np.concatenate(([0], np.cumsum(per_seq)))
    tile_off = np.concatenate(([0], np.cumsum(cnt)))[chunk_off]
    return tiles.reshape(-1, 4), tile_off


def _tile_costs(tiles: np.ndarray, cold_tile: int = COLD_TILE) -> tuple[np.ndarray, np.ndarray]:
    """Per-tile bytes (cost model of the one-CTA-per-item schedule) and estimated ns.  A full
    cold tile has the same estimated time for either tile size (the same code bytes and MMAs)."""
    cold = tiles[:, 0] == _lib.TILE_COLD
    n = tiles[:, 3].astype(np.int64)
    n_cold = n * (COLD_TILE // cold_tile)  # in INT4-tile token units
    nbytes = np.where(cold, n_cold * _COLD_TOKEN_BYTES, n * _HOT_TOKEN_BYTES)
    ns = np.where(cold, _COLD_TILE_NS[0] + (_COLD_TILE_NS[1] * n) // cold_tile,
                  _HOT_TILE_NS[0] + (_HOT_TILE_NS[1] * n) // HOT_TILE)
    return nbytes.astype(np.int64), ns.astype(np.int64)


def _visible_tiles(seq: SequenceLayout, t0: int, t1: int, rb: int, n_heads: int) -> int:
    """End of the tiles row block `rb` can see: new-token tiles wholly after its last
    token are fully masked (k <= past_len + i, latent_attention.py:151-153) and dropped."""
    if not (seq.q_len > 0 and seq.attend_new):
        return t1
    n_new = (seq.q_len + HOT_TILE - 1) // HOT_TILE
    last_row = min(seq.q_len * n_heads, (rb + 1) * ROWS_PER_BLOCK) - 1
    last_token = last_row // n_heads
    return t1 - n_new + last_token // HOT_TILE + 1


def _tile_cost(kind: int, n: int) -> int:
    return n * (_COLD_TOKEN_BYTES if kind == _lib.TILE_COLD else _HOT_TOKEN_BYTES)


def _tile_ns(kind: int, n: int) -> int:
    if kind == _lib.TILE_COLD:
        return _COLD_TILE_NS[0] + (_COLD_TILE_NS[1] * n) // COLD_TILE
    return _HOT_TILE_NS[0] + (_HOT_TILE_NS[1] * n) // HOT_TILE


def _greedy_cut(units, P, T: int, limit: int, min_piece: int = _MIN_PIECE_NS):
    """Fill workers in order with contiguous pieces of the units' tile ranges, each
    worker up to T ns (an item costs _ITEM_NS on top of its tiles).  A unit is cut
    only into pieces of at least `min_piece` ns.  Returns the pieces
    [(unit, a, b, worker)] or None when more than `limit` workers are needed."""
    pieces = []
    w, load = 0, 0

    def next_worker():
        nonlocal w, load
        w, load = w + 1, 0
        return w < limit

    for ui, t0, t1 in units:
        a = t0
        while a < t1:
            rest = P[t1] - P[a]
            fixed = _ITEM_NS + (_PIECE_NS if a > t0 else 0)  # the tail of a cut block is a piece too
            room = T - load - fixed
            if rest <= room or (rest < 2 * min_piece and load == 0):
                pieces.append((ui, a, t1, w))  # the rest fits, or cannot be cut and the worker is empty
                load += fixed + rest
                break
            room = T - load - _ITEM_NS - _PIECE_NS  # this item becomes a piece of a cut block
            if rest < 2 * min_piece or room < min_piece:
                if load > 0:
                    if not next_worker():
                        return None
                    continue
                room = min_piece
            b = bisect.bisect_right(P, P[a] + room, a + 1, t1 + 1) - 1
            if P[t1] - P[b] < min_piece:  # leave the next worker a piece of useful size
                b = bisect.bisect_right(P, P[t1] - min_piece, a + 1, t1 + 1) - 1
            b = min(max(b, a + 1), t1)
            pieces.append((ui, a, b, w))
            load += _ITEM_NS + _PIECE_NS + P[b] - P[a]
            a = b
            if a < t1 and not next_worker():
                return None
    return pieces


def _balanced_cut(units, P, n_workers: int):
    """Smallest per-worker time T (binary search) for which the greedy cut fits."""
    total = int(sum(P[t1] - P[t0] for _, t0, t1 in units)) + _ITEM_NS * len(units)
    longest_tile = int(np.diff(np.asarray(P)).max()) if len(P) > 1 else 0
    lo = max(total // n_workers, _ITEM_NS + longest_tile) - 1
    hi = total + (_ITEM_NS + _PIECE_NS) * (n_workers + len(units)) + int(P[-1])
    # a small batch (little work per SM) cuts its blocks finer, down to one full cold tile of
    # work per piece (one 8k-token sequence: 31.8 -> 28.0 us a step)
    min_piece = max(sum(_COLD_TILE_NS), min(_MIN_PIECE_NS, total // n_workers))
    best = _greedy_cut(units, P, hi, n_workers, min_piece)
    while hi - lo > 1000:  # 1 us resolution
        mid = (lo + hi) // 2
        got = _greedy_cut(units, P, mid, n_workers, min_piece)
        if got is None:
            lo = mid
        else:
            hi, best = mid, got
    return best


def build_plan(
    seqs: list[SequenceLayout],
    n_heads: int,
    *,
    n_sms: int = 148,
    ctas_per_sm: int = 1,
    waves: float = 3.0,
    max_items_per_seq: int | None = None,
    force_partial: bool = False,
    persistent: bool = True,
    cold_tile: int = COLD_TILE,
) -> DecodePlan:
    """Cut the batch into balanced work items.

    ``persistent`` (default): ``n_sms * ctas_per_sm`` workers, each a contiguous share
    of the query blocks' tiles of equal estimated time (``waves`` is not used); with
    ``max_items_per_seq`` the blocks are first cut as below and the items dealt to the
    workers longest first.  ``persistent=False``: one CTA per item, about
    ``waves`` items per SM, longest first.
    ``force_partial``: every (sequence, row block) writes partial records and gets
    a combine job, even when one item covers it (context-parallel decode merges
    these records across ranks).
    ``cold_tile``: tokens of a cold tile, ``COLD_TILE`` for the INT4 schemes and
    ``COLD_TILE_INT8`` for int8 codes (the decode call checks it against the scheme).
    """
    if cold_tile not in (COLD_TILE, COLD_TILE_INT8):
        raise ValueError(f"cold_tile must be {COLD_TILE} or {COLD_TILE_INT8}")
    if n_heads <= 0:
        raise ValueError("n_heads must be positive")
    total_q = 0
    for seq in seqs:
        if not (0 < seq.q_len <= MAX_Q_LEN):
            raise ValueError(f"q_len must be in 1..{MAX_Q_LEN} (got {seq.q_len})")
        total_q = max(total_q, seq.q_start + seq.q_len)
    tile_arr, tile_off = _tile_table(seqs, cold_tile)
    seq_tile_ranges = [(int(a), int(b)) for a, b in zip(tile_off[:-1], tile_off[1:])]
    costs, tile_ns = _tile_costs(tile_arr, cold_tile)
    prefix = np.concatenate(([0], np.cumsum(costs)))

    # work units: (seq, row_block)
    units = []
    total_cost = 0
    for si, seq in enumerate(seqs):
        rows = seq.q_len * n_heads
        t0, t1s = seq_tile_ranges[si]
        for rb in range((rows + ROWS_PER_BLOCK - 1) // ROWS_PER_BLOCK):
            t1 = _visible_tiles(seq, t0, t1s, rb, n_heads)
            c = int(prefix[t1] - prefix[t0])
            units.append((si, rb, t0, t1, c))
            total_cost += c
    n_workers = max(1, int(n_sms * ctas_per_sm))
    unit_rows = []
    for si, rb, t0, t1, c in units:
        seq = seqs[si]
        rows = seq.q_len * n_heads
        unit_rows.append((seq.q_start * n_heads + rb * ROWS_PER_BLOCK, min(ROWS_PER_BLOCK, rows - rb * ROWS_PER_BLOCK)))
    unit_arr = np.asarray(unit_rows, dtype=np.int32).reshape(-1, 2)

    if persistent and max_items_per_seq is None:
        P = np.concatenate(([0], np.cumsum(tile_ns))).tolist()
        work = [(ui, t0, t1) for ui, (_, _, t0, t1, _) in enumerate(units) if t1 > t0]
        pieces = _balanced_cut(work, P, n_workers) if work else []
        by_unit: dict[int, list] = {}
        for ui, a, b, w in pieces:
            by_unit.setdefault(ui, []).append((a, b, w))
        items, separate, fused, n_slots = [], [], [], 0
        for ui, (si, rb, t0, t1, c) in enumerate(units):
            out_row0, n_rows = unit_rows[ui]
            q_len = seqs[si].q_len
            segs = by_unit.get(ui, [(t0, t1, 0)])  # a block with no visible tile: one empty item
            if len(segs) == 1 and not force_partial:
                a, b, w = segs[0]
                items.append((w, a, (ui, rb, a, b, -1, out_row0, n_rows, q_len)))
                continue
            s0 = n_slots
            for a, b, w in segs:
                items.append((w, a, (ui, rb, a, b, n_slots, out_row0, n_rows, q_len)))
                n_slots += 1
            job = (s0, n_slots, out_row0, n_rows)
            if not force_partial and len(segs) <= FUSED_COMBINE_MAX_PARTS:
                fused.append((ui, job))
            else:
                separate.append(job)
        combine = separate + [job for _, job in fused]
        unit_jobs = np.full(len(units), -1, dtype=np.int32)
        for k, (ui, _) in enumerate(fused):
            unit_jobs[ui] = len(separate) + k
        # a worker runs its pieces of cut blocks before its whole blocks, so that the last
        # piece of a block (whose CTA then merges the block) rarely ends with the kernel
        items.sort(key=lambda x: (x[0], x[2][4] < 0, x[1]))
        item_arr = np.asarray([it[2] for it in items], dtype=np.int32).reshape(-1, 8)
        used = max((it[0] for it in items), default=-1) + 1
        counts = np.bincount(np.asarray([it[0] for it in items], dtype=np.int64), minlength=used)
        workers = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
        comb_arr = np.asarray(combine, dtype=np.int32).reshape(-1, 4)
        return DecodePlan(tile_arr, item_arr, comb_arr, n_slots, total_q, n_heads, unit_arr, workers,
                          n_separate_combine=len(separate), unit_jobs=unit_jobs if fused else None,
                          cold_tile=cold_tile)

    slots_target = max(1, int(n_sms * ctas_per_sm * waves))
    item_cost = max(total_cost / slots_target, 4 * COLD_TILE * _COLD_TOKEN_BYTES)

    items = []
    combine = []
    n_slots = 0
    for ui, (si, rb, t0, t1, c) in enumerate(units):
        seq = seqs[si]
        out_row0, n_rows = unit_rows[ui]
        k = max(1, int(np.ceil((c + _ITEM_OVERHEAD_BYTES) / (item_cost + _ITEM_OVERHEAD_BYTES))))
        # one row block never needs more items than can run at once
        k = min(k, t1 - t0, max(1, int(n_sms * ctas_per_sm)))
        if max_items_per_seq is not None:
            k = min(k, max_items_per_seq)
        if k <= 1 and not force_partial:
            items.append((ui, rb, t0, t1, -1, out_row0, n_rows, seq.q_len, c))
            continue
        k = max(k, 1)
        # contiguous ranges of ~equal cost
        targets = prefix[t0] + (c * np.arange(1, k)) / k
        cuts = np.searchsorted(prefix[t0 : t1 + 1], targets, side="left") + t0
        bounds = [t0] + sorted(set(int(x) for x in cuts if t0 < x < t1)) + [t1]
        s0 = n_slots
        for a, b in zip(bounds[:-1], bounds[1:]):
            items.append((ui, rb, a, b, n_slots, out_row0, n_rows, seq.q_len, int(prefix[b] - prefix[a])))
            n_slots += 1
        combine.append((s0, n_slots, out_row0, n_rows))

    items.sort(key=lambda it: -it[8])
    item_arr = np.asarray([it[:8] for it in items], dtype=np.int32).reshape(-1, 8)
    comb_arr = np.asarray(combine, dtype=np.int32).reshape(-1, 4)
    if not persistent or not items:
        return DecodePlan(tile_arr, item_arr, comb_arr, n_slots, total_q, n_heads, unit_arr, cold_tile=cold_tile)
    # deal the items (longest first) to the least loaded of the workers
    P = np.concatenate(([0], np.cumsum(tile_ns)))
    heap = [(0, w) for w in range(min(n_workers, len(items)))]
    owner = []
    for it in item_arr:
        load, w = heapq.heappop(heap)
        owner.append(w)
        heapq.heappush(heap, (load + _ITEM_NS + int(P[it[3]] - P[it[2]]), w))
    order = np.argsort(np.asarray(owner), kind="stable")
    item_arr = item_arr[order]
    counts = np.bincount(np.asarray(owner), minlength=len(heap))
    workers = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
    return DecodePlan(tile_arr, item_arr, comb_arr, n_slots, total_q, n_heads, unit_arr, workers, cold_tile=cold_tile)
