"""Multi-GPU host logic on CPU: sequence sharding and context-parallel partitioning.

World-size-2 process groups on the gloo backend run the same partition and
gather steps the GPU ranks run over NCCL; the per-rank attention state comes
from the oracle, so the check is that the partition covers every key once and
that merging the gathered states reproduces the single-rank decode.
"""
from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import hq4_oracle as O

SCALE = 1.0 / math.sqrt(512 + 64)


def test_lpt_shard_balances_and_covers():
    from asterq.sharding import lpt_shard, shard_sequences
    from asterq.synth import c3_lengths

    lens = c3_lengths(0, 64)
    hot = [min(n, 2048) for n in lens]
    for world in (1, 2, 4, 8):
        parts = shard_sequences(lens, hot, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        from asterq.sharding import step_bytes

        loads = [sum(step_bytes(lens[i], hot[i]) for i in p) for p in parts]
        biggest = max(step_bytes(n, h) for n, h in zip(lens, hot))
        assert max(loads) - min(loads) <= biggest
    assert lpt_shard([5, 5, 5], 2) == [[0, 2], [1]]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_split_chunks_cover_contiguously(world):
    from asterq.context_parallel import rank_layout, split_chunks
    from asterq.plan import SequenceLayout

    chunks = [512] * 248
    ranges = split_chunks(chunks, 4096, world)
    assert ranges[0][0] == 0 and ranges[-1][1] == 248
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    lay = SequenceLayout(cold=[(p, 0, 512) for p in range(248)], hot=[(0, 0, 512)] * 8, q_start=0, q_len=1)
    parts = [rank_layout(lay, r, world) for r in range(world)]
    assert sum(len(p.cold) for p in parts) == 248
    assert [p.attend_new for p in parts] == [False] * (world - 1) + [True]
    assert sum(p.hot_tokens for p in parts) == 4096
    if world > 1:
        costs = [p.cache_bytes for p in parts]
        assert max(costs) - min(costs) <= 2 * 512 * 400 + 4096 * 1152 / world


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_rank(rank: int, world: int, port: int, result_q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from asterq.context_parallel import split_chunks

        rng = np.random.default_rng(0)
        chunk, n_chunks, hot = 64, 9, 100
        lat = O.round_bf16(rng.standard_normal((n_chunks * chunk + hot + 1, 512)).astype(np.float32))
        rope = O.round_bf16(rng.standard_normal((n_chunks * chunk + hot + 1, 64)).astype(np.float32))
        q = O.round_bf16(rng.standard_normal((1, 16, 512)).astype(np.float32))
        qr = O.round_bf16(rng.standard_normal((1, 16, 64)).astype(np.float32))
        cache = O.build_cache_split(lat[:-1], rope[:-1], hot, chunk)
        ranges = split_chunks([c.length for c in cache.cold], hot, world)
        a, b = ranges[rank]
        mine = [(c.dequantized_latent(), c.rope) for c in cache.cold[a:b]]
        if rank == world - 1:
            mine += [(cache.hot_latent, cache.hot_rope), (lat[-1:], rope[-1:])]
        m, l, o = O.partial_attention(q, qr, mine, SCALE)
        rec = torch.from_numpy(np.concatenate([o.ravel(), m.ravel(), l.ravel()]).astype(np.float32))
        gathered = [torch.empty_like(rec) for _ in range(world)]
        dist.all_gather(gathered, rec)
        n_o = o.size
        parts = [(g[n_o: n_o + m.size].numpy().reshape(m.shape), g[n_o + m.size:].numpy().reshape(l.shape),
                  g[:n_o].numpy().reshape(o.shape)) for g in gathered]
        merged = O.merge_partials(parts)
        full = O.decode(q, qr, lat[-1:], rope[-1:], cache, SCALE)
        result_q.put((rank, O.rel_l2(merged, full), O.max_abs(merged, full)))
    finally:
        dist.destroy_process_group()


def test_context_parallel_gloo_world2_matches_single_rank():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cp_rank, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=180)
    results = sorted(q.get(timeout=5) for _ in range(world))
    assert all(pr.exitcode == 0 for pr in procs)
    for rank, rel, mab in results:
        assert rel < 1e-5 and mab < 1e-4, (rank, rel, mab)
