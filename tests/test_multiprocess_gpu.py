"""The multi-GPU paths as separate processes, one per GPU, over NCCL.

* Context parallel (C4's partitioning): each rank builds the same sequence, runs
  ``ContextParallelDecoder.step`` (its chunk range into partial records, the rank-local merge,
  one ``all_gather_into_tensor`` over NCCL, the rank-major combine); every rank's output must
  match the single-GPU oracle decode and be identical across ranks.
* The same with the records exchanged by peer stores into CUDA IPC mailboxes instead of NCCL
  (``use_peer_exchange`` / ``step_peer``): repeated eager steps and CUDA-graph replays.
* Sequence sharding (C3/C5's partitioning): the batch is split with ``shard_sequences``, each
  rank builds only its own sequences from the shared seed and decodes them; every sequence is
  checked against the oracle on the rank that owns it, and the ranks together cover the batch.

Tolerance (north_star): rel-L2 <= 1e-3 and max-abs <= 2e-2, float32 output against the float32
oracle.  Needs two GPUs (skipped otherwise); the ranks are child processes started with
``spawn`` and their process group has a short timeout, so a rank that fails ends the others'
collectives with an error instead of a hang.
"""
from __future__ import annotations

import math
import os
import socket
import traceback

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)
WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _context_parallel_case(rank: int, world: int, dev, q_len: int) -> tuple[float, float, np.ndarray]:
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    ctx, hot = 20 * 512 + 300, 700
    inp = c1_inputs(seed=90 + q_len, ctx=ctx, q_len=q_len)
    b = PoolBuilder([ctx], [hot], q_len=q_len, n_heads=16, device=dev)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    dec = ContextParallelDecoder(wl.pools, wl.layouts[0], 16, rank, world, dev)
    out = torch.empty(q_len, 16, 512, dtype=torch.float32, device=dev)
    dec.step(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
    torch.cuda.synchronize(dev)
    dec.dplan.raise_if_failed()
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    got = out.cpu().numpy()
    return O.rel_l2(got, ref), O.max_abs(got, ref), got


def _peer_exchange_case(rank: int, world: int, dev, q_len: int) -> tuple[float, float, bool]:
    """The same sequence with records exchanged by peer stores (no NCCL in the step): four
    eager steps in a row (the mailboxes alternate record buffers) and three replays of the step
    captured as a CUDA graph, every one checked against the oracle and against the first."""
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    ctx, hot = 20 * 512 + 300, 700
    inp = c1_inputs(seed=90 + q_len, ctx=ctx, q_len=q_len)
    b = PoolBuilder([ctx], [hot], q_len=q_len, n_heads=16, device=dev)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    dec = ContextParallelDecoder(wl.pools, wl.layouts[0], 16, rank, world, dev)
    ex = dec.use_peer_exchange(wait_limit_cycles=4_000_000_000)
    try:
        out = torch.empty(q_len, 16, 512, dtype=torch.float32, device=dev)
        outs = []
        for _ in range(4):
            dec.step_peer(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
            outs.append(out.clone())
        graph = dec.capture_peer(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
        for _ in range(3):
            out.fill_(float("nan"))
            graph.replay()
            outs.append(out.clone())
        torch.cuda.synchronize(dev)
        ex.raise_if_failed()
        dec.dplan.raise_if_failed()
        del graph
    finally:
        ex.close()
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    got = outs[0].cpu().numpy()
    same = all(torch.equal(o, outs[0]) for o in outs)
    return O.rel_l2(got, ref), O.max_abs(got, ref), same


def _sharded_case(rank: int, world: int, dev) -> list[tuple[int, float, float]]:
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.sharding import shard_sequences
    from asterq.synth import make_shard_workload

    lens = [1500, 9000, 3100, 600, 5200, 2047]
    hot = [min(n, 2048) for n in lens]
    shard = shard_sequences(lens, hot, world)[rank]
    wl = make_shard_workload("shard", lens, hot, shard, q_len=1, n_heads=16, seed=21, device=dev,
                             keep_host=set(shard))
    dplan = DeviceDecodePlan(build_plan(wl.layouts, wl.n_heads), dev)
    out = latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                        out_dtype=torch.float32)
    torch.cuda.synchronize(dev)
    dplan.raise_if_failed()
    got = out.cpu().numpy()
    res = []
    for k, gi in enumerate(shard):
        h = wl.host[k]
        want = O.decode_sequence(h["latent"].float().numpy(), h["rope"].float().numpy(), h["q_lat"].float().numpy(),
                                 h["q_rope"].float().numpy(), lens[gi], hot[gi], SCALE)
        res.append((gi, O.rel_l2(got[k : k + 1], want), O.max_abs(got[k : k + 1], want)))
    return res


def _rank_main(rank: int, world: int, port: int, result_q) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        try:
            cp = {}
            for q_len in (1, 3):
                rel, mab, got = _context_parallel_case(rank, world, dev, q_len)
                # every rank combined the same gathered records: identical outputs
                t = torch.from_numpy(got).to(dev)
                peers = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(peers, t)
                same = all(torch.equal(p, t) for p in peers)
                cp[q_len] = (rel, mab, same)
            peer = {q_len: _peer_exchange_case(rank, world, dev, q_len) for q_len in (1, 3)}
            shard = _sharded_case(rank, world, dev)
            dist.barrier()
        finally:
            dist.destroy_process_group()
        result_q.put((rank, "ok", (cp, peer), shard))
    except Exception:
        result_q.put((rank, "error", traceback.format_exc(), None))


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_two_ranks_over_nccl_match_the_oracle():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(WORLD):
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    errors = [r[2] for r in results if r[1] != "ok"]
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs)
    covered = []
    for rank, _, (cp, peer), shard in sorted(results, key=lambda r: r[0]):
        for q_len, (rel, mab, same) in cp.items():
            assert rel <= 1e-3 and mab <= 2e-2, f"context parallel rank {rank} q_len {q_len}: {rel:.3e} {mab:.3e}"
            assert same, f"rank {rank}: the ranks' combined outputs differ"
        for q_len, (rel, mab, same) in peer.items():
            assert rel <= 1e-3 and mab <= 2e-2, f"peer exchange rank {rank} q_len {q_len}: {rel:.3e} {mab:.3e}"
            assert same, f"peer exchange rank {rank} q_len {q_len}: steps or graph replays differ"
        for gi, rel, mab in shard:
            assert rel <= 1e-3 and mab <= 2e-2, f"sharded seq {gi} on rank {rank}: {rel:.3e} {mab:.3e}"
            covered.append(gi)
    assert sorted(covered) == list(range(6))
