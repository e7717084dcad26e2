"""Context-parallel decode on one GPU with the ranks emulated in turn.

Each emulated rank decodes its chunk range into partial records, merges them
with ``asterq_splitkv_merge``, and the records are concatenated rank-major as
``all_gather_into_tensor`` would leave them; ``finish`` (which combines them in
place with ``asterq_splitkv_combine_ranks``) must reproduce the single-GPU
oracle decode (rel-L2 <= 1e-3, max-abs <= 2e-2, fp32 output), with one or
several 16-row blocks per rank (q_len 1 to 3).  Decode and context-parallel
steps recorded as CUDA graphs must replay to the eager result.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)


@pytest.mark.parametrize("world,q_len,n_chunks",
                         [(1, 1, 20), (2, 1, 20), (3, 1, 20), (8, 1, 20), (3, 2, 20), (2, 3, 20), (8, 2, 3)])
def test_emulated_ranks_match_oracle(cuda, world, q_len, n_chunks):
    """(8, 2, 3): more ranks than cold chunks, so some ranks read nothing and send empty records."""
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    ctx, hot = n_chunks * 512 + 300, 700
    inp = c1_inputs(seed=40 + world, ctx=ctx, q_len=q_len)
    b = PoolBuilder([ctx], [hot], q_len=q_len, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    decs = [ContextParallelDecoder(wl.pools, wl.layouts[0], 16, r, world, cuda) for r in range(world)]
    recs = [d.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE).clone() for d in decs]
    out = torch.empty(q_len, 16, 512, dtype=torch.float32, device=cuda)
    decs[0].finish(torch.cat(recs), out)
    torch.cuda.synchronize()
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    got = out.cpu().numpy()
    assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2
    # every rank, not only rank 0, finishes to the same result
    out2 = torch.empty_like(out)
    decs[-1].finish(torch.cat(recs), out2)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("scheme,qrope", [("int8", False), ("float8", True), ("int4", True)])
def test_emulated_ranks_other_cache_schemes(cuda, scheme, qrope):
    """Context-parallel decode of a sequence stored with the other cache schemes: each rank's plan
    cuts its cold pages into the scheme's tiles (64 tokens for int8 / float8)."""
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    world, ctx, hot = 3, 9 * 512 + 200, 600
    inp = c1_inputs(seed=77, ctx=ctx, q_len=1)
    b = PoolBuilder([ctx], [hot], q_len=1, n_heads=16, device=cuda, scheme=scheme, quantize_rope=qrope)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    decs = [ContextParallelDecoder(wl.pools, wl.layouts[0], 16, r, world, cuda) for r in range(world)]
    recs = [d.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE).clone() for d in decs]
    out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)
    decs[1].finish(torch.cat(recs), out)
    torch.cuda.synchronize()
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512, scheme=scheme, quantize_rope=qrope)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    got = out.cpu().numpy()
    assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2


def test_merge_then_combine_equals_direct_combine(cuda):
    from asterq import _lib
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import PoolBuilder, c1_inputs

    ctx = 9000
    inp = c1_inputs(seed=77, ctx=ctx, q_len=1)
    b = PoolBuilder([ctx], [1000], q_len=1, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("m")
    plan = build_plan(wl.layouts, 16, n_sms=64, ctas_per_sm=4, waves=4)
    assert plan.n_slots > 2
    dp = DeviceDecodePlan(plan, cuda)
    direct = latent_decode(wl.pools, dp, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                           out_dtype=torch.float32)
    merged = torch.empty(16 * 514, dtype=torch.float32, device=cuda)
    lib = _lib.load()
    _lib.check(lib.asterq_splitkv_merge(dp.workspace.data_ptr(), plan.n_slots, dp.combine.data_ptr(), 1, 512,
                                        merged.data_ptr(), _lib.stream_handle(cuda)))
    jobs = torch.tensor([[0, 1, 0, 16]], dtype=torch.int32, device=cuda)
    out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)
    _lib.check(lib.asterq_splitkv_combine(merged.data_ptr(), 1, jobs.data_ptr(), 1, 512, out.data_ptr(),
                                          _lib.DTYPE_F32, _lib.stream_handle(cuda)))
    torch.cuda.synchronize()
    assert O.rel_l2(out.cpu().numpy(), direct.cpu().numpy()) < 1e-6


def test_decode_step_replays_as_cuda_graph(cuda):
    """A decode step recorded by ``capture_step`` replays to the eager step's exact output."""
    from asterq.decode import DeviceDecodePlan, capture_step, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import PoolBuilder, c1_inputs

    ctx = 6 * 512 + 200
    inp = c1_inputs(seed=91, ctx=ctx, q_len=1)
    b = PoolBuilder([ctx], [700], q_len=1, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("g")
    dp = DeviceDecodePlan(build_plan(wl.layouts, 16), cuda)
    out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)

    def step():
        latent_decode(wl.pools, dp, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE, out=out)

    step()
    eager = out.clone()
    graph = capture_step(step, cuda)
    out.zero_()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del graph


def test_context_parallel_step_replays_as_cuda_graph(cuda):
    """The context-parallel step (decode, merge, NCCL all-gather, combine) captured at world size 1."""
    import torch.distributed as dist

    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    if dist.is_initialized():
        pytest.skip("a process group is already initialised in this process")
    ctx, hot = 12 * 512 + 100, 600
    inp = c1_inputs(seed=92, ctx=ctx, q_len=1)
    b = PoolBuilder([ctx], [hot], q_len=1, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cpg")
    dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1, device_id=cuda)
    try:
        dec = ContextParallelDecoder(wl.pools, wl.layouts[0], 16, 0, 1, cuda)
        out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)
        dec.step(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
        eager = out.clone()
        graph = dec.capture(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        del graph
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    got = eager.cpu().numpy()
    assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2


def _cp_gloo_rank(rank: int, world: int, port: int, result_q) -> None:
    """One process of a context-parallel step: the product's partial records on the GPU, a real
    all-gather over the process group (gloo, through host copies), the product's combine."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from asterq.context_parallel import ContextParallelDecoder
        from asterq.synth import PoolBuilder, c1_inputs

        dev = torch.device("cuda:0")
        ctx, hot = 20 * 512 + 300, 700
        inp = c1_inputs(seed=60, ctx=ctx, q_len=1)  # CPU generator: the same tensors on every rank
        b = PoolBuilder([ctx], [hot], q_len=1, n_heads=16, device=dev)
        b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
        wl = b.finish("cp")
        dec = ContextParallelDecoder(wl.pools, wl.layouts[0], 16, rank, world, dev)
        rec = dec.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE).cpu()
        gathered = torch.empty(world * rec.numel(), dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, rec)
        out = torch.empty(1, 16, 512, dtype=torch.float32, device=dev)
        dec.finish(gathered.to(dev), out)
        torch.cuda.synchronize()
        result_q.put((rank, out.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_context_parallel_processes_exchange_records(cuda, world):
    """`world` processes (one GPU, kernels that never wait on one another) each decode their chunk
    range, exchange the merged records with a real collective and combine: every rank's output
    matches the single-process oracle decode."""
    import multiprocessing as mp
    import socket

    from asterq.synth import c1_inputs

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cp_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for pr in procs:
        pr.join(timeout=120)
    assert all(pr.exitcode == 0 for pr in procs)
    c, hot = 20 * 512 + 300, 700
    inp = c1_inputs(seed=60, ctx=c, q_len=1)
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:c], rope[:c], hot, 512)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[c:], rope[c:], cache, SCALE)
    for r in range(world):
        got = results[r][0:1]
        assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2, r
        assert np.array_equal(results[r], results[0])


def test_peer_exchange_wait_times_out_without_a_fault(cuda):
    """Failure detection for the peer exchange, without a fault: one process, a mailbox sized for
    two ranks whose second rank never stores its records (a flag that nothing sets).  The
    combine's wait runs into a short cycle limit, sets the status word, leaves the output
    unwritten and returns; the context stays usable."""
    import ctypes

    from asterq import _lib
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    ctx, hot = 6 * 512 + 100, 300
    inp = c1_inputs(seed=61, ctx=ctx)
    b = PoolBuilder([ctx], [hot], q_len=1, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    dec = ContextParallelDecoder(wl.pools, wl.layouts[0], 16, 0, 2, cuda)  # rank 0 of 2
    lib = _lib.load()
    nbytes = lib.asterq_mailbox_bytes(2, dec.n_rb, 512)
    own = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
    _lib.check(lib.asterq_mailbox_create(nbytes, ctypes.byref(own), handle))
    try:
        table = torch.tensor([own.value, own.value], dtype=torch.int64, device=cuda)  # rank 1's slot: never written
        status = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = torch.full((1, 16, 512), float("nan"), dtype=torch.float32, device=cuda)
        stream = dec._decode_records(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE)
        _lib.check(lib.asterq_cp_merge_push(dec.dplan.workspace.data_ptr(), dec.plan.n_slots, dec.dplan.combine.data_ptr(),
                                            dec.n_rb, 512, table.data_ptr(), 2, 0, stream))
        _lib.check(lib.asterq_cp_combine_wait(own.value, 2, dec.n_rb, dec.final_jobs.data_ptr(), 512, out.data_ptr(),
                                              _lib.DTYPE_F32, 2_000_000, status.data_ptr(), stream))
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        assert torch.isnan(out).all()  # nothing was combined
        # the context still works: an ordinary decode afterwards matches the oracle
        from asterq.decode import DeviceDecodePlan, latent_decode
        from asterq.plan import build_plan

        got = latent_decode(wl.pools, DeviceDecodePlan(build_plan(wl.layouts, 16), cuda), wl.q_lat, wl.q_rope,
                            wl.new_latent, wl.new_rope, softmax_scale=SCALE, out_dtype=torch.float32).cpu().numpy()
        lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
        cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, 512)
        ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
        assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2
    finally:
        _lib.check(lib.asterq_mailbox_destroy(own.value))
