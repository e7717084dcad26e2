"""Context-parallel decode on one GPU with the ranks emulated in turn.

Each emulated rank decodes its chunk range into partial records, merges them
with ``asterq_splitkv_merge``, and the records are concatenated rank-major as
``all_gather_into_tensor`` would leave them; ``finish`` must reproduce the
single-GPU oracle decode (rel-L2 <= 1e-3, max-abs <= 2e-2, fp32 output).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_emulated_ranks_match_oracle(cuda, world):
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import PoolBuilder, c1_inputs

    ctx, hot = 20 * 512 + 300, 700
    inp = c1_inputs(seed=40 + world, ctx=ctx, q_len=1)
    b = PoolBuilder([ctx], [hot], q_len=1, n_heads=16, device=cuda)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("cp")
    decs = [ContextParallelDecoder(wl.pools, wl.layouts[0], 16, r, world, cuda) for r in range(world)]
    recs = [d.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE).clone() for d in decs]
    out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)
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
