"""Decode attention on the GPU against the reference (golden fixtures) and the oracle.

Tolerance (north_star): max-abs <= 2e-2 and rel-L2 <= 1e-3, checked on the
float32 output against the float32 reference/oracle and on the bfloat16 output
against the bfloat16-rounded reference/oracle.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)
MAX_ABS = 2e-2
REL_L2 = 1e-3


def assert_close(out: np.ndarray, ref: np.ndarray, what: str) -> None:
    """float32 output vs float32 reference: rel-L2 <= 1e-3 and max-abs <= 2e-2."""
    rel, mab = O.rel_l2(out, ref), O.max_abs(out, ref)
    assert rel <= REL_L2 and mab <= MAX_ABS, f"{what}: rel-L2 {rel:.3e} max-abs {mab:.3e}"


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bfloat16 numbers at |x| (8 significant bits)."""
    ax = np.maximum(np.abs(x), np.float32(2.0 ** -126))
    return np.exp2(np.floor(np.log2(ax)) - 7).astype(np.float32)


def assert_close_bf16(out_bf16: np.ndarray, ref_fp32: np.ndarray, what: str) -> None:
    """bfloat16 output vs the bfloat16-rounded reference: rel-L2 <= 1e-3, and every
    element within max(2e-2, one bf16 ulp).  A bf16 value cannot be closer than one
    ulp when the exact result lies within float32 noise of a rounding boundary, and
    above |x| = 4 one ulp already exceeds 2e-2."""
    ref = O.round_bf16(ref_fp32)
    rel = O.rel_l2(out_bf16, ref)
    err = np.abs(out_bf16.astype(np.float64) - ref)
    bound = np.maximum(MAX_ABS, bf16_ulp(ref_fp32))
    worst = float(np.max(err - bound))
    assert rel <= REL_L2 and worst <= 0.0, f"{what}: rel-L2 {rel:.3e}, worst excess over bound {worst:.3e}"


def run_decode(wl, *, out_dtype=torch.float32, softcap=None, **plan_kw):
    from asterq.decode import COLD_TILE_TOKENS, DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan

    plan_kw.setdefault("cold_tile", COLD_TILE_TOKENS[wl.pools.cold_scheme])
    plan = build_plan(wl.layouts, wl.n_heads, **plan_kw)
    dplan = DeviceDecodePlan(plan, wl.q_lat.device)
    out = latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                        logit_softcap=softcap, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out, plan


def single_sequence_workload(inp, ctx, hot, q_len, device, scheme="hadamard_int4", quantize_rope=False):
    from asterq.synth import PoolBuilder

    b = PoolBuilder([ctx], [hot], q_len=q_len, n_heads=inp["q_lat"].shape[1], device=device, scheme=scheme,
                    quantize_rope=quantize_rope)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    return b.finish("single")


def oracle_for(inp, ctx, hot, q_len, softcap=None, chunk=512, scheme="hadamard_int4", quantize_rope=False):
    lat = inp["latent"].float().numpy()
    rope = inp["rope"].float().numpy()
    cache = O.build_cache_split(lat[:ctx], rope[:ctx], hot, chunk, scheme=scheme, quantize_rope=quantize_rope)
    return O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache,
                    SCALE, softcap)


@pytest.mark.parametrize("case", ["c1", "small", "hotonly", "t3", "qrope", "qr4", "q8", "q8t3", "f8", "f8t3", "q8r", "f8r"])
def test_decode_matches_reference_golden(cuda, golden_decode, case):
    """The reference's own outputs; "qrope" / "qr4": quantize_rope=True caches (cold RoPE keys as
    hadamard_int4 / int4 codes, cache.py:160-164)."""
    from asterq.synth import c1_inputs

    g = {k[len(case) + 1:]: v for k, v in golden_decode.items() if k.startswith(case + "_")}
    ctx, q_len = int(g["ctx"]), int(g["q_len"])
    inp = c1_inputs(seed=int(g["seed"]), ctx=ctx, q_len=q_len)
    scheme = str(g["scheme"]) if "scheme" in g else "hadamard_int4"
    quantize_rope = bool(g["quantize_rope"]) if "quantize_rope" in g else False
    wl = single_sequence_workload(inp, ctx, int(g["hot_tokens"]), q_len, cuda, scheme, quantize_rope)
    ref = g["out_fp32"]
    out32, _ = run_decode(wl, out_dtype=torch.float32)
    assert_close(out32.cpu().numpy(), ref, f"{case} fp32")
    out16, _ = run_decode(wl, out_dtype=torch.bfloat16)
    assert_close_bf16(out16.float().cpu().numpy(), ref, f"{case} bf16")


def test_c1_forced_splits_agree_with_single_item(cuda):
    """Many work items per sequence + the combine kernel == one item."""
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=0)
    wl = single_sequence_workload(inp, 8192, 1024, 1, cuda)
    one, plan1 = run_decode(wl, max_items_per_seq=1)
    many, plan2 = run_decode(wl, n_sms=64, ctas_per_sm=4, waves=4)
    assert plan1.n_slots == 0 and plan2.n_slots > 4
    assert O.rel_l2(many.cpu().numpy(), one.cpu().numpy()) < 1e-4
    assert_close(many.cpu().numpy(), oracle_for(inp, 8192, 1024, 1), "c1 split")


@pytest.mark.parametrize("q_len", [1, 2, 3, 4])
def test_q_len_causal(cuda, q_len):
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=20 + q_len, ctx=3000, q_len=q_len)
    wl = single_sequence_workload(inp, 3000, 700, q_len, cuda)
    out, _ = run_decode(wl)
    assert_close(out.cpu().numpy(), oracle_for(inp, 3000, 700, q_len), f"q_len {q_len}")


@pytest.mark.parametrize("q_len,n_heads", [(40, 16), (100, 16), (37, 6)])
def test_prefill_chunk_over_the_cache(cuda, q_len, n_heads):
    """Chunked prefill (q_len > 32, several new-token tiles) over the quantized cache:
    new token i sees the cache and new tokens 0..i (latent_attention.py:151-153)."""
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=40 + q_len, ctx=2500, q_len=q_len, n_heads=n_heads)
    wl = single_sequence_workload(inp, 2500, 700, q_len, cuda)
    out, plan = run_decode(wl)
    assert int((plan.tiles[:, 0] == 2).sum()) == (q_len + 31) // 32
    assert_close(out.cpu().numpy(), oracle_for(inp, 2500, 700, q_len), f"prefill q_len {q_len}")


@pytest.mark.parametrize("ctx,hot", [(0, 0), (5, 5), (513, 0), (640, 100), (1000, 1000), (4097, 2049)])
def test_edge_layouts(cuda, ctx, hot):
    """Empty cache (new tokens only), tiny caches, cold-only, partial chunks/tiles."""
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=ctx + hot + 1, ctx=ctx, q_len=1)
    wl = single_sequence_workload(inp, ctx, hot, 1, cuda)
    out, _ = run_decode(wl)
    assert_close(out.cpu().numpy(), oracle_for(inp, ctx, hot, 1), f"ctx {ctx} hot {hot}")


def test_softcap(cuda):
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=9, ctx=2500, q_len=1)
    wl = single_sequence_workload(inp, 2500, 600, 1, cuda)
    out, _ = run_decode(wl, softcap=2.0)
    assert_close(out.cpu().numpy(), oracle_for(inp, 2500, 600, 1, softcap=2.0), "softcap")


@pytest.mark.parametrize("q_len", [1, 3])
def test_plain_int4_cold_scheme(cuda, q_len):
    """Cold chunks in kv.py's scheme "int4" (no Hadamard rotation): the query is not
    rotated and the cold accumulator is not rotated back; split items and the
    combine kernel included."""
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=31 + q_len, ctx=6000, q_len=q_len)
    wl = single_sequence_workload(inp, 6000, 900, q_len, cuda, scheme="int4")
    ref = oracle_for(inp, 6000, 900, q_len, scheme="int4")
    one, _ = run_decode(wl, max_items_per_seq=1)
    many, plan = run_decode(wl, n_sms=32, ctas_per_sm=2, waves=4)
    assert plan.n_slots > 2
    assert_close(one.cpu().numpy(), ref, f"int4 q_len {q_len}")
    assert_close(many.cpu().numpy(), ref, f"int4 q_len {q_len} split")


@pytest.mark.parametrize("scheme,q_len", [("hadamard_int4", 1), ("hadamard_int4", 3), ("int4", 1), ("int4", 2)])
def test_quantized_rope_ragged_batch(cuda, scheme, q_len):
    """Cold RoPE keys stored as INT4 codes + one scale per token (quantize_rope=True): ragged
    lengths with partial cold pages (tiles of 1..128 tokens), hot windows and a cold-only sequence."""
    from asterq.synth import PoolBuilder, c1_inputs

    lengths, hot = [1300, 700, 2600, 129, 1031], [300, 0, 1000, 1, 7]
    b = PoolBuilder(lengths, hot, q_len=q_len, n_heads=16, device=cuda, scheme=scheme, quantize_rope=True)
    refs = []
    for i, (n, h) in enumerate(zip(lengths, hot)):
        inp = c1_inputs(seed=60 + i, ctx=n, q_len=q_len)
        b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
        refs.append(oracle_for(inp, n, h, q_len, scheme=scheme, quantize_rope=True))
    wl = b.finish("quantized rope")
    out, _ = run_decode(wl)
    out = out.cpu().numpy()
    for i, ref in enumerate(refs):
        assert_close(out[i * q_len:(i + 1) * q_len], ref, f"sequence {i}")
    split, plan = run_decode(wl, n_sms=16, ctas_per_sm=2, waves=4)
    assert plan.n_slots > 0
    assert O.rel_l2(split.cpu().numpy(), out) < 1e-4


@pytest.mark.parametrize("scheme,q_len,qrope", [("int8", 1, False), ("int8", 3, False), ("float8", 1, False),
                                                ("float8", 3, False), ("int8", 1, True), ("float8", 2, True)])
def test_byte_cold_schemes_ragged_batch(cuda, scheme, q_len, qrope):
    """int8 cold chunks (kv.py scheme "int8": one signed byte a dim, fp16 scale per group of 64, no
    rotation) and float8 chunks (e4m3 bytes, no scales) in 64-token tiles: ragged lengths with
    partial pages and tiles of 1..64 tokens, hot windows, a cold-only sequence; one item per
    block and a split schedule agree.  ``qrope``: the RoPE keys quantized too (quantize_rope=True)."""
    from asterq.synth import PoolBuilder, c1_inputs

    lengths, hot = [1300, 700, 2600, 65, 1031], [300, 0, 1000, 1, 7]
    b = PoolBuilder(lengths, hot, q_len=q_len, n_heads=16, device=cuda, scheme=scheme, quantize_rope=qrope)
    refs = []
    for i, (n, h) in enumerate(zip(lengths, hot)):
        inp = c1_inputs(seed=80 + i, ctx=n, q_len=q_len)
        b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
        refs.append(oracle_for(inp, n, h, q_len, scheme=scheme, quantize_rope=qrope))
    wl = b.finish(scheme)
    out, plan = run_decode(wl)
    assert plan.cold_tile == 64 and int(plan.tiles[plan.tiles[:, 0] == 0][:, 3].max()) == 64
    out = out.cpu().numpy()
    for i, ref in enumerate(refs):
        assert_close(out[i * q_len:(i + 1) * q_len], ref, f"sequence {i}")
    split, plan = run_decode(wl, n_sms=16, ctas_per_sm=2, waves=4)
    assert plan.n_slots > 0
    assert O.rel_l2(split.cpu().numpy(), out) < 1e-4


def test_int8_plan_with_int4_tiles_is_rejected(cuda):
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import PoolBuilder, c1_inputs

    inp = c1_inputs(seed=90, ctx=900, q_len=1)
    b = PoolBuilder([900], [100], q_len=1, n_heads=16, device=cuda, scheme="int8")
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("int8")
    dplan = DeviceDecodePlan(build_plan(wl.layouts, 16), cuda)
    with pytest.raises(ValueError, match="cold tiles"):
        latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE)


def test_quantized_rope_cold_tiles_at_any_offset(cuda):
    """Cold tiles that start and end off the 8-token grid of the RoPE scale copies: the layout
    takes tokens 5..511 of the first cold page, all of the second and 100 tokens from offset 3
    of the third."""
    from asterq.synth import PoolBuilder, c1_inputs

    n, h, q_len = 1500, 300, 2
    inp = c1_inputs(seed=71, ctx=n, q_len=q_len)
    b = PoolBuilder([n], [h], q_len=q_len, n_heads=16, device=cuda, quantize_rope=True)
    b.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    wl = b.finish("offsets")
    (p0, _, _), (p1, _, _), (p2, _, _) = wl.layouts[0].cold
    wl.layouts[0].cold = [(p0, 5, 507), (p1, 0, 512), (p2, 3, 100)]
    out, _ = run_decode(wl)
    lat, rope = inp["latent"].float().numpy(), inp["rope"].float().numpy()
    keep = np.r_[5:512, 512:1024, 1027:1127, n - h:n]
    cache = O.build_cache_split(lat[keep], rope[keep], h, 512, quantize_rope=True)
    ref = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[n:], rope[n:], cache, SCALE)
    assert_close(out.cpu().numpy(), ref, "offsets")


def test_n_heads_not_multiple_of_16(cuda):
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=13, ctx=1500, q_len=3, n_heads=6)  # 18 rows -> 2 row blocks, one ragged
    wl = single_sequence_workload(inp, 1500, 300, 3, cuda)
    out, _ = run_decode(wl)
    assert_close(out.cpu().numpy(), oracle_for(inp, 1500, 300, 3), "6 heads")


def test_c3_ragged_batch_subset(cuda):
    """Config 3 (64 ragged sequences) on the GPU; 6 sequences checked against the oracle."""
    from asterq.synth import c3_lengths, c3_workload

    lens = c3_lengths(0)
    order = np.argsort(lens)
    keep = {int(i) for i in list(order[:4]) + list(order[-2:])}
    wl = c3_workload(cuda, keep_host=keep)
    out32, plan = run_decode(wl)
    out16, _ = run_decode(wl, out_dtype=torch.bfloat16)
    assert plan.items.shape[0] > 148  # the ragged batch fills the GPU
    for i in sorted(keep):
        h = wl.host[i]
        ref = oracle_for(h, wl.lengths[i], wl.hot[i], 1)
        assert_close(out32[i : i + 1].cpu().numpy(), ref, f"seq {i} len {wl.lengths[i]}")
        assert_close_bf16(out16[i : i + 1].float().cpu().numpy(), ref, f"seq {i} bf16")


def test_c5_mtp_subset(cuda):
    """Config 5 shape (q_len 3, contexts 4k-64k) on a reduced batch of 6 sequences."""
    from asterq.synth import c5_lengths, make_workload

    lens = c5_lengths(0)[:6]
    wl = make_workload("c5 subset", lens, [min(n, 2048) for n in lens], q_len=3, seed=3, device=cuda,
                       keep_host={0, 5})
    out, _ = run_decode(wl)
    for i in (0, 5):
        ref = oracle_for(wl.host[i], wl.lengths[i], wl.hot[i], 3)
        assert_close(out[3 * i : 3 * i + 3].cpu().numpy(), ref, f"c5 seq {i}")


def test_deterministic(cuda):
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=0)
    wl = single_sequence_workload(inp, 8192, 1024, 1, cuda)
    a, _ = run_decode(wl, n_sms=32)
    b, _ = run_decode(wl, n_sms=32)
    assert torch.equal(a, b)


def test_rejects_bad_inputs(cuda):
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=1, ctx=600)
    wl = single_sequence_workload(inp, 600, 100, 1, cuda)
    dplan = DeviceDecodePlan(build_plan(wl.layouts, 16), cuda)
    with pytest.raises(ValueError):
        latent_decode(wl.pools, dplan, wl.q_lat.float(), wl.q_rope, wl.new_latent, wl.new_rope)
    with pytest.raises(ValueError):
        latent_decode(wl.pools, dplan, wl.q_lat[:, :8], wl.q_rope, wl.new_latent, wl.new_rope)


def test_timed_out_wait_is_reported_and_the_context_survives(cuda):
    """Failure detection without a fault: a tile whose arrival is never signalled (the
    ASTERQ_TILE_HOLD test hook) makes the pipeline waits run out after a short host-set limit;
    the kernel stops, the status word is set and the host raises.  A normal decode on the same
    context afterwards still matches the oracle."""
    from asterq import _lib
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import c1_inputs

    inp = c1_inputs(seed=31, ctx=3000)
    wl = single_sequence_workload(inp, 3000, 700, 1, cuda)
    dplan = DeviceDecodePlan(build_plan(wl.layouts, 16, n_sms=8), cuda)
    kept = int(dplan.tiles[3, 0].item())
    dplan.tiles[3, 0] = _lib.TILE_HOLD
    latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                  out_dtype=torch.float32, wait_limit_cycles=2_000_000)
    torch.cuda.synchronize()
    assert int(dplan.status.item()) == 1
    with pytest.raises(RuntimeError, match="timed out"):
        dplan.raise_if_failed()
    dplan.tiles[3, 0] = kept
    out = latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                        out_dtype=torch.float32)
    dplan.raise_if_failed()
    assert_close(out.cpu().numpy(), oracle_for(inp, 3000, 700, 1), "after a timed-out call")
