"""The paged drop-in cache and attention mirror against the oracle's replay of the reference.

* cold chunks: codes and scales bit-identical to ``quantize_tensor`` on the same
  tokens, flushed at the reference's threshold (cache.py:167-177), whether the
  history arrives at once or token by token;
* lengths and ``num_bytes`` as the reference accounts them (cache.py:72-87);
* ``materialize_*`` / ``iter_chunks`` equal the oracle's dequantized view bit for bit;
* ``latent_attention`` / ``LatentAttentionKernels`` within the decode tolerance
  (rel-L2 <= 1e-3, max-abs <= 2e-2 on fp32 outputs).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)


def _inputs(seed, n, q_len=1):
    from asterq.synth import c1_inputs

    return c1_inputs(seed=seed, ctx=n, q_len=q_len)


def _bf16_np(t):
    return t.float().cpu().numpy()


def test_bulk_append_matches_reference_flush(cuda):
    from asterq.cache import LatentLayerCache

    inp = _inputs(1, 3000)
    lat, rope = inp["latent"][:3000], inp["rope"][:3000]
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=512, chunk_tokens=512)
    cache.append(lat[None].to(cuda), rope[None].to(cuda), None, 0)
    ref = O.build_cache_from_tokens(_bf16_np(lat), _bf16_np(rope), 512, 512)
    assert cache.cold_chunks == len(ref.cold) and cache.length == ref.length == 3000
    assert cache.hot_length == ref.hot_latent.shape[0]
    for q, r, c in zip(cache.cold_latent, cache.cold_rope, ref.cold):
        np.testing.assert_array_equal(q.data[0].cpu().numpy(), c.codes)
        np.testing.assert_array_equal(q.scale[0, :, :, 0].cpu().numpy(), c.scales)
        np.testing.assert_array_equal(_bf16_np(r[0]), c.rope)
    np.testing.assert_array_equal(_bf16_np(cache.latent[0]), ref.hot_latent)
    np.testing.assert_array_equal(_bf16_np(cache.rope_key[0]), ref.hot_rope)
    assert cache.num_bytes == ref.cold_length * 400 + ref.hot_latent.shape[0] * 1152


def test_token_by_token_append_equals_bulk(cuda):
    from asterq.cache import LatentLayerCache

    inp = _inputs(2, 1700)
    lat, rope = inp["latent"][:1700].to(cuda), inp["rope"][:1700].to(cuda)
    bulk = LatentLayerCache("hadamard_int4", 64, recent_tokens=256, chunk_tokens=512)
    bulk.append(lat[None], rope[None], None, 0)
    step = LatentLayerCache("hadamard_int4", 64, recent_tokens=256, chunk_tokens=512)
    step.append(lat[None, :900], rope[None, :900], None, 0)
    for i in range(900, 1700, 40):
        step.append(lat[None, i:i + 40], rope[None, i:i + 40], None, 0)
        assert step.hot_length <= 256 + 512
    assert step.cold_chunks == bulk.cold_chunks and step.length == bulk.length
    for a, b in zip(step.cold_latent, bulk.cold_latent):
        assert torch.equal(a.data, b.data) and torch.equal(a.scale, b.scale)
    assert torch.equal(step.latent, bulk.latent)


def test_batch_rows_are_independent(cuda):
    from asterq.cache import LatentLayerCache

    a, b = _inputs(3, 1400), _inputs(4, 1400)
    lat = torch.stack([a["latent"][:1400], b["latent"][:1400]]).to(cuda)
    rope = torch.stack([a["rope"][:1400], b["rope"][:1400]]).to(cuda)
    both = LatentLayerCache("hadamard_int4", 64, recent_tokens=128, chunk_tokens=256)
    both.append(lat, rope, None, 0)
    for row in range(2):
        one = LatentLayerCache("hadamard_int4", 64, recent_tokens=128, chunk_tokens=256)
        one.append(lat[row:row + 1], rope[row:row + 1], None, 0)
        for x, y in zip(both.cold_latent, one.cold_latent):
            assert torch.equal(x.data[row], y.data[0]) and torch.equal(x.scale[row], y.scale[0])
        assert torch.equal(both.latent[row], one.latent[0])


@pytest.mark.parametrize("scheme", ["hadamard_int4", "int4", "int8", "float8"])
def test_materialize_and_iter_chunks_match_oracle(cuda, scheme):
    from asterq.cache import LatentLayerCache

    inp = _inputs(5, 2100)
    lat, rope = inp["latent"][:2100], inp["rope"][:2100]
    cache = LatentLayerCache(scheme, 64, recent_tokens=512, chunk_tokens=512)
    cache.append(lat[None].to(cuda), rope[None].to(cuda), None, 0)
    ref = O.build_cache_from_tokens(_bf16_np(lat), _bf16_np(rope), 512, 512, scheme=scheme)
    want_lat, want_rope = ref.materialize()
    got_lat = cache.materialize_latent(dtype=torch.float32)[0].cpu().numpy()
    got_rope = cache.materialize_rope(dtype=torch.float32)[0].cpu().numpy()
    np.testing.assert_array_equal(got_lat, want_lat)
    np.testing.assert_array_equal(got_rope, want_rope)
    chunks = list(cache.iter_chunks(dtype=torch.float32, device=cuda))
    assert len(chunks) == len(ref.cold) + 1
    np.testing.assert_array_equal(torch.cat([c[0] for c in chunks], dim=1)[0].cpu().numpy(), want_lat)


@pytest.mark.parametrize("q_len,scheme", [(1, "hadamard_int4"), (3, "hadamard_int4"), (1, "int4"), (3, "int4"),
                                          (1, "int8"), (3, "int8"), (1, "float8"), (3, "float8")])
def test_latent_attention_over_the_cache(cuda, q_len, scheme):
    """Every cold scheme the kernels read: hadamard_int4 (scores in the rotated basis), plain
    int4 (kv.py scheme "int4", no rotation) and int8 (one signed byte a dim, 64-token tiles);
    planned on the GPU from the cache's device page tables."""
    from asterq.attention import latent_attention
    from asterq.cache import LatentLayerCache

    n = 4000
    inp = _inputs(6 + q_len, n, q_len)
    cache = LatentLayerCache(scheme, 64, recent_tokens=512, chunk_tokens=512)
    cache.append(inp["latent"][None, :n].to(cuda), inp["rope"][None, :n].to(cuda), None, 0)
    out = latent_attention(inp["q_lat"][None].to(cuda), inp["q_rope"][None].to(cuda),
                           inp["latent"][None, n:].to(cuda), inp["rope"][None, n:].to(cuda), cache,
                           softmax_scale=SCALE)
    lat, rope = _bf16_np(inp["latent"]), _bf16_np(inp["rope"])
    ref_cache = O.build_cache_from_tokens(lat[:n], rope[:n], 512, 512, scheme=scheme)
    ref = O.decode(_bf16_np(inp["q_lat"]), _bf16_np(inp["q_rope"]), lat[n:], rope[n:], ref_cache, SCALE)
    got = out[0].cpu().numpy()
    assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2


@pytest.mark.parametrize("scheme,dtype", [("hadamard_int4", torch.bfloat16), ("int4", torch.bfloat16),
                                          ("hadamard_int4", torch.float32), ("int8", torch.bfloat16),
                                          ("float8", torch.bfloat16), ("int8", torch.float32)])
def test_quantize_rope_cache_matches_reference(cuda, scheme, dtype):
    """quantize_rope=True (cache.py:64, :160-164): each flushed chunk's RoPE keys are quantized from
    the values as stored (the caller's dtype) with the cold scheme, one group of 64 -- codes and
    scales bit-exact to quantize_tensor, the reference's byte accounting (32 code bytes and one fp16
    scale a token for INT4, 64 bytes and a scale for int8, 64 e4m3 bytes for float8), dequantized
    views bit-exact -- and attention reads the codes directly (q_len 1 and 3, within the decode
    tolerance)."""
    from asterq.attention import latent_attention
    from asterq.cache import LatentLayerCache
    from asterq.kv import QuantizedTensor

    n = 3300
    inp = _inputs(41, n, 3)
    lat, rope = inp["latent"].to(dtype), inp["rope"].to(dtype)
    cache = LatentLayerCache(scheme, 64, recent_tokens=512, chunk_tokens=512, quantize_rope=True)
    cache.append(lat[None, :1200].to(cuda), rope[None, :1200].to(cuda), None, 0)
    cache.append(lat[None, 1200:n].to(cuda), rope[None, 1200:n].to(cuda), None, 0)
    lat_np, rope_np = lat.float().numpy(), rope.float().numpy()
    ref = O.build_cache_from_tokens(lat_np[:n], rope_np[:n], 512, 512, scheme=scheme, quantize_rope=True)
    assert cache.cold_chunks == len(ref.cold) > 0 and cache.length == n
    for q, r, c in zip(cache.cold_latent, cache.cold_rope, ref.cold):
        np.testing.assert_array_equal(q.data[0].view(torch.uint8).cpu().numpy(), c.codes.view(np.uint8))
        assert isinstance(r, QuantizedTensor) and r.scheme == scheme and r.original_shape == (1, 512, 64)
        np.testing.assert_array_equal(r.data[0].view(torch.uint8).cpu().numpy(), c.rope_codes.view(np.uint8))
        if scheme == "float8":
            assert r.scale is None and c.rope_scales is None
        else:
            np.testing.assert_array_equal(r.scale[0, :, 0, 0].cpu().numpy(), c.rope_scales)
    cold = cache.cold_length
    per_cold = {"hadamard_int4": 256 + 16 + 32 + 2, "int4": 256 + 16 + 32 + 2, "int8": 512 + 16 + 64 + 2,
                "float8": 512 + 64}[scheme]
    assert cache.num_bytes == cold * per_cold + (n - cold) * (512 + 64) * dtype.itemsize
    got_rope = cache.materialize_rope(dtype=torch.float32)[0].cpu().numpy()
    np.testing.assert_array_equal(got_rope, ref.materialize()[1])

    bf = O.round_bf16
    view = ref if dtype == torch.bfloat16 else O.LatentCacheView(
        cold=ref.cold, hot_latent=bf(ref.hot_latent), hot_rope=bf(ref.hot_rope))
    for q_len in (1, 3):
        out = latent_attention(inp["q_lat"][None, :q_len].to(cuda), inp["q_rope"][None, :q_len].to(cuda),
                               lat[None, n:n + q_len].to(cuda), rope[None, n:n + q_len].to(cuda), cache,
                               softmax_scale=SCALE)
        want = O.decode(_bf16_np(inp["q_lat"][:q_len]), _bf16_np(inp["q_rope"][:q_len]), bf(lat_np[n:n + q_len]),
                        bf(rope_np[n:n + q_len]), view, SCALE)
        got = out[0].cpu().numpy()
        assert O.rel_l2(got, want) <= 1e-3 and O.max_abs(got, want) <= 2e-2, q_len


@pytest.mark.parametrize("scheme", ["int8", "float8"])
def test_byte_cache_codes_bytes_and_decode_loop(cuda, scheme):
    """cache_dtype="int8" (kv.py:76-118 with qmax 127) and "float8" (kv.py:85-89, no scales):
    flushed chunks hold the reference's codes (and scales) bit for bit, ``num_bytes`` counts 512
    code bytes a cold token, and a decode loop of appends and attention (device planner, 64-token
    cold tiles) matches the oracle."""
    from asterq.attention import latent_attention
    from asterq.cache import LatentLayerCache

    n, steps = 2000, 40
    inp = _inputs(43, n + steps, 1)
    lat, rope = inp["latent"], inp["rope"]
    cache = LatentLayerCache(scheme, 64, recent_tokens=256, chunk_tokens=512)
    cache.append(lat[None, :n].to(cuda), rope[None, :n].to(cuda), None, 0)
    ref = O.build_cache_from_tokens(_bf16_np(lat[:n]), _bf16_np(rope[:n]), 256, 512, scheme=scheme)
    assert cache.cold_chunks == len(ref.cold) > 0
    for q, c in zip(cache.cold_latent, ref.cold):
        assert q.scheme == scheme and q.data.dtype == (torch.int8 if scheme == "int8" else torch.float8_e4m3fn)
        np.testing.assert_array_equal(q.data[0].view(torch.uint8).cpu().numpy(), c.codes.view(np.uint8))
        if scheme == "int8":
            np.testing.assert_array_equal(q.scale[0, :, :, 0].cpu().numpy(), c.scales)
        else:
            assert q.scale is None
    cold = cache.cold_length
    assert cache.num_bytes == cold * (512 + (16 if scheme == "int8" else 0) + 128) + (n - cold) * 1152
    q = inp["q_lat"][:1]
    qr = inp["q_rope"][:1]
    lat_np, rope_np = _bf16_np(lat), _bf16_np(rope)
    for t in range(n, n + steps):
        out = latent_attention(q[None].to(cuda), qr[None].to(cuda), lat[None, t:t + 1].to(cuda),
                               rope[None, t:t + 1].to(cuda), cache, softmax_scale=SCALE)
        if t in (n, n + steps - 1):
            view = O.build_cache_from_tokens(lat_np[:t], rope_np[:t], 256, 512, scheme=scheme)
            want = O.decode(_bf16_np(q), _bf16_np(qr), lat_np[t:t + 1], rope_np[t:t + 1], view, SCALE)
            got = out[0].cpu().numpy()
            assert O.rel_l2(got, want) <= 1e-3 and O.max_abs(got, want) <= 2e-2, t
        cache.append(lat[None, t:t + 1].to(cuda), rope[None, t:t + 1].to(cuda), None, 0)
    assert cache.length == n + steps


def test_empty_cache_prefill_is_causal(cuda):
    from asterq.attention import latent_attention

    inp = _inputs(9, 0, 4)
    out = latent_attention(inp["q_lat"][None].to(cuda), inp["q_rope"][None].to(cuda),
                           inp["latent"][None].to(cuda), inp["rope"][None].to(cuda), None, softmax_scale=SCALE)
    ref = O.decode(_bf16_np(inp["q_lat"]), _bf16_np(inp["q_rope"]), _bf16_np(inp["latent"]), _bf16_np(inp["rope"]),
                   O.LatentCacheView(cold=[], hot_latent=np.zeros((0, 512), np.float32),
                                     hot_rope=np.zeros((0, 64), np.float32)), SCALE)
    got = out[0].cpu().numpy()
    assert O.rel_l2(got, ref) <= 1e-3 and O.max_abs(got, ref) <= 2e-2


def test_kernel_module_absorbs_weights(cuda):
    from asterq.attention import LatentAttentionKernels
    from asterq.cache import LatentLayerCache

    n, heads, hd = 2500, 16, 64
    inp = _inputs(10, n)
    g = torch.Generator().manual_seed(11)
    wk = (torch.randn(heads * hd, 512, generator=g) / 24).to(cuda)
    wv = (torch.randn(heads * hd, 512, generator=g) / 24).to(cuda)
    mod = LatentAttentionKernels(wk, wv, heads, hd)
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=512, chunk_tokens=512)
    cache.append(inp["latent"][None, :n].to(cuda), inp["rope"][None, :n].to(cuda), None, 0)
    q_content = torch.randn(1, 1, heads, hd, generator=g).to(cuda)
    q_rope = inp["q_rope"][None].float().to(cuda)
    out = mod._absorbed_decode(q_content, q_rope, inp["latent"][None, n:].float().to(cuda),
                               inp["rope"][None, n:].float().to(cuda), cache)
    # oracle: same absorbed query, oracle attention, same value projection
    q_lat = torch.einsum("bthd,hdl->bthl", q_content, wk.view(heads, hd, 512))
    q_lat_bf = q_lat.to(torch.bfloat16).float()[0].cpu().numpy()
    lat, rope = _bf16_np(inp["latent"]), _bf16_np(inp["rope"])
    ctx = O.decode(q_lat_bf, _bf16_np(inp["q_rope"]), lat[n:], rope[n:], O.build_cache_from_tokens(lat[:n], rope[:n], 512, 512),
                   1.0 / math.sqrt(hd + 64))
    want = torch.einsum("thl,hdl->thd", torch.from_numpy(ctx), wv.view(heads, hd, 512).cpu()).numpy()
    got = out[0].cpu().numpy()
    assert O.rel_l2(got, want) <= 1e-3


def test_window_trim_keeps_sink_and_recent(cuda):
    from asterq.cache import LatentLayerCache

    inp = _inputs(12, 3000)
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=256, chunk_tokens=256)
    lat, rope = inp["latent"][None, :3000].to(cuda), inp["rope"][None, :3000].to(cuda)
    cache.append(lat[:, :2000], rope[:, :2000], 1000, 4)
    assert cache.length == 1000
    cache.append(lat[:, 2000:2100], rope[:, 2000:2100], 1000, 4)
    assert cache.length <= 1000 + 256 and cache.hot_length <= 512


def test_float32_caller_keeps_float32_and_codes_come_from_it(cuda):
    """The reference keeps the appended dtype in the hot window (cache.py:193-200) and quantizes
    flushed chunks from it (cache.py:172); cold RoPE keys become bf16 (cache.py:162-164).  A
    float32 caller therefore gets float32 hot tokens back unchanged, codes and scales bit-exact
    to quantizing the float32 values, and float32 hot bytes in ``num_bytes``.  The decode kernel
    reads bf16 operands of the hot window, the new tokens and the query; its result is checked
    against the oracle on exactly those operands."""
    import dataclasses

    from asterq.attention import latent_attention
    from asterq.cache import LatentLayerCache

    n = 2300
    g = torch.Generator().manual_seed(13)
    lat = torch.randn(n + 1, 512, generator=g)
    lat[:, :5] *= 20.0
    rope = torch.randn(n + 1, 64, generator=g)
    q_lat, q_rope = torch.randn(1, 16, 512, generator=g), torch.randn(1, 16, 64, generator=g)
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=512, chunk_tokens=512)
    cache.append(lat[None, :1000].to(cuda), rope[None, :1000].to(cuda), None, 0)
    cache.append(lat[None, 1000:n].to(cuda), rope[None, 1000:n].to(cuda), None, 0)

    lat_np, rope_np = lat.numpy(), rope.numpy()
    ref = O.build_cache_from_tokens(lat_np[:n], O.round_bf16(rope_np[:n]), 512, 512)
    assert cache.cold_chunks == len(ref.cold) > 0 and cache.length == n
    for q, r, c in zip(cache.cold_latent, cache.cold_rope, ref.cold):
        np.testing.assert_array_equal(q.data[0].cpu().numpy(), c.codes)
        np.testing.assert_array_equal(q.scale[0, :, :, 0].cpu().numpy(), c.scales)
        assert r.dtype == torch.bfloat16
        np.testing.assert_array_equal(r[0].float().cpu().numpy(), c.rope)
    cold = cache.cold_length
    assert cache.latent.dtype == torch.float32 and cache.rope_key.dtype == torch.float32
    np.testing.assert_array_equal(cache.latent[0].cpu().numpy(), lat_np[cold:n])
    np.testing.assert_array_equal(cache.rope_key[0].cpu().numpy(), rope_np[cold:n])
    assert cache.materialize_latent().dtype == torch.float32
    assert cache.num_bytes == cold * 400 + (n - cold) * (512 + 64) * 4
    with pytest.raises(ValueError, match="dtype"):
        cache.append(lat[None, n:].to(cuda).bfloat16(), rope[None, n:].to(cuda).bfloat16(), None, 0)

    out = latent_attention(q_lat[None].to(cuda), q_rope[None].to(cuda), lat[None, n:].to(cuda),
                           rope[None, n:].to(cuda), cache, softmax_scale=SCALE)
    bf = O.round_bf16
    view = dataclasses.replace(ref, hot_latent=bf(ref.hot_latent), hot_rope=bf(ref.hot_rope))
    want = O.decode(bf(q_lat.numpy()), bf(q_rope.numpy()), bf(lat_np[n:]), bf(rope_np[n:]), view, SCALE)
    got = out[0].cpu().numpy()
    assert O.rel_l2(got, want) <= 1e-3 and O.max_abs(got, want) <= 2e-2


def test_window_trim_by_pages_keeps_codes_and_matches_the_oracle(cuda):
    """trim_mode="pages": the cold pages between the sink and the recent tokens are released
    whole; the kept pages' codes are the ones written at flush time (no re-quantization), and
    decoding over the trimmed cache equals the oracle over exactly the kept tokens."""
    from asterq.attention import latent_attention
    from asterq.cache import LatentLayerCache

    P, n = 256, 3000
    inp = _inputs(14, n)
    lat, rope = inp["latent"][:n], inp["rope"][:n]
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=256, chunk_tokens=P, trim_mode="pages")
    cache.append(lat[None].to(cuda), rope[None].to(cuda), 1500, 4)
    # 10 cold pages + 440 hot; page 0 holds the sink, pages 5-9 and the hot window the recent tokens
    assert cache.cold_chunks == 6 and cache.hot_length == 440 and cache.length == 6 * P + 440
    full = O.build_cache_from_tokens(_bf16_np(lat), _bf16_np(rope), 256, P)
    kept = [full.cold[0]] + full.cold[5:]
    for q, c in zip(cache.cold_latent, kept):
        np.testing.assert_array_equal(q.data[0].cpu().numpy(), c.codes)
        np.testing.assert_array_equal(q.scale[0, :, :, 0].cpu().numpy(), c.scales)
    import dataclasses

    view = dataclasses.replace(full, cold=kept)
    out = latent_attention(inp["q_lat"][None].to(cuda), inp["q_rope"][None].to(cuda), inp["latent"][None, n:].to(cuda),
                           inp["rope"][None, n:].to(cuda), cache, softmax_scale=SCALE)
    want = O.decode(_bf16_np(inp["q_lat"]), _bf16_np(inp["q_rope"]), _bf16_np(inp["latent"][n:]),
                    _bf16_np(inp["rope"][n:]), view, SCALE)
    got = out[0].cpu().numpy()
    assert O.rel_l2(got, want) <= 1e-3 and O.max_abs(got, want) <= 2e-2
    # a second append re-checks the window: nothing left between sink and recent pages
    cache.append(lat[None, :8].to(cuda), rope[None, :8].to(cuda), 1500, 4)
    assert cache.cold_chunks == 6


def test_decode_loop_through_the_drop_in_cache_plans_on_the_gpu(cuda, monkeypatch):
    """The reference-interface loop (latent_attention over the cache, then cache.append of the
    step's token, as latent_attention.py:233-253 and cache.py:186-201 do it) with flushes along
    the way: no host-built schedule (the host planner is made to fail), the new tokens land in
    the hot pages through the in-place append kernel, and the outputs follow the oracle."""
    import asterq.attention as attn_mod
    from asterq.cache import LatentLayerCache

    def no_host_plan(*a, **k):
        raise AssertionError("the host planner ran")

    n, B = 700, 2
    g = torch.Generator().manual_seed(15)
    lat = torch.randn(B, n + 80, 512, generator=g)
    lat[..., :5] *= 20.0
    lat = lat.to(torch.bfloat16)
    rope = torch.randn(B, n + 80, 64, generator=g).to(torch.bfloat16)
    cache = LatentLayerCache("hadamard_int4", 64, recent_tokens=128, chunk_tokens=128)
    cache.append(lat[:, :n].to(cuda), rope[:, :n].to(cuda), None, 0)
    monkeypatch.setattr(attn_mod, "build_plan", no_host_plan)
    for step in range(80):
        k = n + step
        q = torch.randn(B, 1, 16, 512, generator=g).to(torch.bfloat16)
        qr = torch.randn(B, 1, 16, 64, generator=g).to(torch.bfloat16)
        out = attn_mod.latent_attention(q.to(cuda), qr.to(cuda), lat[:, k : k + 1].to(cuda), rope[:, k : k + 1].to(cuda),
                                        cache, softmax_scale=SCALE)
        if step % 19 == 0 or step == 79:
            got = out.cpu().numpy()
            for b in range(B):
                lb, rb = _bf16_np(lat[b, : k + 1]), _bf16_np(rope[b, : k + 1])
                want = O.decode(_bf16_np(q[b]), _bf16_np(qr[b]), lb[k:], rb[k:],
                                O.build_cache_from_tokens(lb[:k], rb[:k], 128, 128), SCALE)
                assert O.rel_l2(got[b], want) <= 1e-3 and O.max_abs(got[b], want) <= 2e-2, (step, b)
        cache.append(lat[:, k : k + 1].to(cuda), rope[:, k : k + 1].to(cuda), None, 0)
    cache.raise_if_failed()
    assert cache.length == n + 80 and cache.cold_chunks == len(O.build_cache_from_tokens(
        _bf16_np(lat[0, : n + 80]), _bf16_np(rope[0, : n + 80]), 128, 128).cold)
    np.testing.assert_array_equal(_bf16_np(cache.latent[1]), _bf16_np(lat[1, cache.cold_length : n + 80]))
