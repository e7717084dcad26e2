"""Pin the CPU oracle against outputs of the reference itself (golden fixtures).

The fixtures come from tests/golden/make_golden.py, which runs AsterLM's own
quantize_tensor / LatentLayerCache / LatentAttention code.  Codes and scales must
match bit for bit; decode outputs within float32 reassociation noise.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O
from asterq.synth import c1_inputs

SCALE = 1.0 / math.sqrt(512 + 64)


def _sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def test_oracle_encode_matches_reference_bit_exact(golden_encode):
    x = O.bf16_to_f32(golden_encode["enc_x_bits"])
    q = O.quantize(x, "hadamard_int4", 64)
    np.testing.assert_array_equal(q.data, golden_encode["enc_codes"])
    np.testing.assert_array_equal(q.scale.reshape(x.shape[0], -1).view(np.uint16),
                                  golden_encode["enc_scales"].view(np.uint16))


@pytest.mark.parametrize("scheme", ["hadamard_int4", "int4", "int8"])
def test_oracle_reference_test_case(golden_encode, scheme):
    """The reference's tests/test_quantization.py:9-12 input (48 -> 64 padding, group 16)."""
    x = O.bf16_to_f32(golden_encode["small_x_bits"])
    q = O.quantize(x, scheme, 16)
    np.testing.assert_array_equal(q.data.view(np.uint8), golden_encode[f"small_{scheme}_codes"].view(np.uint8))
    np.testing.assert_array_equal(q.scale.view(np.uint16), golden_encode[f"small_{scheme}_scales"].view(np.uint16))
    restored = O.dequantize(q)
    assert restored.shape == x.shape
    if scheme != "int8":
        assert float(np.sqrt(np.mean((restored - x) ** 2))) < 0.18  # tests/test_quantization.py:15


def test_oracle_round_half_even_ties(golden_encode):
    x = O.bf16_to_f32(golden_encode["tie_x_bits"])
    q = O.quantize(x, "int4", 16)
    np.testing.assert_array_equal(q.data, golden_encode["tie_int4_codes"])
    codes = O.unpack_int4(q.data, 16)[0]
    # 0.5 -> 0, 1.5 -> 2, 2.5 -> 2, 3.5 -> 4, 4.5 -> 4, 5.5 -> 6, 6.5 -> 6 (and mirrored)
    assert codes.tolist() == [7, 0, 2, 2, 0, -2, -2, 4, -4, 4, -4, 6, -6, 6, -6, 0]


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    v = rng.integers(-7, 8, size=(5, 64)).astype(np.int8)
    np.testing.assert_array_equal(O.unpack_int4(O.pack_int4(v), 64), v)


def test_fwht_is_self_inverse():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, 512)).astype(np.float32)
    np.testing.assert_allclose(O.normalized_fwht(O.normalized_fwht(x)), x, atol=1e-5)


def test_oracle_float8_matches_reference(golden_encode):
    """float8 (kv.py:85-89) from bf16 and float32 inputs, edge values included."""
    x16 = O.bf16_to_f32(golden_encode["f8_x_bits"])
    np.testing.assert_array_equal(O.quantize(x16, "float8").data, golden_encode["f8_codes_bf16"])
    np.testing.assert_array_equal(O.quantize(golden_encode["f8_x_f32"], "float8").data, golden_encode["f8_codes_f32"])


@pytest.mark.parametrize("scheme", ["hadamard_int4", "int4"])
def test_oracle_rope_quantization_matches_reference(golden_encode, scheme):
    """quantize_rope=True encodes [tokens, 64] RoPE keys as one group of 64 (cache.py:160-164)."""
    x = O.bf16_to_f32(golden_encode["rope_x_bits"])
    q = O.quantize(x, scheme, 64)
    np.testing.assert_array_equal(q.data, golden_encode[f"rope_{scheme}_codes"])
    np.testing.assert_array_equal(q.scale.reshape(-1).view(np.uint16),
                                  golden_encode[f"rope_{scheme}_scales"].view(np.uint16))


@pytest.mark.parametrize("case", ["c1", "small", "hotonly", "t3", "qrope", "qr4", "q8", "q8t3", "f8", "f8t3", "q8r", "f8r"])
def test_oracle_decode_matches_reference(golden_decode, case):
    g = {k[len(case) + 1:]: v for k, v in golden_decode.items() if k.startswith(case + "_")}
    ctx, q_len = int(g["ctx"]), int(g["q_len"])
    inp = c1_inputs(seed=int(g["seed"]), ctx=ctx, q_len=q_len)
    assert _sha(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"]) == str(g["input_sha256"])
    lat = inp["latent"].float().numpy()
    rope = inp["rope"].float().numpy()
    scheme = str(g["scheme"]) if "scheme" in g else "hadamard_int4"
    quantize_rope = bool(g["quantize_rope"]) if "quantize_rope" in g else False
    cache = O.build_cache_from_tokens(lat[:ctx], rope[:ctx], int(g["recent"]), int(g["chunk"]), scheme=scheme,
                                      quantize_rope=quantize_rope)
    assert len(cache.cold) == int(g["cold_chunks"])
    if quantize_rope:
        assert _sha(*[torch.from_numpy(c.rope_codes) for c in cache.cold]) == str(g["rope_codes_sha256"])
    assert cache.hot_latent.shape[0] == int(g["hot_tokens"])
    out = O.decode(inp["q_lat"].float().numpy(), inp["q_rope"].float().numpy(), lat[ctx:], rope[ctx:], cache, SCALE)
    ref = g["out_fp32"]
    assert out.shape == ref.shape
    assert O.rel_l2(out, ref) < 1e-5
    assert O.max_abs(out, ref) < 1e-3  # outputs reach ~30; float32 reassociation in SDPA
    # the bf16-arithmetic reference is informational: its own noise exceeds 1e-3
    assert O.rel_l2(g["out_bf16"], ref) < 1e-2


def test_causal_row0_equals_absorbed(golden_decode):
    """_full_attention row 0 == _absorbed_decode (the q_len>1 and q_len=1 paths agree)."""
    inp = c1_inputs(seed=7, ctx=1500, q_len=3)
    lat = inp["latent"].float().numpy()
    rope = inp["rope"].float().numpy()
    cache = O.build_cache_from_tokens(lat[:1500], rope[:1500], 512, 512)
    q = inp["q_lat"].float().numpy()
    qr = inp["q_rope"].float().numpy()
    full = O.causal_attention(q, qr, lat[1500:], rope[1500:], cache, SCALE)
    one = O.absorbed_decode(q[:1], qr[:1], lat[1500:1501], rope[1500:1501], cache, SCALE)
    assert O.rel_l2(full[:1], one) < 1e-5
