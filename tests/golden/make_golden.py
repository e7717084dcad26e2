"""Generate the golden fixtures by running the reference implementation.

Run in a container that has the AsterLM-Frontier source tree (it is imported
from ``$ASTERLM_REF_SRC``, default ``/root/reference/src``); the fixtures are
committed so that tests never need the reference at run time:

    python tests/golden/make_golden.py

Every input is regenerated from a seed with torch's CPU generator
(``asterq.synth.c1_inputs``), so fixtures store only outputs plus a SHA-256 of
the inputs (the tests recompute it to detect a changed generator).

Reference code exercised (paths relative to the reference's project root):
  quantize_tensor            src/asterlm/quantization/kv.py:76-118
  LatentLayerCache.append    src/asterlm/cache.py:186-201 (flush: :167-177)
  LatentAttention._absorbed_decode  src/asterlm/layers/latent_attention.py:177-231
  LatentAttention._full_attention   src/asterlm/layers/latent_attention.py:116-175
The decode entry points run as unbound functions on a duck-typed ``self`` with
identity absorption (head_dim = latent_rank = 512, W_k = W_v = stacked
identities), in float32 (the parity contract) and in bfloat16 (informational).
"""
from __future__ import annotations

import hashlib
import math
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "asterlm-frontier_b200"))
sys.path.insert(0, os.environ.get("ASTERLM_REF_SRC", "/root/reference/src"))

from asterlm.cache import LatentLayerCache  # noqa: E402
from asterlm.layers.latent_attention import LatentAttention  # noqa: E402
from asterlm.quantization.kv import quantize_tensor  # noqa: E402

from asterq.synth import c1_inputs  # noqa: E402  (pure torch, no CUDA needed)

H, L, R = 16, 512, 64


def sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def fake_attention(dtype: torch.dtype, n_heads: int = H):
    def linear() -> torch.nn.Linear:
        m = torch.nn.Linear(L, n_heads * L, bias=False)
        m.weight.data = torch.eye(L).repeat(n_heads, 1).to(dtype)
        return m

    return types.SimpleNamespace(
        n_heads=n_heads, head_dim=L, latent_rank=L, rope_dim=R, logit_softcap=None, training=False, dropout_p=0.0,
        qk_stat_tokens=0, k_up=linear(), v_up=linear(), _record_qk_statistics=lambda *a: None,
    )


def reference_cache(lat, rope, recent, chunk, group=64, scheme="hadamard_int4", quantize_rope=False):
    cache = LatentLayerCache(cache_dtype=scheme, group_size=group, recent_tokens=recent, chunk_tokens=chunk,
                             quantize_rope=quantize_rope)
    cache.append(lat.unsqueeze(0), rope.unsqueeze(0), window_size=None, sink_tokens=0)
    return cache


def decode_case(seed, ctx, q_len, recent, chunk, scheme="hadamard_int4", quantize_rope=False):
    inp = c1_inputs(seed=seed, ctx=ctx, q_len=q_len)
    lat, rope, q, qr = inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"]
    cache = reference_cache(lat[:ctx], rope[:ctx], recent, chunk, scheme=scheme, quantize_rope=quantize_rope)
    outs = {}
    for name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        f = fake_attention(dtype)
        args = (q.unsqueeze(0).to(dtype), qr.unsqueeze(0).to(dtype), lat[ctx:].unsqueeze(0).to(dtype),
                rope[ctx:].unsqueeze(0).to(dtype), cache)
        if q_len == 1:
            out = LatentAttention._absorbed_decode(f, *args)
        else:
            out = LatentAttention._full_attention(f, *args)
        outs[name] = out[0].detach().float().numpy()
    return {
        "input_sha256": sha(lat, rope, q, qr),
        "cold_chunks": len(cache.cold_latent),
        "hot_tokens": int(cache.latent.shape[1]),
        "cache_num_bytes": cache.num_bytes,
        "out_fp32": outs["fp32"],
        "out_bf16": outs["bf16"],
        "codes_sha256": sha(*[c.data for c in cache.cold_latent]),
        "scales_sha256": sha(*[c.scale for c in cache.cold_latent if c.scale is not None]),
        **({"rope_codes_sha256": sha(*[c.data for c in cache.cold_rope]),
            "rope_scales_sha256": sha(*[c.scale for c in cache.cold_rope if c.scale is not None])}
           if quantize_rope else {}),
    }


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    fixtures: dict[str, np.ndarray] = {}

    # ---- write path -------------------------------------------------------------
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1024, L, generator=g)
    x[:, torch.randperm(L, generator=g)[:5]] *= 20
    edge = torch.zeros(8, L)
    edge[1] = 1e-30  # below the 1e-8 clamp
    edge[2] = 3.0e4  # large magnitude
    edge[3, ::2] = 1.0
    edge[3, 1::2] = -1.0
    edge[4, 0] = 5.0  # single spike
    edge[5] = torch.linspace(-4, 4, L)
    edge[6] = 1e-6
    edge[7, :64] = 7.0
    x = torch.cat((x, edge)).to(torch.bfloat16)
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    fixtures["enc_x_bits"] = bf16_bits(x)
    fixtures["enc_codes"] = q.data.numpy()
    fixtures["enc_scales"] = q.scale.numpy().reshape(x.shape[0], -1)

    # the reference's own test input (tests/test_quantization.py:9-12): randn(2, 7, 48) bf16, group 16
    torch.manual_seed(1)
    xt = torch.randn(2, 7, 48, dtype=torch.bfloat16)
    fixtures["small_x_bits"] = bf16_bits(xt)
    for scheme in ("hadamard_int4", "int4", "int8"):
        qs = quantize_tensor(xt, scheme, group_size=16)
        fixtures[f"small_{scheme}_codes"] = qs.data.numpy()
        fixtures[f"small_{scheme}_scales"] = qs.scale.numpy()
    # exact .5 ties for the non-rotated schemes: amax 7 -> scale 1 -> values k + 0.5
    tie = torch.tensor([[7.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5, 0.0]])
    tie = tie.to(torch.bfloat16)
    fixtures["tie_x_bits"] = bf16_bits(tie)
    q4 = quantize_tensor(tie, "int4", group_size=16)
    fixtures["tie_int4_codes"] = q4.data.numpy()
    fixtures["tie_int4_scales"] = q4.scale.numpy()
    # RoPE keys as the cache quantizes them with quantize_rope=True (cache.py:160-164): [tokens, 64],
    # one group of 64, for both INT4 schemes
    g = torch.Generator().manual_seed(9)
    xr = (torch.randn(96, R, generator=g) * torch.linspace(0.1, 6.0, R)).to(torch.bfloat16)
    fixtures["rope_x_bits"] = bf16_bits(xr)
    for scheme in ("hadamard_int4", "int4"):
        qr = quantize_tensor(xr, scheme, group_size=64)
        fixtures[f"rope_{scheme}_codes"] = qr.data.numpy()
        fixtures[f"rope_{scheme}_scales"] = qr.scale.numpy().reshape(xr.shape[0])
    # float8 (kv.py:85-89: x.to(torch.float8_e4m3fn), no scales) from bf16 and from float32:
    # normal values, subnormals and their rounding ties, the top of the range (448 < |x| <= 464
    # rounds to 448, beyond it NaN), infinities, NaN and signed zeros
    g = torch.Generator().manual_seed(12)
    xf = torch.randn(64, 512, generator=g) * torch.logspace(-3, 2.5, 512)
    edge = torch.tensor([0.0, -0.0, 2.0 ** -10, -(2.0 ** -10), 3 * 2.0 ** -11, 2.0 ** -9, 1e-30, 447.0, 448.0,
                         456.0, 460.0, 464.0, 464.5, 470.0, 1e4, -1e4, float("inf"), float("-inf"), float("nan"),
                         1.0625, 1.1875, -1.0625, 0.01, -0.01, 240.0, 248.0, 232.0, 3.0e-3, -7.8e-3, 1.5, 2.5, 3.5])
    xf[0, : edge.numel()] = edge
    fixtures["f8_x_bits"] = bf16_bits(xf.to(torch.bfloat16))
    fixtures["f8_codes_bf16"] = quantize_tensor(xf.to(torch.bfloat16), "float8").data.view(torch.uint8).numpy()
    fixtures["f8_x_f32"] = xf.numpy()
    fixtures["f8_codes_f32"] = quantize_tensor(xf, "float8").data.view(torch.uint8).numpy()
    np.savez_compressed(HERE / "encode_golden.npz", **fixtures)

    # ---- decode -----------------------------------------------------------------
    cases = {
        # config 1 exactly: 8192 cached tokens -> 14 cold chunks + 1024 hot (recent 512, chunk 512)
        "c1": dict(seed=0, ctx=8192, q_len=1, recent=512, chunk=512),
        # one partial-free cold chunk + short hot window
        "small": dict(seed=3, ctx=1100, q_len=1, recent=512, chunk=512),
        # hot only (cache shorter than recent + chunk)
        "hotonly": dict(seed=4, ctx=700, q_len=1, recent=512, chunk=512),
        # q_len = 3 causal verification over a populated cache (config 5 shape)
        "t3": dict(seed=5, ctx=4096, q_len=3, recent=512, chunk=512),
        # quantize_rope=True: the cold chunks' RoPE keys quantized too (cache.py:160-164)
        "qrope": dict(seed=6, ctx=2200, q_len=1, recent=512, chunk=512, quantize_rope=True),
        "qr4": dict(seed=8, ctx=2700, q_len=1, recent=512, chunk=512, scheme="int4", quantize_rope=True),
        # int8 cold chunks (kv.py scheme "int8": one signed byte a dim, no rotation)
        "q8": dict(seed=10, ctx=2400, q_len=1, recent=512, chunk=512, scheme="int8"),
        "q8t3": dict(seed=11, ctx=1900, q_len=3, recent=512, chunk=512, scheme="int8"),
        # float8 cold chunks (kv.py:85-89: e4m3 values, no scales)
        "f8": dict(seed=13, ctx=2300, q_len=1, recent=512, chunk=512, scheme="float8"),
        "f8t3": dict(seed=14, ctx=1800, q_len=3, recent=512, chunk=512, scheme="float8"),
        # quantize_rope=True with the one-byte schemes (RoPE keys as int8 codes / e4m3 bytes)
        "q8r": dict(seed=15, ctx=2100, q_len=1, recent=512, chunk=512, scheme="int8", quantize_rope=True),
        "f8r": dict(seed=16, ctx=2500, q_len=1, recent=512, chunk=512, scheme="float8", quantize_rope=True),
    }
    dec: dict[str, np.ndarray] = {}
    for name, kw in cases.items():
        res = decode_case(**kw)
        for k, v in kw.items():
            dec[f"{name}_{k}"] = np.asarray(v)
        for k, v in res.items():
            dec[f"{name}_{k}"] = np.asarray(v)
        d = res["out_bf16"] - res["out_fp32"]
        print(name, "cold", res["cold_chunks"], "hot", res["hot_tokens"], "bf16-vs-fp32 relL2",
              float(np.linalg.norm(d) / np.linalg.norm(res["out_fp32"])))
    np.savez_compressed(HERE / "decode_golden.npz", **dec)
    print("softmax scale", 1 / math.sqrt(L + R))


if __name__ == "__main__":
    main()
