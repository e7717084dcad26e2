"""CPU oracle for AsterLM's Hadamard-INT4 latent-cache decode path.

TEST INFRASTRUCTURE ONLY.  This module is the checker the parity tests, the
``smoke()`` entry point and the ``cpu_baseline`` leg of ``bench.py`` compare the
CUDA kernels against.  Product code never imports it: the CUDA path fails
loudly when its extension is missing instead of falling back to this file.

It restates, in numpy, the reference's own algorithm (AsterLM-Frontier,
``src/asterlm``), step for step and in the same floating-point order where the
result is meant to be bit-exact:

* ``normalized_fwht``      quantization/kv.py:13-32
* ``pack_int4``            quantization/kv.py:41-48
* ``unpack_int4``          quantization/kv.py:51-55
* ``quantize``             quantization/kv.py:76-118 (the float8 scheme, kv.py:85-89, is torch's
                           own cast, which ``float8_bytes`` calls rather than restates)
* ``dequantize``           quantization/kv.py:121-134
* ``absorbed_decode``      layers/latent_attention.py:177-231 (q_len == 1)
* ``causal_attention``     layers/latent_attention.py:116-175 (q_len >= 1)

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree) on seeded inputs and stores its codes, scales
and decode outputs under ``tests/golden``; ``tests/test_oracle_golden.py``
checks this module against those fixtures (codes/scales bit-exact, decode
within float32 reassociation noise).

numpy has no bfloat16 type, so bfloat16 tensors travel as ``uint16`` bit
patterns and are widened exactly to float32 with ``bf16_to_f32``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# --------------------------------------------------------------------------
# bfloat16 helpers (exact widening; round-to-nearest-even narrowing like
# torch's float32 -> bfloat16 conversion)
# --------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    rounded = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    rounded[np.isnan(x)] = 0x7FC0
    return rounded


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Values of ``x`` rounded to bfloat16, returned as float32."""
    return bf16_to_f32(f32_to_bf16(x))


# --------------------------------------------------------------------------
# Quantizer (quantization/kv.py)
# --------------------------------------------------------------------------


def next_power_of_two(value: int) -> int:
    """quantization/kv.py:9-10."""
    return 1 if value <= 1 else 1 << (value - 1).bit_length()


def normalized_fwht(x: np.ndarray) -> np.ndarray:
    """Orthonormal Walsh-Hadamard transform over the last axis (kv.py:13-32).

    Stage h = 1, 2, 4, ... pairs element j with j + h inside blocks of 2h and
    replaces them by (a + b, a - b) (kv.py:24-31); the result is then divided by
    sqrt(n) as a float32 scalar (kv.py:32).  Every operation is a single IEEE
    float32 add, subtract or divide, so the output is bit-reproducible.
    """
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    if n & (n - 1):
        raise ValueError("FWHT length must be a power of two")
    y = x.reshape(-1, n)
    h = 1
    while h < n:
        blocks = y.reshape(-1, n // (2 * h), 2, h)
        a = blocks[:, :, 0, :]
        b = blocks[:, :, 1, :]
        y = np.stack((a + b, a - b), axis=2).reshape(-1, n)
        h *= 2
    return (y / np.float32(math.sqrt(n))).reshape(x.shape)


def _pad_last(x: np.ndarray, target: int) -> np.ndarray:
    """quantization/kv.py:35-38."""
    if x.shape[-1] == target:
        return x
    pad = [(0, 0)] * (x.ndim - 1) + [(0, target - x.shape[-1])]
    return np.pad(x, pad)


def pack_int4(values: np.ndarray) -> np.ndarray:
    """quantization/kv.py:41-48: u = q + 8, byte k = u[2k] | u[2k+1] << 4."""
    values = np.asarray(values).astype(np.int8)
    if values.shape[-1] % 2:
        values = _pad_last(values, values.shape[-1] + 1)
    unsigned = (np.clip(values, -7, 7) + 8).astype(np.uint8)
    return (unsigned[..., 0::2] | (unsigned[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray, width: int) -> np.ndarray:
    """quantization/kv.py:51-55: low nibble is the even index."""
    packed = np.asarray(packed, dtype=np.uint8)
    low = (packed & 0x0F).astype(np.int16) - 8
    high = ((packed >> 4) & 0x0F).astype(np.int16) - 8
    out = np.stack((low, high), axis=-1).reshape(*packed.shape[:-1], -1)
    return out[..., :width].astype(np.int8)


@dataclass
class Quantized:
    """Mirror of ``QuantizedTensor`` (kv.py:58-73)."""

    data: np.ndarray
    scale: np.ndarray | None
    original_shape: tuple[int, ...]
    padded_dim: int
    group_size: int
    scheme: str

    @property
    def num_bytes(self) -> int:
        total = self.data.nbytes
        if self.scale is not None:
            total += self.scale.nbytes
        return int(total)


def float8_bytes(x: np.ndarray) -> np.ndarray:
    """kv.py:85-89: ``x.to(torch.float8_e4m3fn)`` as raw bytes.  The reference's float8 scheme
    is torch's own cast (round to nearest even, NaN for |x| > 464 and non-finite values), so
    the oracle calls the same cast on the CPU rather than restating it."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32)))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def float8_values(codes: np.ndarray) -> np.ndarray:
    """The float32 values of e4m3 bytes (exact)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(codes, dtype=np.uint8))
    return t.view(torch.float8_e4m3fn).float().numpy()


def quantize(x: np.ndarray, scheme: str = "hadamard_int4", group_size: int = 64) -> Quantized:
    """Groupwise absmax quantizer (kv.py:76-118) for int8 / int4 / hadamard_int4, and the
    scale-free float8 cast (kv.py:85-89).

    ``x`` holds the source values already widened to float32 (the reference's
    ``x.float()``, kv.py:96).  The scale is ``amax(|g|).clamp_min(1e-8) / qmax``
    in float32 (kv.py:105-106); codes are ``round(g / scale)`` with
    round-half-to-even, clamped (kv.py:107); the stored scale is the float32
    scale rounded to float16 (kv.py:112).
    """
    if scheme == "float8":
        x = np.asarray(x, dtype=np.float32)
        return Quantized(data=float8_bytes(x), scale=None, original_shape=tuple(x.shape), padded_dim=x.shape[-1],
                         group_size=group_size, scheme=scheme)
    if scheme not in {"int8", "int4", "hadamard_int4"}:
        raise ValueError(f"unsupported quantization scheme: {scheme}")
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    x = np.asarray(x, dtype=np.float32)
    original_shape = tuple(x.shape)
    transformed = x
    padded_dim = x.shape[-1]
    if scheme == "hadamard_int4":
        padded_dim = next_power_of_two(x.shape[-1])
        transformed = normalized_fwht(_pad_last(transformed, padded_dim))
    padded_group_dim = math.ceil(transformed.shape[-1] / group_size) * group_size
    transformed = _pad_last(transformed, padded_group_dim)
    groups = transformed.reshape(*transformed.shape[:-1], -1, group_size)
    qmax = np.float32(127.0 if scheme == "int8" else 7.0)
    amax = np.abs(groups).max(axis=-1, keepdims=True)
    scale = np.maximum(amax, np.float32(1e-8)) / qmax
    quant = np.clip(np.rint(groups / scale), -qmax, qmax).astype(np.int8)
    flat = quant.reshape(*transformed.shape[:-1], padded_group_dim)
    data = flat if scheme == "int8" else pack_int4(flat)
    return Quantized(
        data=data,
        scale=scale.astype(np.float16),
        original_shape=original_shape,
        padded_dim=padded_dim,
        group_size=group_size,
        scheme=scheme,
    )


def dequantize(q: Quantized) -> np.ndarray:
    """kv.py:121-134, returning float32 (the oracle never narrows)."""
    if q.scheme == "float8":
        return float8_values(q.data).reshape(q.original_shape).astype(np.float32)
    if q.scale is None:
        raise RuntimeError("integer quantized tensor is missing scales")
    width = q.scale.shape[-2] * q.group_size
    values = q.data if q.scheme == "int8" else unpack_int4(q.data, width)
    groups = values.reshape(*values.shape[:-1], -1, q.group_size).astype(np.float32)
    restored = (groups * q.scale.astype(np.float32)).reshape(*values.shape[:-1], width)
    if q.scheme == "hadamard_int4":
        restored = normalized_fwht(restored[..., : q.padded_dim])
    restored = restored[..., : q.original_shape[-1]]
    return restored.reshape(q.original_shape).astype(np.float32)


# --------------------------------------------------------------------------
# Cache and decode (cache.py, layers/latent_attention.py)
# --------------------------------------------------------------------------


@dataclass
class ColdChunk:
    """One cold chunk: packed codes [n, D/2] u8, scales [n, D/G] f16, RoPE [n, R] f32.

    With ``quantize_rope`` (cache.py:160-164) the RoPE keys are stored like the latent
    (``rope_codes`` [n, R/2] u8 for INT4, [n, R] for int8 / float8; ``rope_scales`` [n] f16, one
    group of R = 64, none for float8) and ``rope``
    holds their dequantized values (kv.py:121-134), which is what ``iter_chunks`` yields.
    """

    codes: np.ndarray
    scales: np.ndarray
    rope: np.ndarray
    latent_dim: int
    group_size: int = 64
    scheme: str = "hadamard_int4"
    rope_codes: np.ndarray | None = None
    rope_scales: np.ndarray | None = None

    @property
    def length(self) -> int:
        return int(self.codes.shape[0])

    def dequantized_latent(self) -> np.ndarray:
        """Dequantize like ``iter_chunks`` (cache.py:143-148 -> kv.py:121-134)."""
        padded = next_power_of_two(self.latent_dim) if self.scheme == "hadamard_int4" else self.latent_dim
        q = Quantized(
            data=self.codes,
            scale=None if self.scales is None else self.scales.reshape(self.length, -1, 1),
            original_shape=(self.length, self.latent_dim),
            padded_dim=padded,
            group_size=self.group_size,
            scheme=self.scheme,
        )
        return dequantize(q)


@dataclass
class LatentCacheView:
    """Snapshot of one ``LatentLayerCache`` (cache.py:52-68) in float32."""

    cold: list[ColdChunk]
    hot_latent: np.ndarray  # [S_hot, L] float32
    hot_rope: np.ndarray  # [S_hot, R] float32

    @property
    def cold_length(self) -> int:
        return sum(c.length for c in self.cold)

    @property
    def length(self) -> int:
        return self.cold_length + int(self.hot_latent.shape[0])

    def iter_chunks(self):
        """cache.py:139-159: dequantized cold chunks in order, then the hot window."""
        for chunk in self.cold:
            yield chunk.dequantized_latent(), chunk.rope.astype(np.float32)
        if self.hot_latent.shape[0]:
            yield self.hot_latent.astype(np.float32), self.hot_rope.astype(np.float32)

    def materialize(self) -> tuple[np.ndarray, np.ndarray]:
        """cache.py:89-137 (``materialize_latent`` / ``materialize_rope``)."""
        lat = [lat for lat, _ in self.iter_chunks()]
        rope = [rope for _, rope in self.iter_chunks()]
        if not lat:
            dim_l = self.hot_latent.shape[-1]
            dim_r = self.hot_rope.shape[-1]
            return np.zeros((0, dim_l), np.float32), np.zeros((0, dim_r), np.float32)
        return np.concatenate(lat, axis=0), np.concatenate(rope, axis=0)


def absorbed_decode(
    q_lat: np.ndarray,
    q_rope: np.ndarray,
    new_latent: np.ndarray,
    new_rope: np.ndarray,
    cache: LatentCacheView,
    softmax_scale: float,
    logit_softcap: float | None = None,
) -> np.ndarray:
    """One-token absorbed decode with online softmax (latent_attention.py:177-231).

    Inputs are one sequence's float32 tensors: ``q_lat`` [1, H, L] (the
    absorbed query ``q_content @ W_k``, latent_attention.py:188), ``q_rope``
    [1, H, R], the new token's ``new_latent`` [1, L] and ``new_rope`` [1, R].
    Chunks are consumed cold-first, then the hot window, then the new token
    itself (:222-227).  Returns the context latent [1, H, L] in float32, i.e.
    ``running_context / running_sum.clamp_min(1e-20)`` (:229) before the value
    up-projection, which is a caller-side GEMM.
    """
    q_lat = np.asarray(q_lat, np.float32)
    q_rope = np.asarray(q_rope, np.float32)
    scale = np.float32(softmax_scale)
    running_max = running_sum = running_ctx = None

    def consume(chunk_latent: np.ndarray, chunk_rope: np.ndarray) -> None:
        nonlocal running_max, running_sum, running_ctx
        scores = (np.einsum("thl,sl->hts", q_lat, chunk_latent) + np.einsum("thr,sr->hts", q_rope, chunk_rope)) * scale
        if logit_softcap is not None:
            cap = np.float32(logit_softcap)
            scores = cap * np.tanh(scores / cap)
        chunk_max = scores.max(axis=-1)
        if running_max is None:
            running_max = chunk_max
            p = np.exp(scores - running_max[..., None])
            running_sum = p.sum(axis=-1)
            running_ctx = np.einsum("hts,sl->htl", p, chunk_latent)
            return
        new_max = np.maximum(running_max, chunk_max)
        old_scale = np.exp(running_max - new_max)
        p = np.exp(scores - new_max[..., None])
        running_sum = running_sum * old_scale + p.sum(axis=-1)
        running_ctx = running_ctx * old_scale[..., None] + np.einsum("hts,sl->htl", p, chunk_latent)
        running_max = new_max

    for chunk_latent, chunk_rope in cache.iter_chunks():
        consume(chunk_latent, chunk_rope)
    consume(np.asarray(new_latent, np.float32), np.asarray(new_rope, np.float32))
    ctx = running_ctx / np.maximum(running_sum, np.float32(1e-20))[..., None]
    return ctx.transpose(1, 0, 2).astype(np.float32)  # [T, H, L]


def causal_attention(
    q_lat: np.ndarray,
    q_rope: np.ndarray,
    new_latent: np.ndarray,
    new_rope: np.ndarray,
    cache: LatentCacheView,
    softmax_scale: float,
    logit_softcap: float | None = None,
) -> np.ndarray:
    """q_len >= 1 attention over cache + new tokens (latent_attention.py:116-175).

    The reference materializes the cache (:126-130), up-projects keys and values
    per head and applies the causal mask ``k_index <= past_len + q_index``
    (:151-153).  With keys expressed through the absorbed query (the kernel's
    contract: scores ``q_lat . latent + q_rope . rope``) this is the same
    computation; the output is the context latent [T, H, L] in float32.
    """
    q_lat = np.asarray(q_lat, np.float32)
    q_rope = np.asarray(q_rope, np.float32)
    past_lat, past_rope = cache.materialize()
    all_lat = np.concatenate((past_lat, np.asarray(new_latent, np.float32)), axis=0)
    all_rope = np.concatenate((past_rope, np.asarray(new_rope, np.float32)), axis=0)
    past_len = past_lat.shape[0]
    t_len = q_lat.shape[0]
    scores = (np.einsum("thl,sl->hts", q_lat, all_lat) + np.einsum("thr,sr->hts", q_rope, all_rope)) * np.float32(
        softmax_scale
    )
    if logit_softcap is not None:
        cap = np.float32(logit_softcap)
        scores = cap * np.tanh(scores / cap)
    k_index = np.arange(all_lat.shape[0])[None, :]
    q_index = np.arange(t_len)[:, None]
    allowed = k_index <= (past_len + q_index)
    scores = np.where(allowed[None], scores, np.float32(-np.inf))
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.einsum("hts,sl->htl", p, all_lat)
    return out.transpose(1, 0, 2).astype(np.float32)


def decode(q_lat, q_rope, new_latent, new_rope, cache, softmax_scale, logit_softcap=None):
    """Dispatch like ``LatentAttention.forward`` (latent_attention.py:241-244)."""
    if q_lat.shape[0] == 1 and cache.length:
        return absorbed_decode(q_lat, q_rope, new_latent, new_rope, cache, softmax_scale, logit_softcap)
    return causal_attention(q_lat, q_rope, new_latent, new_rope, cache, softmax_scale, logit_softcap)


def partial_attention(
    q_lat: np.ndarray,
    q_rope: np.ndarray,
    chunks: list[tuple[np.ndarray, np.ndarray]],
    softmax_scale: float,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Unnormalised softmax state over a subset of one sequence's keys.

    Returns (m [T, H], l [T, H], o [T, H, L]) with m the score maximum, l the sum
    of exp(s - m) and o the exp(s - m)-weighted sum of latents: the running
    state of latent_attention.py:203-220 after consuming only `chunks`
    (latent [n, L], rope [n, R] pairs).  An empty subset gives (-inf, 0, 0).
    """
    q_lat = np.asarray(q_lat, np.float32)
    q_rope = np.asarray(q_rope, np.float32)
    t, h, dim = q_lat.shape
    if not chunks:
        return (np.full((t, h), -np.inf, np.float32), np.zeros((t, h), np.float32), np.zeros((t, h, dim), np.float32))
    lat = np.concatenate([c[0] for c in chunks]).astype(np.float32)
    rope = np.concatenate([c[1] for c in chunks]).astype(np.float32)
    s = (np.einsum("thl,sl->ths", q_lat, lat) + np.einsum("thr,sr->ths", q_rope, rope)) * np.float32(softmax_scale)
    m = s.max(axis=-1)
    p = np.exp(s - m[..., None])
    return m, p.sum(axis=-1), np.einsum("ths,sl->thl", p, lat)


def merge_partials(parts: list[tuple[np.ndarray, np.ndarray, np.ndarray]]) -> np.ndarray:
    """Combine partial states with the online-softmax rule (latent_attention.py:212-220); returns o / max(l, 1e-20)."""
    m = np.max(np.stack([p[0] for p in parts]), axis=0)
    msub = np.where(np.isneginf(m), 0.0, m)
    l = np.zeros_like(parts[0][1])
    o = np.zeros_like(parts[0][2])
    for pm, pl, po in parts:
        w = np.exp(pm - msub)
        l += w * pl
        o += w[..., None] * po
    return (o / np.maximum(l, np.float32(1e-20))[..., None]).astype(np.float32)


def cold_chunk(latent: np.ndarray, rope: np.ndarray, group_size: int = 64, scheme: str = "hadamard_int4",
               quantize_rope: bool = False) -> ColdChunk:
    """``LatentLayerCache._encode`` of one chunk (cache.py:160-164): the latent always, the RoPE
    keys only with ``quantize_rope`` (else kept as they are)."""
    q = quantize(latent, scheme, group_size)
    scales = None if q.scale is None else q.scale.reshape(latent.shape[0], -1)
    chunk = ColdChunk(codes=q.data, scales=scales, rope=rope.copy(),
                      latent_dim=latent.shape[-1], group_size=group_size, scheme=scheme)
    if quantize_rope:
        qr = quantize(rope, scheme, group_size)
        chunk.rope_codes = qr.data
        chunk.rope_scales = None if qr.scale is None else qr.scale.reshape(rope.shape[0])
        chunk.rope = dequantize(qr)
    return chunk


def build_cache_from_tokens(
    latent: np.ndarray,
    rope: np.ndarray,
    recent_tokens: int,
    chunk_tokens: int,
    group_size: int = 64,
    scheme: str = "hadamard_int4",
    quantize_rope: bool = False,
) -> LatentCacheView:
    """Replay ``LatentLayerCache.append`` + ``_flush_cold_chunks`` (cache.py:167-201).

    The whole history is appended at once (window_size=None); while the hot
    window is longer than ``recent + chunk``, its oldest ``chunk`` tokens are
    encoded into a cold chunk (cache.py:170-177).  ``latent``/``rope`` are the
    bfloat16 values widened to float32.
    """
    latent = np.asarray(latent, np.float32)
    rope = np.asarray(rope, np.float32)
    threshold = recent_tokens + chunk_tokens
    cold: list[ColdChunk] = []
    start = 0
    while latent.shape[0] - start > threshold:
        cold.append(cold_chunk(latent[start : start + chunk_tokens], rope[start : start + chunk_tokens], group_size,
                               scheme, quantize_rope))
        start += chunk_tokens
    return LatentCacheView(cold=cold, hot_latent=latent[start:].copy(), hot_rope=rope[start:].copy())


def build_cache_split(
    latent: np.ndarray,
    rope: np.ndarray,
    hot_tokens: int,
    chunk_tokens: int,
    group_size: int = 64,
    scheme: str = "hadamard_int4",
    quantize_rope: bool = False,
) -> LatentCacheView:
    """Cold/hot split used by the ragged workloads: the newest ``hot_tokens``
    stay hot, the rest is cut oldest-first into ``chunk_tokens`` chunks whose
    newest one may be partial (``_piece_length``/``iter_chunks`` handle partial
    chunks, cache.py:17-19, 139-159)."""
    latent = np.asarray(latent, np.float32)
    rope = np.asarray(rope, np.float32)
    n = latent.shape[0]
    n_cold = max(0, n - hot_tokens)
    cold = []
    for start in range(0, n_cold, chunk_tokens):
        end = min(start + chunk_tokens, n_cold)
        cold.append(cold_chunk(latent[start:end], rope[start:end], group_size, scheme, quantize_rope))
    return LatentCacheView(cold=cold, hot_latent=latent[n_cold:].copy(), hot_rope=rope[n_cold:].copy())


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def decode_sequence(latent: np.ndarray, rope: np.ndarray, q_lat: np.ndarray, q_rope: np.ndarray, n: int, hot: int,
                    softmax_scale: float, chunk: int = 512, scheme: str = "hadamard_int4",
                    quantize_rope: bool = False) -> np.ndarray:
    """One sequence of a ragged batch: tokens [0, n) are the cache (the newest ``hot`` in the hot
    window, older ones in ``chunk``-token cold chunks, the newest possibly partial), tokens
    [n, n + q_len) the step's new tokens; returns the context latents [q_len, H, 512]
    (latent_attention.py:177-231 for q_len 1, :116-175 otherwise).  A module-level function so
    that a process pool can run sequences in parallel."""
    latent = np.asarray(latent, dtype=np.float32)
    rope = np.asarray(rope, dtype=np.float32)
    cache = build_cache_split(latent[:n], rope[:n], hot, chunk, scheme=scheme, quantize_rope=quantize_rope)
    return decode(np.asarray(q_lat, np.float32), np.asarray(q_rope, np.float32), latent[n:], rope[n:], cache,
                  softmax_scale)
