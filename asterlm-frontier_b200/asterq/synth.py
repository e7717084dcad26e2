"""Seeded synthetic decode workloads with the BASELINE configs' shapes.

Latents and queries are N(0, 1); 1% of the latent channels (5 of 512) are
scaled x20 as outliers; everything is rounded to bfloat16.  The reference
publishes no dataset for this path, so these seeded tensors stand in for real
activations.  Cold chunks are encoded with the product write-path kernel.

* ``c1_inputs``: the reference's own CPU-runnable case (CPU torch generator,
  reproducible without a GPU): B=1, 8192 cached tokens, q_len 1.
* ``make_workload``: ragged batches built on the GPU (configs 3, 4, 5).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .decode import GROUP_SIZE, LATENT_DIM, ROPE_DIM, LatentPools
from .plan import SequenceLayout

OUTLIER_FRACTION = 0.01
OUTLIER_SCALE = 20.0


def outlier_channels(seed: int, dim: int = LATENT_DIM) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(dim, generator=g)[: max(1, round(OUTLIER_FRACTION * dim))]


def c1_inputs(seed: int = 0, ctx: int = 8192, q_len: int = 1, n_heads: int = 16) -> dict[str, torch.Tensor]:
    """Config 1 on the CPU: latents [ctx + q_len, 512], RoPE keys [ctx + q_len, 64],
    q_lat [q_len, H, 512], q_rope [q_len, H, 64], all bfloat16.  The last q_len
    tokens are the step's new tokens."""
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(1, ctx + q_len, LATENT_DIM, generator=g)
    out_ch = torch.randperm(LATENT_DIM, generator=g)[: max(1, round(OUTLIER_FRACTION * LATENT_DIM))]
    lat[..., out_ch] *= OUTLIER_SCALE
    lat = lat.to(torch.bfloat16)
    rope = torch.randn(1, ctx + q_len, ROPE_DIM, generator=g).to(torch.bfloat16)
    q_lat = torch.randn(1, q_len, n_heads, LATENT_DIM, generator=g).to(torch.bfloat16)
    q_rope = torch.randn(1, q_len, n_heads, ROPE_DIM, generator=g).to(torch.bfloat16)
    return {"latent": lat[0], "rope": rope[0], "q_lat": q_lat[0], "q_rope": q_rope[0]}


@dataclass
class Workload:
    name: str
    n_heads: int
    q_len: int
    lengths: list[int]  # cached tokens per sequence (excluding the new ones)
    hot: list[int]
    pools: LatentPools
    layouts: list[SequenceLayout]
    q_lat: torch.Tensor
    q_rope: torch.Tensor
    new_latent: torch.Tensor
    new_rope: torch.Tensor
    host: dict[int, dict[str, torch.Tensor]] = field(default_factory=dict)  # kept sequences (CPU bf16)

    @property
    def total_q(self) -> int:
        return int(self.q_lat.shape[0])

    def algorithmic_bytes(self) -> int:
        """HBM bytes one decode step must read/write (each byte once)."""
        cold = sum(n - h for n, h in zip(self.lengths, self.hot))
        hot = sum(self.hot) + self.total_q
        per_q = self.n_heads * (LATENT_DIM + ROPE_DIM) * 2 + self.n_heads * LATENT_DIM * 2
        rope = (ROPE_DIM // 2 + 2) if self.pools.rope_quantized else ROPE_DIM * 2  # codes + scale, or bf16
        codes = int(self.pools.cold_codes.shape[-1])  # 256 (INT4) or 512 (int8, float8)
        scales = 2 * int(self.pools.cold_scales.shape[-1])  # 16, or 0 for float8
        return cold * (codes + scales + rope) + hot * (1024 + 128) + self.total_q * per_q

    def flops(self) -> int:
        """Useful multiply-adds x 2 (QK over 576 dims + PV over 512) for all rows."""
        total = 0
        for n in self.lengths:
            total += self.q_len * self.n_heads * (n + self.q_len) * 2 * (LATENT_DIM + ROPE_DIM + LATENT_DIM)
        return total


def c3_lengths(seed: int = 0, n: int = 64) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1024, 32769, (n,), generator=g).tolist()


def c5_lengths(seed: int = 0, n: int = 256) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(4096, 65537, (n,), generator=g).tolist()


class PoolBuilder:
    """Fill pools sequence by sequence from BF16 tokens already on the device.

    Sequence tokens are ``[n + q_len]`` rows: the first ``n`` are the cache, the
    last ``q_len`` the step's new tokens.  The newest ``hot`` cached tokens stay
    BF16 in hot pages; older ones are cut oldest-first into ``page_tokens``
    chunks (the newest possibly partial) and encoded with the write-path kernel.
    """

    def __init__(self, lengths, hot, *, q_len, n_heads, page_tokens=512, device="cuda", scheme="hadamard_int4",
                 quantize_rope=False):
        from . import _lib

        self._lib = _lib
        self.lib = _lib.load()
        self.device = torch.device(device)
        self.q_len, self.n_heads, self.page_tokens = q_len, n_heads, page_tokens
        self.lengths, self.hot = list(lengths), list(hot)
        n_cold_pages = sum(math.ceil(max(0, n - h) / page_tokens) for n, h in zip(lengths, hot))
        n_hot_pages = sum(math.ceil(h / page_tokens) for h in hot)
        # quantize_rope: cold RoPE keys encoded like the latent (cold scheme, one group of 64)
        self.pools = LatentPools.empty(n_cold_pages, n_hot_pages, page_tokens, self.device, quantize_rope=quantize_rope,
                                       cold_scheme=scheme)
        self._scheme_id = {"hadamard_int4": _lib.SCHEME_HADAMARD_INT4, "int4": _lib.SCHEME_INT4,
                           "int8": _lib.SCHEME_INT8, "float8": _lib.SCHEME_FLOAT8}[scheme]
        total_q = len(self.lengths) * q_len
        dev = self.device
        self.q_lat = torch.zeros(total_q, n_heads, LATENT_DIM, dtype=torch.bfloat16, device=dev)
        self.q_rope = torch.zeros(total_q, n_heads, ROPE_DIM, dtype=torch.bfloat16, device=dev)
        self.new_latent = torch.zeros(total_q, LATENT_DIM, dtype=torch.bfloat16, device=dev)
        self.new_rope = torch.zeros(total_q, ROPE_DIM, dtype=torch.bfloat16, device=dev)
        self.layouts: list[SequenceLayout] = []
        self._cold_page = 0
        self._hot_page = 0

    def add(self, lat: torch.Tensor, rope: torch.Tensor, q_lat: torch.Tensor, q_rope: torch.Tensor) -> None:
        i = len(self.layouts)
        n, h, q_len, P = self.lengths[i], self.hot[i], self.q_len, self.page_tokens
        if not 0 <= h <= n:
            raise ValueError("hot tokens must be within the sequence length")
        if lat.shape != (n + q_len, LATENT_DIM) or rope.shape != (n + q_len, ROPE_DIM):
            raise ValueError("token tensors must be [n + q_len, 512] / [n + q_len, 64]")
        lat = lat.to(self.device, torch.bfloat16).contiguous()
        rope = rope.to(self.device, torch.bfloat16).contiguous()
        pools = self.pools
        cold = n - h
        lay = SequenceLayout(q_start=i * q_len, q_len=q_len)
        if cold:
            r0 = self._cold_page * P
            codes = pools.cold_codes.view(-1, pools.cold_codes.shape[-1])
            n_scales = int(pools.cold_scales.shape[-1])  # 0 for float8 (no scales)
            scales_ptr = pools.cold_scales.view(-1, n_scales)[r0].data_ptr() if n_scales else None
            self._lib.check(
                self.lib.asterq_quantize(
                    lat.data_ptr(), self._lib.DTYPE_BF16, cold, LATENT_DIM, LATENT_DIM,
                    self._scheme_id, GROUP_SIZE, codes[r0].data_ptr(), scales_ptr,
                    self._lib.stream_handle(self.device),
                )
            )
            if pools.rope_quantized:
                self._lib.check(
                    self.lib.asterq_quantize(
                        rope.data_ptr(), self._lib.DTYPE_BF16, cold, ROPE_DIM, ROPE_DIM, self._scheme_id, GROUP_SIZE,
                        pools.cold_rope.view(-1, pools.cold_rope.shape[-1])[r0].data_ptr(),
                        None if pools.cold_rope_scales is None else pools.cold_rope_scales.view(-1)[r0:].data_ptr(),
                        self._lib.stream_handle(self.device),
                    )
                )
            else:
                pools.cold_rope.view(-1, ROPE_DIM)[r0 : r0 + cold].copy_(rope[:cold])
            for s in range(0, cold, P):
                lay.cold.append((self._cold_page, 0, min(P, cold - s)))
                self._cold_page += 1
        if h:
            r0 = self._hot_page * P
            pools.hot_latent.view(-1, LATENT_DIM)[r0 : r0 + h].copy_(lat[cold:n])
            pools.hot_rope.view(-1, ROPE_DIM)[r0 : r0 + h].copy_(rope[cold:n])
            for s in range(0, h, P):
                lay.hot.append((self._hot_page, 0, min(P, h - s)))
                self._hot_page += 1
        sl = slice(i * q_len, (i + 1) * q_len)
        self.q_lat[sl].copy_(q_lat.reshape(q_len, self.n_heads, LATENT_DIM))
        self.q_rope[sl].copy_(q_rope.reshape(q_len, self.n_heads, ROPE_DIM))
        self.new_latent[sl].copy_(lat[n:])
        self.new_rope[sl].copy_(rope[n:])
        self.layouts.append(lay)

    def finish(self, name: str, host=None) -> "Workload":
        if len(self.layouts) != len(self.lengths):
            raise RuntimeError("not every sequence was added")
        return Workload(name, self.n_heads, self.q_len, self.lengths, self.hot, self.pools, self.layouts,
                        self.q_lat, self.q_rope, self.new_latent, self.new_rope, host or {})


def make_workload(
    name: str,
    lengths: list[int],
    hot: list[int],
    *,
    q_len: int = 1,
    n_heads: int = 16,
    seed: int = 0,
    device="cuda",
    page_tokens: int = 512,
    keep_host: set[int] | None = None,
    quantize_rope: bool = False,
    scheme: str = "hadamard_int4",
) -> Workload:
    """Generate every sequence on the device and build its pools.

    ``keep_host``: indices whose BF16 tokens are copied to the CPU for the oracle.
    """
    device = torch.device(device)
    keep_host = keep_host or set()
    b = PoolBuilder(lengths, hot, q_len=q_len, n_heads=n_heads, page_tokens=page_tokens, device=device,
                    quantize_rope=quantize_rope, scheme=scheme)
    host: dict[int, dict[str, torch.Tensor]] = {}
    for i, lat, rope, ql, qr in generate_sequences(lengths, q_len=q_len, n_heads=n_heads, seed=seed, device=device):
        b.add(lat, rope, ql, qr)
        if i in keep_host:
            host[i] = {"latent": lat.cpu(), "rope": rope.cpu(), "q_lat": ql.cpu(), "q_rope": qr.cpu()}
    return b.finish(name, host)


def generate_sequences(lengths, *, q_len: int = 1, n_heads: int = 16, seed: int = 0, device="cuda"):
    """The seeded tensors of a batch, sequence by sequence, in the order every workload draws them:
    yields (index, latent [n + q_len, 512], rope [n + q_len, 64], q_lat [q_len, H, 512],
    q_rope [q_len, H, 64]), bfloat16 on `device`; the last q_len tokens are the step's new tokens."""
    device = torch.device(device)
    out_ch = outlier_channels(seed).to(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    for i, n in enumerate(lengths):
        lat = torch.randn(n + q_len, LATENT_DIM, generator=gen, device=device)
        lat[:, out_ch] *= OUTLIER_SCALE
        lat = lat.to(torch.bfloat16)
        rope = torch.randn(n + q_len, ROPE_DIM, generator=gen, device=device).to(torch.bfloat16)
        ql = torch.randn(q_len, n_heads, LATENT_DIM, generator=gen, device=device).to(torch.bfloat16)
        qr = torch.randn(q_len, n_heads, ROPE_DIM, generator=gen, device=device).to(torch.bfloat16)
        yield i, lat, rope, ql, qr


def host_sequences(lengths, indices, *, q_len: int = 1, n_heads: int = 16, seed: int = 0, device="cuda"):
    """CPU copies of the sequences `indices` of a seeded batch, without building any pool
    (no asterq kernel runs): the inputs of a CPU baseline on exactly the tensors the GPU times."""
    want = set(indices)
    out = {}
    for i, lat, rope, ql, qr in generate_sequences(lengths, q_len=q_len, n_heads=n_heads, seed=seed, device=device):
        if i in want:
            out[i] = {"latent": lat.cpu(), "rope": rope.cpu(), "q_lat": ql.cpu(), "q_rope": qr.cpu()}
        if len(out) == len(want):
            break
    return out


def make_shard_workload(
    name: str,
    lengths: list[int],
    hot: list[int],
    shard: list[int],
    *,
    q_len: int = 1,
    n_heads: int = 16,
    seed: int = 0,
    device="cuda",
    page_tokens: int = 512,
    keep_host: set[int] | None = None,
    scheme: str = "hadamard_int4",
    quantize_rope: bool = False,
) -> Workload:
    """The sequences `shard` (indices into `lengths`) of a seeded batch, with pools for them
    only: every rank of a sequence-sharded job draws the whole batch from the same seed and
    keeps its own sequences, so the shards together are exactly the one-GPU batch.
    ``keep_host`` indices are batch indices; ``Workload.host`` is keyed by position in the shard."""
    device = torch.device(device)
    pos = {gi: k for k, gi in enumerate(shard)}
    b = PoolBuilder([lengths[i] for i in shard], [hot[i] for i in shard], q_len=q_len, n_heads=n_heads,
                    page_tokens=page_tokens, device=device, scheme=scheme, quantize_rope=quantize_rope)
    keep_host = keep_host or set()
    host: dict[int, dict[str, torch.Tensor]] = {}
    pending: dict[int, tuple] = {}
    for i, lat, rope, ql, qr in generate_sequences(lengths, q_len=q_len, n_heads=n_heads, seed=seed, device=device):
        if i not in pos:
            continue
        pending[pos[i]] = (lat, rope, ql, qr)
        if i in keep_host:
            host[pos[i]] = {"latent": lat.cpu(), "rope": rope.cpu(), "q_lat": ql.cpu(), "q_rope": qr.cpu()}
        while len(b.layouts) in pending:  # add in shard order
            b.add(*pending.pop(len(b.layouts)))
    return b.finish(name, host)


def c3_workload(device="cuda", seed: int = 0, n_seqs: int = 64, keep_host=None, quantize_rope: bool = False,
                scheme: str = "hadamard_int4") -> Workload:
    lens = c3_lengths(seed, n_seqs)
    return make_workload("C3 ragged decode", lens, [min(n, 2048) for n in lens], q_len=1, seed=seed, device=device,
                         keep_host=keep_host, quantize_rope=quantize_rope, scheme=scheme)


def c5_workload(device="cuda", seed: int = 0, n_seqs: int = 256, keep_host=None) -> Workload:
    lens = c5_lengths(seed, n_seqs)
    return make_workload("C5 MTP verification", lens, [min(n, 2048) for n in lens], q_len=3, seed=seed,
                         device=device, keep_host=keep_host)


def c4_workload(device="cuda", seed: int = 0, keep_host=None) -> Workload:
    return make_workload("C4 long context", [131072], [4096], q_len=1, seed=seed, device=device, keep_host=keep_host)
