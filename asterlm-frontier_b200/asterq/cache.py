"""Drop-in for AsterLM's latent cache (src/asterlm/cache.py) on paged device pools.

``LatentLayerCache`` keeps the reference's fields, properties and methods
(cache.py:52-221): ``length``, ``cold_length``, ``num_bytes``, ``append``,
``iter_chunks``, ``materialize_latent`` / ``materialize_rope`` and the
``latent`` / ``rope_key`` / ``cold_latent`` / ``cold_rope`` pieces.  Storage is
different: every batch row's tokens live in fixed-size pages of two pools
(``chunk_tokens`` tokens per page),

* hot pages: bf16 latent [page, 512] + bf16 RoPE key [page, 64],
* cold pages: INT4 codes [page, 256] + fp16 scales [page, 8] + bf16 RoPE key,

so that appending writes the new token in place (no re-concatenation of the
hot window, cache.py:195-200) and a flush (cache.py:167-177) encodes the oldest
full hot page of every row straight into a cold page with the write-path kernel
and releases the hot page.  The page lists are mirrored in device page tables
(``device_tables``), rebuilt only when pages change: bf16 appends run the in-place
append kernel on them, and ``asterq.attention.latent_attention`` plans each step on
the GPU from them (``device_planner``), so a decode step needs no host schedule, no
host index tensors and no per-call allocation.  Nothing is materialized on the
decode path.

The hot window holds at most ``recent_tokens + chunk_tokens`` tokens, exactly as
in the reference: after every append, whole chunks move from the front of the
hot window to the cold pool while the hot length exceeds that threshold.

The hot window keeps the caller's dtype (cache.py:193-200 stores the appended
tensors as they come): a caller appending float32 (or float16) latents gets them
back from ``latent`` / ``materialize_*`` unchanged, and flushed chunks are
quantized from those values (cache.py:172, bit-exact codes and scales).  The
decode kernel reads bf16 operands, so for such callers the hot pages also hold
a bf16 copy that only the kernel reads (bf16 rounding of the hot keys and
values, like the bf16 rounding of the query).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from . import _lib
from .decode import COLD_TILE_TOKENS, GROUP_SIZE, LATENT_DIM, ROPE_DIM, LatentPools
from .kv import QuantizedTensor, dequantize_tensor
from .plan import SequenceLayout

_KERNEL_SCHEMES = ("hadamard_int4", "int4", "int8", "float8", "bfloat16")
_SCHEME_IDS = {"hadamard_int4": _lib.SCHEME_HADAMARD_INT4, "int4": _lib.SCHEME_INT4, "int8": _lib.SCHEME_INT8,
               "float8": _lib.SCHEME_FLOAT8}
# code storage of the one-byte schemes (else packed INT4 bytes, uint8); float8 pages hold the raw
# e4m3 bytes (torch has no float8 page copies) and are viewed as float8_e4m3fn when handed out
_CODE_DTYPES = {"int8": torch.int8, "float8": torch.uint8}


class _Pool:
    """Growable set of equally sized pages with a free list (one tensor per field)."""

    def __init__(self, fields: dict[str, tuple[tuple[int, ...], torch.dtype]], page_tokens: int, device) -> None:
        self.fields = fields
        self.page_tokens = page_tokens
        self.device = torch.device(device)
        self.capacity = 0
        self.tensors = {name: torch.empty((0, page_tokens, *shape), dtype=dt, device=self.device)
                        for name, (shape, dt) in fields.items()}
        self.free: list[int] = []

    def alloc(self, n: int) -> list[int]:
        while len(self.free) < n:
            self._grow(max(n - len(self.free), self.capacity))
        out, self.free = self.free[:n], self.free[n:]
        return out

    def release(self, pages: list[int]) -> None:
        self.free.extend(pages)
        self.free.sort()

    def _grow(self, extra: int) -> None:
        extra = max(extra, 4)
        for name, (shape, dt) in self.fields.items():
            new = torch.empty((self.capacity + extra, self.page_tokens, *shape), dtype=dt, device=self.device)
            if self.capacity:
                new[: self.capacity].copy_(self.tensors[name])
            self.tensors[name] = new
        self.free.extend(range(self.capacity, self.capacity + extra))
        self.capacity += extra

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.tensors[name]


def trim_page_range(n_cold: int, cold_tokens, hot_tokens: int, page_tokens: int, window_size: int,
                    sink_tokens: int) -> tuple[int, int] | None:
    """The cold pages [a, b) a whole-page window trim drops, or None: pages [0, a) hold the first
    min(sink, window) tokens (the sink), pages [b, n_cold) with the hot window hold at least the
    last window - sink tokens (cache.py:210-219 keeps exactly these token ranges)."""
    sink = min(sink_tokens, window_size)
    recent = window_size - sink
    a, held = 0, 0
    while a < n_cold and held < sink:
        held += int(cold_tokens[a])
        a += 1
    b, back = n_cold, hot_tokens
    while b > a and back < recent:
        b -= 1
        back += int(cold_tokens[b])
    return (a, b) if b > a else None


@dataclass
class LatentLayerCache:
    """Hot/cold latent cache for one global-attention layer (cache.py:52).

    Same constructor fields and defaults as the reference.  The decode kernels
    serve ``cache_dtype`` "hadamard_int4", "int4" and "int8" (cold chunks; int8 codes are one
    signed byte a dim, 512 bytes a token) and "bfloat16" (never flushes, cache.py:169);
    ``group_size`` must be 64.  With ``quantize_rope`` (INT4 schemes) the cold chunks' RoPE
    keys are quantized with the cold scheme as well (cache.py:160-164: one group of 64, 32
    code bytes and one fp16 scale per token), and the kernel scores those codes directly.
    """

    cache_dtype: str = "bfloat16"
    group_size: int = 64
    recent_tokens: int = 512
    chunk_tokens: int = 1024
    quantize_rope: bool = False
    # window trimming (cache.py:203-221): "requantize" keeps exactly sink + recent tokens and
    # re-encodes them, as the reference does (double quantization); "pages" drops whole cold
    # pages between the sink and the recent tokens instead, with no re-quantization (up to a page
    # more on each side is kept, and a window shorter than the hot window keeps the hot window)
    trim_mode: str = "requantize"
    _batch: int = field(default=0, repr=False)
    _hot_len: int = field(default=0, repr=False)
    _hot_pages: list[list[int]] = field(default_factory=list, repr=False)
    _cold_pages: list[list[int]] = field(default_factory=list, repr=False)
    _hot: _Pool | None = field(default=None, repr=False)
    _cold: _Pool | None = field(default=None, repr=False)
    _dtype: torch.dtype = field(default=torch.bfloat16, repr=False)
    # device page tables mirroring the page lists (asterq.batch.BatchTables), rebuilt only when
    # pages change, with the GPU planner bound to them: appends and attention need no host
    # plan, host index tensors or per-call allocations
    _dev: Any = field(default=None, repr=False)

    def __post_init__(self) -> None:
        if self.cache_dtype not in _KERNEL_SCHEMES:
            raise NotImplementedError(
                f"cache_dtype {self.cache_dtype!r}: the asterq pools serve 'hadamard_int4', 'int4' and 'bfloat16'")
        if self.cache_dtype in _SCHEME_IDS and self.cache_dtype != "float8" and self.group_size != GROUP_SIZE:
            raise NotImplementedError(f"group_size {self.group_size}: the decode kernels use groups of {GROUP_SIZE}")
        if self.chunk_tokens <= 0 or self.chunk_tokens % 16:
            raise ValueError("chunk_tokens must be a positive multiple of 16 (one chunk per page)")
        if self.recent_tokens < 0:
            raise ValueError("recent_tokens must be non-negative")
        if self.trim_mode not in ("requantize", "pages"):
            raise ValueError("trim_mode must be 'requantize' or 'pages'")

    # ------------------------------------------------------------------ sizes
    @property
    def page_tokens(self) -> int:
        return self.chunk_tokens

    @property
    def batch_size(self) -> int:
        return self._batch

    @property
    def cold_chunks(self) -> int:
        return len(self._cold_pages[0]) if self._cold_pages else 0

    @property
    def cold_length(self) -> int:
        return self.cold_chunks * self.chunk_tokens

    @property
    def hot_length(self) -> int:
        return self._hot_len

    @property
    def length(self) -> int:
        return self.cold_length + self._hot_len

    @property
    def num_bytes(self) -> int:
        """Bytes the reference would account (cache.py:79-87): codes + scales + cold RoPE + hot tensors."""
        b, cold = self._batch, self.cold_length
        # RoPE: codes + scale (none for float8), or bf16
        rope = (self._rope_code_bytes + (self.cache_dtype != "float8") * 2) if self._rope_quantized else ROPE_DIM * 2
        total = b * cold * (self._code_bytes + self._n_scales * 2 + rope)
        total += b * self._hot_len * (LATENT_DIM + ROPE_DIM) * self._dtype.itemsize
        return int(total)

    # ------------------------------------------------------------------ pools
    def _ensure_pools(self, batch: int, device: torch.device, dtype: torch.dtype) -> None:
        if self._hot is None:
            self._batch = batch
            self._dtype = dtype
            fields = {"latent": ((LATENT_DIM,), torch.bfloat16), "rope": ((ROPE_DIM,), torch.bfloat16)}
            if dtype != torch.bfloat16:
                # the caller's own values (the reference keeps the appended dtype), beside the
                # bf16 operands the decode kernel reads
                fields.update(src_latent=((LATENT_DIM,), dtype), src_rope=((ROPE_DIM,), dtype))
            self._hot = _Pool(fields, self.page_tokens, device)
            code_dtype = _CODE_DTYPES.get(self.cache_dtype, torch.uint8)
            cold = {"codes": ((self._code_bytes,), code_dtype), "scales": ((self._n_scales,), torch.float16)}
            if self._rope_quantized:
                # RoPE codes of the cold scheme (float8: raw e4m3 bytes) and, but for float8, their scales
                cold.update(rope=((self._rope_code_bytes,), _CODE_DTYPES.get(self.cache_dtype, torch.uint8)))
                if self.cache_dtype != "float8":
                    cold.update(rope_scales=((), torch.float16))
            else:
                cold.update(rope=((ROPE_DIM,), torch.bfloat16))
            self._cold = _Pool(cold, self.page_tokens, device)
            self._hot_pages = [[] for _ in range(batch)]
            self._cold_pages = [[] for _ in range(batch)]
        elif batch != self._batch:
            raise ValueError(f"batch size changed from {self._batch} to {batch}")
        elif dtype != self._dtype:
            raise ValueError(f"latent dtype changed from {self._dtype} to {dtype} (the hot window keeps one dtype)")

    @property
    def _code_bytes(self) -> int:
        """Code bytes of a cold token: one a dim for int8, two dims a byte for the INT4 schemes."""
        return LATENT_DIM if self.cache_dtype in _CODE_DTYPES else LATENT_DIM // 2

    @property
    def _rope_code_bytes(self) -> int:
        return ROPE_DIM if self.cache_dtype in _CODE_DTYPES else ROPE_DIM // 2

    @property
    def _n_scales(self) -> int:
        """fp16 scales of a cold token: one per group of 64, none for float8 (kv.py:85-89)."""
        return 0 if self.cache_dtype == "float8" else LATENT_DIM // GROUP_SIZE

    @property
    def _rope_quantized(self) -> bool:
        """Cold RoPE keys stored as codes (cache.py:163: only the integer schemes with quantize_rope)."""
        return self.quantize_rope and self.cache_dtype in _SCHEME_IDS

    @property
    def _src(self) -> str:
        """Prefix of the hot-pool fields holding the caller's values ("" when they are the bf16 operands)."""
        return "" if self._dtype == torch.bfloat16 else "src_"

    def pools(self) -> LatentPools:
        """The five device pools in the layout the decode C ABI reads."""
        if self._hot is None:
            raise RuntimeError("empty cache")
        return LatentPools(cold_codes=self._cold["codes"], cold_scales=self._cold["scales"],
                           cold_rope=self._cold["rope"], hot_latent=self._hot["latent"], hot_rope=self._hot["rope"],
                           cold_scheme=self.cache_dtype if self.cache_dtype in _SCHEME_IDS else "hadamard_int4",
                           cold_rope_scales=(self._cold["rope_scales"] if self._rope_quantized and
                                             self.cache_dtype != "float8" else None))

    def decode_layouts(self, q_len: int) -> list[SequenceLayout]:
        """One SequenceLayout per batch row; row b's new tokens are rows b*q_len.. of the step's arrays."""
        P = self.page_tokens
        out = []
        for b in range(self._batch):
            cold = [(pg, 0, P) for pg in self._cold_pages[b]]
            hot = []
            left = self._hot_len
            for pg in self._hot_pages[b]:
                n = min(P, left)
                if n > 0:
                    hot.append((pg, 0, n))
                left -= n
            out.append(SequenceLayout(cold=cold, hot=hot, q_start=b * q_len, q_len=q_len))
        return out

    # ------------------------------------------------------------------ writes
    def append(self, latent: torch.Tensor, rope_key: torch.Tensor, window_size: int | None = None,
               sink_tokens: int = 0) -> None:
        """Append [B, T, 512] latents and [B, T, 64] RoPE keys (cache.py:185-221)."""
        latent = latent.detach()
        rope_key = rope_key.detach()
        if latent.dim() != 3 or latent.shape[-1] != LATENT_DIM or rope_key.shape != (*latent.shape[:2], ROPE_DIM):
            raise ValueError("latent must be [B, T, 512] and rope_key [B, T, 64]")
        if not latent.is_cuda:
            raise RuntimeError("asterq caches live on the GPU; there is no CPU path")
        bsz, t = latent.shape[:2]
        self._ensure_pools(bsz, latent.device, latent.dtype)
        if t:
            self._write_hot(latent, rope_key)
        self._flush_cold_chunks()
        trim_slack = self.chunk_tokens if window_size is not None and window_size > 2 * self.chunk_tokens else 0
        if window_size is not None and self.length > window_size + trim_slack:
            if self.trim_mode == "pages":
                self._trim_pages(window_size, sink_tokens)
            else:
                self._trim(window_size, sink_tokens, latent.dtype, latent.device)

    def _trim_pages(self, window_size: int, sink_tokens: int) -> None:
        """Keep the cold pages holding the first min(sink, window) tokens and the newest cold pages
        that, with the hot window, hold the last window - sink tokens; release the pages between
        (whole pages, codes untouched)."""
        drop = trim_page_range(self.cold_chunks, [self.chunk_tokens] * self.cold_chunks, self._hot_len,
                               self.chunk_tokens, window_size, sink_tokens)
        if drop is None:
            return
        a, b = drop
        self._mark_dirty()
        for row in range(self._batch):
            pages = self._cold_pages[row]
            self._cold.release(pages[a:b])
            self._cold_pages[row] = pages[:a] + pages[b:]

    # ------------------------------------------------------------------ device tables
    def _mark_dirty(self) -> None:
        if self._dev is not None:
            self._dev.dirty = True

    def device_tables(self, q_len: int):
        """The page tables on the GPU (``asterq.batch.BatchTables``), every row with ``q_len`` new
        tokens at rows ``b * q_len``; rebuilt from the page lists and uploaded (one copy) only when
        pages changed or ``q_len`` did since the last call."""
        import types

        import numpy as np

        from .batch import BatchTables

        P, B = self.page_tokens, self._batch
        n_cold = self.cold_chunks
        n_hot = max((len(pg) for pg in self._hot_pages), default=0)
        st = self._dev
        if st is None or st.tables.max_cold_pages < max(1, n_cold) or st.tables.max_hot_pages < max(1, n_hot):
            tables = BatchTables(B, max(16, 2 * n_cold), max(4, 2 * n_hot), self._hot.device)
            st = self._dev = types.SimpleNamespace(tables=tables, dirty=True, q_len=None, planner=None,
                                                   status=torch.zeros(1, dtype=torch.int32, device=self._hot.device))
        if st.dirty or st.q_len != q_len:
            h = st.tables.host
            h["cold_pages"][:] = 0
            h["cold_tokens"][:] = 0
            h["hot_pages"][:] = -1
            h["n_cold"][:] = n_cold
            for b in range(B):
                h["cold_pages"][b, :n_cold] = self._cold_pages[b]
                h["cold_tokens"][b, :n_cold] = P
                h["hot_pages"][b, : len(self._hot_pages[b])] = self._hot_pages[b]
            h["hot_tokens"][:] = self._hot_len
            h["q_len"][:] = q_len
            h["q_start"][:] = np.arange(B, dtype=np.int32) * q_len
            st.tables.upload()
            st.dirty, st.q_len = False, q_len
        return st.tables

    def device_planner(self, n_heads: int, q_len: int):
        """A GPU planner (``asterq.batch.DevicePlanner``) bound to ``device_tables(q_len)``, kept
        across calls (re-created only when the tables are re-created or a step has more rows)."""
        from .batch import DevicePlanner

        tables = self.device_tables(q_len)
        st = self._dev
        pl = st.planner
        if pl is None or pl.tables is not tables or pl.n_heads != n_heads or pl.max_q_len < q_len:
            max_q = max(q_len, pl.max_q_len if (pl is not None and pl.tables is tables) else 1)
            st.planner = pl = DevicePlanner(tables, n_heads, self.page_tokens, max_q_len=max_q,
                                            cold_tile=COLD_TILE_TOKENS.get(self.cache_dtype, 128))
        return pl

    def raise_if_failed(self) -> None:
        """Synchronize; raise if an in-place append found a hot page missing."""
        if self._dev is not None and int(self._dev.status.item()) != 0:
            self._dev.status.zero_()
            raise RuntimeError("asterq cache: an append found a hot page missing")

    def _write_hot(self, latent: torch.Tensor, rope_key: torch.Tensor) -> None:
        P, (bsz, t) = self.page_tokens, latent.shape[:2]
        end = self._hot_len + t
        need = (end + P - 1) // P
        for b in range(bsz):
            missing = need - len(self._hot_pages[b])
            if missing > 0:
                self._hot_pages[b].extend(self._hot.alloc(missing))
                self._mark_dirty()
        if not self._src and latent.dtype == torch.bfloat16 and rope_key.dtype == torch.bfloat16 and t <= 2048:
            # in place on the device page tables (asterq_batch_append): no host index tensors
            import ctypes

            tables = self.device_tables(t)
            lat = latent.reshape(bsz * t, LATENT_DIM).contiguous()
            rope = rope_key.reshape(bsz * t, ROPE_DIM).contiguous()
            d = tables.desc(1, P, 1)
            _lib.check(_lib.load().asterq_batch_append(
                ctypes.byref(d), tables.dev["hot_tokens"].data_ptr(), lat.data_ptr(), rope.data_ptr(), bsz * t,
                self._hot["latent"].data_ptr(), self._hot["rope"].data_ptr(), int(self._hot["latent"].shape[0]),
                self._dev.status.data_ptr(), _lib.stream_handle(latent.device)))
            tables.host["hot_tokens"][:] = end  # the kernel advanced the device copy
            self._hot_len = end
            return
        self._mark_dirty()
        pos = torch.arange(self._hot_len, end, device=latent.device)
        pages = torch.tensor(self._hot_pages, dtype=torch.int64, device=latent.device)  # [B, n_pages]
        slot = pages[:, pos // P] * P + (pos % P)  # [B, T]
        flat = slot.reshape(-1)
        lat, rope = latent.reshape(-1, LATENT_DIM), rope_key.reshape(-1, ROPE_DIM).to(latent.dtype)
        self._hot["latent"].view(-1, LATENT_DIM).index_copy_(0, flat, lat.to(torch.bfloat16))
        self._hot["rope"].view(-1, ROPE_DIM).index_copy_(0, flat, rope.to(torch.bfloat16))
        if self._src:
            self._hot["src_latent"].view(-1, LATENT_DIM).index_copy_(0, flat, lat.to(self._dtype))
            self._hot["src_rope"].view(-1, ROPE_DIM).index_copy_(0, flat, rope.to(self._dtype))
        self._hot_len = end

    def _flush_cold_chunks(self) -> None:
        """cache.py:167-177: while hot > recent + chunk, encode the oldest chunk of every row."""
        if self.cache_dtype == "bfloat16" or self._hot is None:
            return
        threshold = self.recent_tokens + self.chunk_tokens
        while self._hot_len > threshold:
            self._flush_one()

    def _flush_one(self) -> None:
        P, bsz = self.page_tokens, self._batch
        dev = self._hot.device
        self._mark_dirty()
        src = torch.tensor([self._hot_pages[b][0] for b in range(bsz)], dtype=torch.int64).pin_memory().to(
            dev, non_blocking=True)
        dst_pages = self._cold.alloc(bsz)
        dst = torch.tensor(dst_pages, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
        # quantized from the caller's values (cache.py:172 encodes the hot tensor as stored)
        x = self._hot[self._src + "latent"].index_select(0, src).reshape(bsz * P, LATENT_DIM)
        codes = torch.empty(bsz * P, self._code_bytes, dtype=self._cold["codes"].dtype, device=dev)
        scales = torch.empty(bsz * P, max(self._n_scales, 1), dtype=torch.float16, device=dev)
        lib = _lib.load()
        _lib.check(lib.asterq_quantize(x.data_ptr(), _lib.dtype_code(x.dtype), bsz * P, LATENT_DIM, LATENT_DIM,
                                       _SCHEME_IDS[self.cache_dtype], GROUP_SIZE, codes.data_ptr(), scales.data_ptr(),
                                       _lib.stream_handle(dev)))
        self._cold["codes"].index_copy_(0, dst, codes.view(bsz, P, -1))
        if self._n_scales:
            self._cold["scales"].index_copy_(0, dst, scales.view(bsz, P, -1))
        if self._rope_quantized:
            # quantize_rope (cache.py:163): the RoPE keys as stored, cold scheme, one group of 64
            r = self._hot[self._src + "rope"].index_select(0, src).reshape(bsz * P, ROPE_DIM)
            rcodes = torch.empty(bsz * P, self._rope_code_bytes, dtype=self._cold["rope"].dtype, device=dev)
            rscales = torch.empty(bsz * P, 1, dtype=torch.float16, device=dev)
            _lib.check(lib.asterq_quantize(r.data_ptr(), _lib.dtype_code(r.dtype), bsz * P, ROPE_DIM, ROPE_DIM,
                                           _SCHEME_IDS[self.cache_dtype], GROUP_SIZE, rcodes.data_ptr(),
                                           rscales.data_ptr(), _lib.stream_handle(dev)))
            self._cold["rope"].index_copy_(0, dst, rcodes.view(bsz, P, -1))
            if self.cache_dtype != "float8":
                self._cold["rope_scales"].index_copy_(0, dst, rscales.view(bsz, P))
        else:
            # cold RoPE keys are bf16 whatever the caller's dtype (cache.py:162-164)
            self._cold["rope"].index_copy_(0, dst, self._hot["rope"].index_select(0, src))
        freed = []
        for b in range(bsz):
            self._cold_pages[b].append(dst_pages[b])
            freed.append(self._hot_pages[b].pop(0))
        self._hot.release(freed)
        self._hot_len -= P

    def _trim(self, window_size: int, sink_tokens: int, dtype: torch.dtype, device: torch.device) -> None:
        """cache.py:203-221: keep sink + recent tokens and re-encode them (double quantization, as the reference)."""
        all_latent = self.materialize_latent(dtype=dtype, device=device)
        all_rope = self.materialize_rope(dtype=dtype, device=device)
        sink = min(sink_tokens, window_size)
        recent = window_size - sink
        if sink and recent:
            all_latent = torch.cat((all_latent[:, :sink], all_latent[:, -recent:]), dim=1)
            all_rope = torch.cat((all_rope[:, :sink], all_rope[:, -recent:]), dim=1)
        elif recent:
            all_latent, all_rope = all_latent[:, -recent:], all_rope[:, -recent:]
        else:
            all_latent, all_rope = all_latent[:, :sink], all_rope[:, :sink]
        self._release_all()
        self._write_hot(all_latent.contiguous(), all_rope.contiguous())
        self._flush_cold_chunks()

    def _release_all(self) -> None:
        self._mark_dirty()
        for b in range(self._batch):
            self._hot.release(self._hot_pages[b])
            self._cold.release(self._cold_pages[b])
            self._hot_pages[b] = []
            self._cold_pages[b] = []
        self._hot_len = 0

    # ------------------------------------------------------------------ reads (API parity, not the decode path)
    @property
    def latent(self) -> torch.Tensor | None:
        """Hot window [B, S_hot, 512] in the caller's dtype (a gathered copy of the hot pages)."""
        return self._gather_hot(self._src + "latent")

    @property
    def rope_key(self) -> torch.Tensor | None:
        return self._gather_hot(self._src + "rope")

    def _gather_hot(self, name: str) -> torch.Tensor | None:
        if self._hot is None:
            return None
        pool = self._hot[name]
        rows = [torch.cat([pool[pg] for pg in self._hot_pages[b]], dim=0)[: self._hot_len] if self._hot_pages[b]
                else pool.new_empty(0, pool.shape[-1]) for b in range(self._batch)]
        return torch.stack(rows).to(self._dtype)

    @property
    def cold_latent(self) -> list[QuantizedTensor]:
        """One reference-format QuantizedTensor per cold chunk (kv.py:58-73): data [B, chunk, 256] (INT4) or
        [B, chunk, 512] (int8, float8), scale [B, chunk, 8, 1] (None for float8)."""
        out = []
        for c in range(self.cold_chunks):
            pages = [self._cold_pages[b][c] for b in range(self._batch)]
            data = torch.stack([self._cold["codes"][pg] for pg in pages])
            if self.cache_dtype == "float8":
                data = data.view(torch.float8_e4m3fn)
            scale = torch.stack([self._cold["scales"][pg] for pg in pages]).unsqueeze(-1) if self._n_scales else None
            out.append(QuantizedTensor(data=data, scale=scale, original_shape=(self._batch, self.chunk_tokens, LATENT_DIM),
                                       padded_dim=LATENT_DIM, group_size=GROUP_SIZE, scheme=self.cache_dtype,
                                       source_dtype=self._dtype))
        return out

    @property
    def cold_rope(self) -> list[torch.Tensor] | list[QuantizedTensor]:
        """Cold RoPE pieces: bf16 [B, chunk, 64], or with quantize_rope one QuantizedTensor per
        chunk (data [B, chunk, 32] INT4 / [B, chunk, 64] int8 or float8, scale [B, chunk, 1, 1] or
        None for float8), as the reference stores them."""
        if not self._rope_quantized:
            return [torch.stack([self._cold["rope"][self._cold_pages[b][c]] for b in range(self._batch)])
                    for c in range(self.cold_chunks)]
        out = []
        for c in range(self.cold_chunks):
            pages = [self._cold_pages[b][c] for b in range(self._batch)]
            data = torch.stack([self._cold["rope"][pg] for pg in pages])
            if self.cache_dtype == "float8":
                data, scale = data.view(torch.float8_e4m3fn), None
            else:
                scale = torch.stack([self._cold["rope_scales"][pg] for pg in pages]).reshape(self._batch, -1, 1, 1)
            out.append(QuantizedTensor(data=data, scale=scale, original_shape=(self._batch, self.chunk_tokens, ROPE_DIM),
                                       padded_dim=ROPE_DIM, group_size=GROUP_SIZE, scheme=self.cache_dtype,
                                       source_dtype=self._dtype))
        return out

    @staticmethod
    def _rope_piece(piece, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        if isinstance(piece, QuantizedTensor):
            return dequantize_tensor(piece, dtype=dtype).to(device)
        return piece.to(device=device, dtype=dtype)

    def iter_chunks(self, *, dtype: torch.dtype, device: torch.device):
        """cache.py:139-159: dequantized (latent, rope) per cold chunk, then the hot window."""
        for q, rope in zip(self.cold_latent, self.cold_rope, strict=True):
            yield dequantize_tensor(q, dtype=dtype).to(device), self._rope_piece(rope, dtype, device)
        if self._hot_len:
            yield self.latent.to(device=device, dtype=dtype), self.rope_key.to(device=device, dtype=dtype)

    def materialize_latent(self, *, dtype: torch.dtype | None = None, device: torch.device | None = None):
        """cache.py:89-116."""
        if self._hot is None or self.length == 0:
            return None
        dtype = self._dtype if dtype is None else dtype
        device = self._hot.device if device is None else device
        parts = [dequantize_tensor(q, dtype=dtype).to(device) for q in self.cold_latent]
        if self._hot_len:
            parts.append(self.latent.to(device=device, dtype=dtype))
        return torch.cat(parts, dim=1)

    def materialize_rope(self, *, dtype: torch.dtype | None = None, device: torch.device | None = None):
        """cache.py:118-137."""
        if self._hot is None or self.length == 0:
            return None
        dtype = self._dtype if dtype is None else dtype
        device = self._hot.device if device is None else device
        parts = [self._rope_piece(r, dtype, device) for r in self.cold_rope]
        if self._hot_len:
            parts.append(self.rope_key.to(device=device, dtype=dtype))
        return torch.cat(parts, dim=1)


@dataclass
class AsterCache:
    """Latent-layer part of the reference's mixed cache (cache.py:224-292)."""

    seen_tokens: int = 0
    latent: dict[int, LatentLayerCache] = field(default_factory=dict)
    kda_states: dict[int, torch.Tensor] = field(default_factory=dict)
    cache_dtype: str = "bfloat16"
    cache_group_size: int = 64
    cache_recent_tokens: int = 512
    cache_chunk_tokens: int = 1024
    cache_quantize_rope: bool = False

    @classmethod
    def create(cls, config: Any | None = None) -> "AsterCache":
        kwargs: dict[str, Any] = {}
        if config is not None:
            kwargs = {"cache_dtype": config.cache_dtype, "cache_group_size": config.cache_group_size,
                      "cache_recent_tokens": config.cache_recent_tokens, "cache_chunk_tokens": config.cache_chunk_tokens,
                      "cache_quantize_rope": config.cache_quantize_rope}
        return cls(**kwargs)

    def latent_layer(self, layer_idx: int) -> LatentLayerCache:
        if layer_idx not in self.latent:
            self.latent[layer_idx] = LatentLayerCache(cache_dtype=self.cache_dtype, group_size=self.cache_group_size,
                                                      recent_tokens=self.cache_recent_tokens,
                                                      chunk_tokens=self.cache_chunk_tokens,
                                                      quantize_rope=self.cache_quantize_rope)
        return self.latent[layer_idx]

    @property
    def num_bytes(self) -> int:
        total = sum(layer.num_bytes for layer in self.latent.values())
        total += sum(s.numel() * s.element_size() for s in self.kda_states.values())
        return int(total)

    def reset(self) -> None:
        self.seen_tokens = 0
        self.latent.clear()
        self.kda_states.clear()
