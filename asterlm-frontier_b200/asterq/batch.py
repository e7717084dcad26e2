"""Continuous-batching decode with the schedule built on the GPU.

The reference serves one uniform batch: every step ``LatentLayerCache.append`` re-concatenates
the hot window (cache.py:185-221) and ``LatentAttention._absorbed_decode`` walks the chunks on
the host (latent_attention.py:177-231, cache.py:139-159).  Here a batch of sequences of
different lengths lives in page pools whose page tables and lengths are on the GPU
(``asterq_batch_desc``), and a decode step is three launches on the caller's stream:

1. ``asterq_plan_batch``: the schedule (tiles, work items, worker shares, combine jobs) from
   the device tables, into buffers of fixed capacity;
2. ``asterq_latent_decode`` on those tables: attention of the step's queries over each
   sequence's cache plus its own new tokens;
3. ``asterq_batch_append``: the step's new tokens into the hot windows, in place.

The host keeps a mirror of the page tables and lengths only to hand out pages ahead of need
and to trigger flushes: after a step, a sequence whose hot window exceeds
``recent_tokens + page_tokens`` has its oldest (full) hot page encoded into a cold page by the
write-path kernel (cache.py:167-177, one chunk per page).  Steps without a flush or a new page
cost the host three C calls, and the three launches can be recorded in a CUDA graph
(``PagedLatentBatch.capture``).

``BatchTables`` and ``DevicePlanner`` are the two reusable parts: the device tables with their
host mirror, and the planner's buffers with the decode call bound to them.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from .decode import COLD_SCHEMES, COLD_TILE_TOKENS, GROUP_SIZE, LATENT_DIM, ROPE_DIM, LatentPools, set_cold_pools
from .plan import QPREP_BYTES

COLD_TILE = 128
HOT_TILE = 32
ROWS_PER_BLOCK = 16
RECORD_BYTES = ROWS_PER_BLOCK * (LATENT_DIM + 2) * 4
MAX_Q_LEN = 2048


def _pinned(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


class BatchTables:
    """The device arrays of an ``asterq_batch_desc`` and their host mirror (numpy, same shapes).

    Row s describes sequence slot s: ``n_cold`` cold pages ``cold_pages[s, :n_cold]`` holding
    ``cold_tokens[s, j]`` tokens each, ``hot_tokens[s]`` hot tokens in ``hot_pages[s, :]``
    (-1: no page), and ``q_len[s]`` new tokens per step at rows ``q_start[s]`` ..
    (q_len 0: an empty slot).  ``upload`` copies the mirror to the device on the current
    stream; the append kernel advances ``hot_tokens`` on the device, and the owner advances
    the mirror to match.
    """

    def __init__(self, n_seqs: int, max_cold_pages: int, max_hot_pages: int, device) -> None:
        self.device = torch.device(device)
        self.n_seqs = int(n_seqs)
        self.host = {
            "n_cold": np.zeros(n_seqs, np.int32),
            "cold_pages": np.zeros((n_seqs, max(1, max_cold_pages)), np.int32),
            "cold_tokens": np.zeros((n_seqs, max(1, max_cold_pages)), np.int32),
            "hot_tokens": np.zeros(n_seqs, np.int32),
            "hot_pages": np.full((n_seqs, max(1, max_hot_pages)), -1, np.int32),
            "q_len": np.zeros(n_seqs, np.int32),
            "q_start": np.zeros(n_seqs, np.int32),
        }
        self.generation = 0  # bumped whenever a device array is reallocated (bound pointers change)
        self._build_device()
        self.upload()

    def _build_device(self) -> None:
        """All arrays as views of one device buffer, so an upload is one copy, staged through two
        pinned buffers used in turn (a staging buffer is refilled only after its last copy has run)."""
        offs, total = {}, 0
        for name, a in self.host.items():
            offs[name] = total
            total += (a.size + 3) // 4 * 4  # each array 16-byte aligned
        self._offs, self._total = offs, total
        self._flat = torch.zeros(total, dtype=torch.int32, device=self.device)
        self.dev = {k: self._flat[o : o + self.host[k].size].view(self.host[k].shape) for k, o in offs.items()}
        self._stage = [torch.zeros(total, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._stage_done: list = [None, None]
        self._stage_next = 0

    @property
    def max_cold_pages(self) -> int:
        return int(self.host["cold_pages"].shape[1])

    @property
    def max_hot_pages(self) -> int:
        return int(self.host["hot_pages"].shape[1])

    def grow(self, max_cold_pages: int | None = None, max_hot_pages: int | None = None) -> None:
        """Widen the page tables (reallocates the device arrays)."""
        h = self.host
        grown = False
        for name, want, fill in (("cold_pages", max_cold_pages, 0), ("cold_tokens", max_cold_pages, 0),
                                 ("hot_pages", max_hot_pages, -1)):
            if want is not None and want > h[name].shape[1]:
                wide = np.full((self.n_seqs, want), fill, np.int32)
                wide[:, : h[name].shape[1]] = h[name]
                h[name] = wide
                grown = True
        if grown:
            self._build_device()
            self.upload()
            self.generation += 1

    def shadow(self) -> "BatchTables":
        """A second set of device arrays over the same host mirror (``upload`` fills it): what a
        planner reads while the primary arrays are being changed by the step in flight."""
        t = BatchTables.__new__(BatchTables)
        t.device, t.n_seqs, t.host = self.device, self.n_seqs, self.host
        t.generation = 0
        t._build_device()
        return t

    def upload(self, names=None) -> None:
        """Copy the whole mirror to the device on the current stream (one copy; `names` is accepted
        for compatibility and ignored)."""
        j = self._stage_next
        self._stage_next ^= 1
        if self._stage_done[j] is not None:
            self._stage_done[j].synchronize()
        st = self._stage[j].numpy()
        for name, a in self.host.items():
            o = self._offs[name]
            st[o : o + a.size] = a.reshape(-1)
        self._flat.copy_(self._stage[j], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._stage_done[j] = ev

    def desc(self, n_heads: int, page_tokens: int, n_workers: int) -> _lib.BatchDesc:
        d = _lib.BatchDesc()
        d.n_seqs, d.n_heads, d.page_tokens, d.n_workers = self.n_seqs, n_heads, page_tokens, n_workers
        d.max_cold_pages, d.max_hot_pages = self.max_cold_pages, self.max_hot_pages
        dev = self.dev
        d.n_cold_pages, d.cold_pages, d.cold_page_tokens = (dev["n_cold"].data_ptr(), dev["cold_pages"].data_ptr(),
                                                           dev["cold_tokens"].data_ptr())
        d.hot_tokens, d.hot_pages = dev["hot_tokens"].data_ptr(), dev["hot_pages"].data_ptr()
        d.q_len, d.q_start = dev["q_len"].data_ptr(), dev["q_start"].data_ptr()
        return d


def tables_from_layouts(layouts, page_tokens: int, device, *, n_seqs: int | None = None) -> BatchTables:
    """``BatchTables`` describing ``SequenceLayout`` s of a batch in place (their page ids, their
    q_start / q_len; chunks must start at page offset 0 and hot pages be full except the last)."""
    P = page_tokens
    n_seqs = len(layouts) if n_seqs is None else n_seqs
    max_cold = max([len(l.cold) for l in layouts] + [1])
    max_hot = max([len(l.hot) for l in layouts] + [1])
    t = BatchTables(n_seqs, max_cold, max_hot, device)
    h = t.host
    for s, lay in enumerate(layouts):
        if any(off != 0 for _, off, _ in lay.cold + lay.hot) or any(n != P for _, _, n in lay.hot[:-1]):
            raise ValueError("chunks must start at page offset 0 and hot pages be full except the last")
        h["n_cold"][s] = len(lay.cold)
        h["cold_pages"][s, : len(lay.cold)] = [pg for pg, _, _ in lay.cold]
        h["cold_tokens"][s, : len(lay.cold)] = [n for _, _, n in lay.cold]
        h["hot_pages"][s, : len(lay.hot)] = [pg for pg, _, _ in lay.hot]
        h["hot_tokens"][s] = sum(n for _, _, n in lay.hot)
        h["q_len"][s] = lay.q_len if lay.attend_new else 0
        h["q_start"][s] = lay.q_start
    t.upload()
    return t


class DevicePlanner:
    """Plan buffers of fixed capacity for one ``BatchTables`` and the decode call bound to them.

    The capacities are the most the tables can describe (every sequence with all its cold and
    hot pages full and ``max_q_len`` new tokens), so no step can exceed them; the planner's
    status (``counts[5]``) is checked by ``raise_if_failed``.
    """

    def __init__(self, tables: BatchTables, n_heads: int, page_tokens: int, *, max_q_len: int = 1,
                 n_workers: int | None = None, cold_tile: int = COLD_TILE) -> None:
        if not 0 < max_q_len <= MAX_Q_LEN:
            raise ValueError(f"max_q_len must be in 1..{MAX_Q_LEN}")
        if page_tokens <= 0 or page_tokens % 16:
            raise ValueError("page_tokens must be a positive multiple of 16")
        self.tables = tables
        if cold_tile not in (64, COLD_TILE):
            raise ValueError("cold_tile must be 64 (int8 codes) or 128")
        self.n_heads, self.page_tokens, self.max_q_len, self.cold_tile = n_heads, page_tokens, max_q_len, cold_tile
        dev = tables.device
        if n_workers is None:
            n_workers = torch.cuda.get_device_properties(dev).multi_processor_count
        self.n_workers = int(n_workers)
        self._bound_generation = -1
        self._alloc()

    def _alloc(self) -> None:
        t, P, S = self.tables, self.page_tokens, self.tables.n_seqs
        dev = t.device
        per_seq = (t.max_cold_pages * math.ceil(P / self.cold_tile) + t.max_hot_pages * math.ceil(P / HOT_TILE)
                   + math.ceil(self.max_q_len / HOT_TILE))
        self.cap_tiles = max(1, S * per_seq)
        self.cap_units = max(1, S * math.ceil(self.max_q_len * self.n_heads / ROWS_PER_BLOCK))
        self.cap_items = self.cap_units + self.n_workers
        i32 = torch.int32
        self.tiles = torch.zeros(self.cap_tiles, 4, dtype=i32, device=dev)
        self.units = torch.zeros(self.cap_units, 2, dtype=i32, device=dev)
        self.items = torch.zeros(self.cap_items, 8, dtype=i32, device=dev)
        self.combine = torch.zeros(self.cap_units, 4, dtype=i32, device=dev)
        self.unit_jobs = torch.full((self.cap_units,), -1, dtype=i32, device=dev)
        self.workers = torch.zeros(self.n_workers + 1, dtype=i32, device=dev)
        self.counts = torch.zeros(8, dtype=i32, device=dev)
        self.desc = t.desc(self.n_heads, self.page_tokens, self.n_workers)
        self.desc.cold_tile_tokens = self.cold_tile
        nbytes = _lib.load().asterq_plan_scratch_bytes(ctypes.byref(self.desc), self.cap_tiles, self.cap_units,
                                                       self.cap_items)
        if nbytes <= 0:
            raise ValueError("asterq_plan_scratch_bytes rejected the batch shape")
        self.scratch = torch.empty((nbytes + 15) // 16 * 4, dtype=torch.int32, device=dev)
        ws = self.cap_items * RECORD_BYTES + self.cap_units * _QPREP_BYTES + (self.cap_units * 4 + 15) // 16 * 16
        self.workspace = torch.empty(max(4, ws // 4), dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=i32, device=dev)
        b = _lib.PlanBuffers()
        b.cap_tiles, b.cap_units, b.cap_items = self.cap_tiles, self.cap_units, self.cap_items
        b.tiles, b.units, b.items = self.tiles.data_ptr(), self.units.data_ptr(), self.items.data_ptr()
        b.combine, b.unit_jobs, b.workers = self.combine.data_ptr(), self.unit_jobs.data_ptr(), self.workers.data_ptr()
        b.counts, b.scratch = self.counts.data_ptr(), self.scratch.data_ptr()
        self.buffers = b
        self._params = None
        self._bound_generation = self.tables.generation

    def _refresh(self) -> None:
        if self._bound_generation != self.tables.generation:
            self._alloc()

    def plan(self, stream: int | None = None) -> None:
        """Enqueue ``asterq_plan_batch`` on the current (or given) stream."""
        self._refresh()
        s = _lib.stream_handle(self.tables.device) if stream is None else stream
        _lib.check(_lib.load().asterq_plan_batch(ctypes.byref(self.desc), ctypes.byref(self.buffers), s))

    def params(self, pools: LatentPools, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float,
               logit_softcap: float | None = None, wait_limit_cycles: int = 0) -> _lib.DecodeParams:
        """``asterq_decode_params`` for the planned tables (built once, pointers refreshed per call)."""
        self._refresh()
        p = self._params
        if p is None:
            p = _lib.DecodeParams()
            p.n_heads, p.latent_dim, p.rope_dim, p.group_size = self.n_heads, LATENT_DIM, ROPE_DIM, GROUP_SIZE
            p.page_tokens = self.page_tokens
            p.n_tiles, p.n_items, p.n_units, p.n_slots = self.cap_tiles, self.cap_items, self.cap_units, self.cap_items
            p.n_combine = (self.n_workers + 15) // 16
            p.n_combine_total = self.cap_units
            p.tiles, p.items, p.combine = self.tiles.data_ptr(), self.items.data_ptr(), self.combine.data_ptr()
            p.units, p.unit_jobs = self.units.data_ptr(), self.unit_jobs.data_ptr()
            p.workers, p.n_workers = self.workers.data_ptr(), self.n_workers
            p.workspace, p.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel() * 4
            p.device_status = self.status.data_ptr()
            p.plan_counts = self.counts.data_ptr()
            self._params = p
        p.out_dtype = _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16
        p.softmax_scale = float(softmax_scale)
        p.logit_softcap = float(logit_softcap) if logit_softcap else 0.0
        p.wait_limit_cycles = int(wait_limit_cycles)
        set_cold_pools(p, pools)
        p.n_hot_pages = int(pools.hot_latent.shape[0])
        p.hot_latent = pools.hot_latent.data_ptr() if pools.hot_latent.numel() else None
        p.hot_rope = pools.hot_rope.data_ptr() if pools.hot_rope.numel() else None
        p.total_q = int(q_lat.shape[0])
        p.q_lat, p.q_rope = q_lat.data_ptr(), q_rope.data_ptr()
        p.new_latent, p.new_rope, p.out = new_latent.data_ptr(), new_rope.data_ptr(), out.data_ptr()
        return p

    def decode(self, pools: LatentPools, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float,
               logit_softcap: float | None = None, wait_limit_cycles: int = 0, stream: int | None = None) -> None:
        """Enqueue the decode on the planned tables (``plan`` must have been enqueued before it)."""
        p = self.params(pools, q_lat, q_rope, new_latent, new_rope, out, softmax_scale=softmax_scale,
                        logit_softcap=logit_softcap, wait_limit_cycles=wait_limit_cycles)
        s = _lib.stream_handle(self.tables.device) if stream is None else stream
        _lib.check(_lib.load().asterq_latent_decode(ctypes.byref(p), s))

    def host_counts(self) -> dict[str, int]:
        """The planner's counts (synchronizes)."""
        c = self.counts.cpu().tolist()
        return dict(n_tiles=c[0], n_units=c[1], n_items=c[2], n_slots=c[3], n_jobs=c[4], status=c[5], n_separate=c[6])

    def raise_if_failed(self) -> None:
        """Synchronize; raise if the planner ran out of capacity or a decode wait timed out."""
        if int(self.counts[5].item()) != 0:
            raise RuntimeError("asterq plan_batch: the batch exceeds the planner's capacities")
        if int(self.status.item()) != 0:
            self.status.zero_()
            raise RuntimeError("asterq decode: a pipeline wait timed out on the device (output not valid)")


_QPREP_BYTES = QPREP_BYTES  # prepared query operands of one 16-row block


class _PagePool:
    """Fixed set of pages of one pool with a free list (pages are handed out lowest first)."""

    def __init__(self, n_pages: int) -> None:
        self.n_pages = int(n_pages)
        self.free = list(range(self.n_pages - 1, -1, -1))

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise MemoryError(f"page pool exhausted: {n} pages wanted, {len(self.free)} free of {self.n_pages}")
        return [self.free.pop() for _ in range(n)]

    def release(self, pages) -> None:
        self.free.extend(int(p) for p in pages)
        self.free.sort(reverse=True)


class PagedLatentBatch:
    """A continuous-batching hot/cold latent cache of one global-attention layer.

    ``max_seqs`` sequence slots, each decoding ``q_len`` new tokens per step (1 for plain
    decode, 1 + MTP depth for verification).  Slot s's queries and new tokens are rows
    ``s * q_len`` .. of the step's arrays ([max_seqs * q_len, H, 512] etc.; rows of empty
    slots are ignored).  Pools have fixed capacities (``hot_pool_pages``, ``cold_pool_pages``
    pages of ``page_tokens`` tokens), so the step's pointers never change and a captured step
    stays valid.  ``cache_dtype`` "hadamard_int4", "int4", "int8" or "float8" (cold pages) as in the
    reference; ``quantize_rope`` stores the cold RoPE keys as codes of the same scheme
    (cache.py:160-164), else they stay bf16.
    """

    def __init__(self, n_heads: int, *, max_seqs: int, q_len: int = 1, page_tokens: int = 512,
                 recent_tokens: int = 512, cache_dtype: str = "hadamard_int4", max_cold_pages: int = 64,
                 hot_pool_pages: int | None = None, cold_pool_pages: int | None = None,
                 n_workers: int | None = None, plan_ahead: bool = False, window_size: int | None = None,
                 sink_tokens: int = 0, quantize_rope: bool = False, device="cuda") -> None:
        if cache_dtype not in COLD_SCHEMES:
            raise NotImplementedError(f"cache_dtype {cache_dtype!r}: the serving batch pools {tuple(COLD_SCHEMES)}")
        if not 0 < q_len <= page_tokens:
            raise ValueError("q_len must be in 1..page_tokens")
        self.device = torch.device(device)
        self.n_heads, self.q_len, self.page_tokens = n_heads, q_len, page_tokens
        self.recent_tokens, self.cache_dtype = recent_tokens, cache_dtype
        self.threshold = recent_tokens + page_tokens  # cache.py:170: flush while hot > recent + chunk
        # sliding window with sink tokens (cache.py:203-221), trimmed by dropping whole cold pages
        # (no re-quantization): once a sequence is longer than window (+ one page of slack when
        # the window exceeds two pages), the cold pages between its sink and recent tokens go
        if window_size is not None and window_size <= 0:
            raise ValueError("window_size must be positive")
        self.window_size, self.sink_tokens = window_size, int(sink_tokens)
        self.pages_trimmed = 0
        P = page_tokens
        max_hot_pages = math.ceil((self.threshold + q_len) / P) + 1
        self.tables = BatchTables(max_seqs, max_cold_pages, max_hot_pages, self.device)
        h = self.tables.host
        h["q_start"][:] = np.arange(max_seqs, dtype=np.int32) * q_len
        if hot_pool_pages is None:
            hot_pool_pages = max_seqs * max_hot_pages
        if cold_pool_pages is None:
            cold_pool_pages = max_seqs * max_cold_pages
        self.pools = LatentPools.empty(cold_pool_pages, hot_pool_pages, P, self.device, cold_scheme=cache_dtype,
                                       quantize_rope=quantize_rope)
        self.cold_tile = COLD_TILE_TOKENS[cache_dtype]
        self._hot_free, self._cold_free = _PagePool(hot_pool_pages), _PagePool(cold_pool_pages)
        # plan_ahead: the next step's schedule is built on a side stream while this step decodes,
        # on the one SM the decode leaves free (one worker fewer), into the other of two planners
        # whose tables are copies of the host mirror taken after this step's bookkeeping
        self.plan_ahead = bool(plan_ahead)
        if self.plan_ahead and n_workers is None:
            n_workers = torch.cuda.get_device_properties(self.device).multi_processor_count - 1
        self.planner = DevicePlanner(self.tables, n_heads, P, max_q_len=q_len, n_workers=n_workers,
                                     cold_tile=self.cold_tile)
        self._ahead: list[DevicePlanner] = []
        self._ahead_gen = -1
        self._ahead_ready: int | None = None  # planner index holding the next step's schedule
        self._ahead_cur = 0
        if self.plan_ahead:
            self._plan_stream = torch.cuda.Stream(self.device)
            self._planned = [torch.cuda.Event(), torch.cuda.Event()]
            self._decoded = [torch.cuda.Event(), torch.cuda.Event()]
        self.append_status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.flushes = 0  # pages encoded into the cold pool so far
        self.flush_launches = 0  # encode launches those flushes took (one per step that flushed)
        self._provisional = False  # a verify() step awaits accept()
        self.tables.upload()

    # ------------------------------------------------------------------ sizes
    @property
    def max_seqs(self) -> int:
        return self.tables.n_seqs

    def active(self) -> np.ndarray:
        return np.nonzero(self.tables.host["q_len"] > 0)[0]

    def length(self, slot: int) -> int:
        h = self.tables.host
        return int(h["cold_tokens"][slot, : h["n_cold"][slot]].sum() + h["hot_tokens"][slot])

    def hot_length(self, slot: int) -> int:
        return int(self.tables.host["hot_tokens"][slot])

    # ------------------------------------------------------------------ sequences
    def _free_slot(self) -> int:
        free = np.nonzero(self.tables.host["q_len"] == 0)[0]
        if not free.size:
            raise RuntimeError(f"all {self.max_seqs} sequence slots are in use")
        return int(free[0])

    def add_sequence(self, latent: torch.Tensor, rope: torch.Tensor) -> int:
        """Admit a sequence with its prompt's latents [n, 512] and RoPE keys [n, 64] (bf16 on the
        GPU); returns its slot.  The prompt is split as the reference's bulk append leaves it
        (cache.py:167-177): whole chunks encoded into cold pages while more than
        ``recent_tokens + page_tokens`` tokens would stay hot."""
        if latent.dim() != 2 or latent.shape[1] != LATENT_DIM or rope.shape != (latent.shape[0], ROPE_DIM):
            raise ValueError("latent must be [n, 512] and rope [n, 64]")
        if not latent.is_cuda:
            raise RuntimeError("asterq caches live on the GPU; there is no CPU path")
        P, n = self.page_tokens, int(latent.shape[0])
        k = 0
        while n - k * P > self.threshold:
            k += 1
        slot = self._free_slot()
        h = self.tables.host
        if k > self.tables.max_cold_pages:
            self.tables.grow(max_cold_pages=max(k, 2 * self.tables.max_cold_pages))
        latent = latent.to(torch.bfloat16).contiguous()
        rope = rope.to(torch.bfloat16).contiguous()
        if k:
            dst = self._cold_free.alloc(k)
            self._encode_into(latent[: k * P], rope[: k * P], dst)
            h["cold_pages"][slot, :k] = dst
            h["cold_tokens"][slot, :k] = P
        h["n_cold"][slot] = k
        hot = n - k * P
        pages = self._hot_free.alloc(math.ceil((hot + self.q_len) / P))
        h["hot_pages"][slot, :] = -1
        h["hot_pages"][slot, : len(pages)] = pages
        if hot:
            self._write_rows(latent[k * P :], rope[k * P :], pages)
        h["hot_tokens"][slot] = hot
        h["q_len"][slot] = self.q_len
        self.tables.upload()
        self._invalidate_plan()
        return slot

    def add_layout(self, pools: LatentPools, cold: list[tuple[int, int, int]], hot: list[tuple[int, int, int]]) -> int:
        """Admit a sequence whose cache already sits in other pools (``SequenceLayout`` chunks:
        cold (page, 0, n) oldest first, hot (page, 0, n) with every page but the last full); its
        pages are copied into this batch's pools as they are.  Returns the slot."""
        P = self.page_tokens
        if pools.page_tokens != P:
            raise ValueError("page sizes differ")
        if any(off != 0 for _, off, _ in cold + hot) or any(n != P for _, _, n in hot[:-1]):
            raise ValueError("chunks must start at page offset 0 and hot pages be full except the last")
        slot = self._free_slot()
        h = self.tables.host
        if len(cold) > self.tables.max_cold_pages:
            self.tables.grow(max_cold_pages=max(len(cold), 2 * self.tables.max_cold_pages))
        hot_len = sum(n for _, _, n in hot)
        if hot_len + self.q_len > (self.tables.max_hot_pages - 1) * P:
            raise ValueError(f"hot window of {hot_len} tokens exceeds the batch's hot pages")
        dev = self.device
        if cold:
            dst = self._cold_free.alloc(len(cold))
            src = torch.tensor([pg for pg, _, _ in cold], dtype=torch.int64, device=dev)
            di = torch.tensor(dst, dtype=torch.int64, device=dev)
            names = ["cold_codes", "cold_scales", "cold_rope"]
            if self.pools.cold_rope_scales is not None:
                names.append("cold_rope_scales")
            for name in names:  # (the source pools must use the batch's scheme and RoPE form)
                getattr(self.pools, name).index_copy_(0, di, getattr(pools, name).index_select(0, src))
            h["cold_pages"][slot, : len(cold)] = dst
            h["cold_tokens"][slot, : len(cold)] = [n for _, _, n in cold]
        h["n_cold"][slot] = len(cold)
        pages = self._hot_free.alloc(math.ceil((hot_len + self.q_len) / P))
        if hot:
            src = torch.tensor([pg for pg, _, _ in hot], dtype=torch.int64, device=dev)
            di = torch.tensor(pages[: len(hot)], dtype=torch.int64, device=dev)
            for name in ("hot_latent", "hot_rope"):
                getattr(self.pools, name).index_copy_(0, di, getattr(pools, name).index_select(0, src))
        h["hot_pages"][slot, :] = -1
        h["hot_pages"][slot, : len(pages)] = pages
        h["hot_tokens"][slot] = hot_len
        h["q_len"][slot] = self.q_len
        self.tables.upload()
        self._invalidate_plan()
        return slot

    def remove_sequence(self, slot: int) -> None:
        h = self.tables.host
        self._cold_free.release(h["cold_pages"][slot, : h["n_cold"][slot]])
        self._hot_free.release(p for p in h["hot_pages"][slot] if p >= 0)
        h["n_cold"][slot] = 0
        h["hot_tokens"][slot] = 0
        h["hot_pages"][slot, :] = -1
        h["q_len"][slot] = 0
        self.tables.upload()
        self._invalidate_plan()

    # ------------------------------------------------------------------ pools
    def _write_rows(self, latent: torch.Tensor, rope: torch.Tensor, pages: list[int]) -> None:
        P, n = self.page_tokens, latent.shape[0]
        pos = torch.arange(n, device=self.device)
        pg = torch.tensor(pages, dtype=torch.int64, device=self.device)
        rows = pg[pos // P] * P + pos % P
        self.pools.hot_latent.view(-1, LATENT_DIM).index_copy_(0, rows, latent)
        self.pools.hot_rope.view(-1, ROPE_DIM).index_copy_(0, rows, rope)

    def _encode_into(self, latent: torch.Tensor, rope: torch.Tensor, pages: list[int]) -> None:
        """Encode len(pages) full chunks of bf16 tokens into the given cold pages."""
        P, n = self.page_tokens, latent.shape[0]
        lib = _lib.load()
        codes = torch.empty(n, self.pools.cold_codes.shape[-1], dtype=self.pools.cold_codes.dtype, device=self.device)
        n_scales = int(self.pools.cold_scales.shape[-1])  # 0 for float8
        scales = torch.empty(n, max(n_scales, 1), dtype=torch.float16, device=self.device)
        _lib.check(lib.asterq_quantize(latent.data_ptr(), _lib.DTYPE_BF16, n, LATENT_DIM, LATENT_DIM,
                                       COLD_SCHEMES[self.cache_dtype], GROUP_SIZE, codes.data_ptr(),
                                       scales.data_ptr(), _lib.stream_handle(self.device)))
        di = _pinned(np.asarray(pages, np.int64)).to(self.device, non_blocking=True)
        self.pools.cold_codes.index_copy_(0, di, codes.view(len(pages), P, -1))
        if n_scales:
            self.pools.cold_scales.index_copy_(0, di, scales.view(len(pages), P, -1))
        if self.pools.rope_quantized:
            # quantize_rope (cache.py:163): RoPE keys as codes of the cold scheme, one group of 64
            rcodes = torch.empty(n, self.pools.cold_rope.shape[-1], dtype=self.pools.cold_rope.dtype, device=self.device)
            rscales = torch.empty(n, 1, dtype=torch.float16, device=self.device)
            rope = rope.reshape(n, ROPE_DIM).to(torch.bfloat16).contiguous()
            _lib.check(lib.asterq_quantize(rope.data_ptr(), _lib.DTYPE_BF16, n, ROPE_DIM, ROPE_DIM,
                                           COLD_SCHEMES[self.cache_dtype], GROUP_SIZE, rcodes.data_ptr(),
                                           rscales.data_ptr(), _lib.stream_handle(self.device)))
            self.pools.cold_rope.index_copy_(0, di, rcodes.view(len(pages), P, -1))
            if self.pools.cold_rope_scales is not None:
                self.pools.cold_rope_scales.index_copy_(0, di, rscales.view(len(pages), P))
        else:
            self.pools.cold_rope.index_copy_(0, di, rope.reshape(len(pages), P, ROPE_DIM))

    # ------------------------------------------------------------------ steps
    def _ahead_planners(self) -> list[DevicePlanner]:
        if self._ahead_gen != self.tables.generation:  # (re)bind to the tables as they are now
            self._ahead = [DevicePlanner(self.tables.shadow(), self.n_heads, self.page_tokens, max_q_len=self.q_len,
                                         n_workers=self.planner.n_workers, cold_tile=self.cold_tile)
                           for _ in range(2)]
            self._ahead_gen = self.tables.generation
            self._ahead_ready = None
        return self._ahead

    def _plan_into(self, i: int) -> None:
        """Side stream: copy the host mirror into planner i's tables and plan into its buffers, once
        the decode that last read those buffers is done."""
        pl = self._ahead_planners()[i]
        side = self._plan_stream
        side.wait_event(self._decoded[i])
        with torch.cuda.stream(side):
            pl.tables.upload()
            pl.plan(side.cuda_stream)
            self._planned[i].record(side)

    def _invalidate_plan(self) -> None:
        self._ahead_ready = None

    def enqueue_step(self, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float | None = None,
                     logit_softcap: float | None = None, wait_limit_cycles: int = 0) -> None:
        """Enqueue plan + decode + append for every active slot (no host bookkeeping; see ``step``).
        With ``plan_ahead`` the schedule comes from the side stream (planned during the previous
        step, or now if the batch changed since)."""
        if softmax_scale is None:
            softmax_scale = 1.0 / math.sqrt(LATENT_DIM + ROPE_DIM)
        stream = _lib.stream_handle(self.device)
        if self.plan_ahead:
            i = self._ahead_ready
            if i is None:
                i = self._ahead_cur
                self._plan_into(i)
            torch.cuda.current_stream(self.device).wait_event(self._planned[i])
            planner = self._ahead_planners()[i]
            planner.decode(self.pools, q_lat, q_rope, new_latent, new_rope, out, softmax_scale=softmax_scale,
                           logit_softcap=logit_softcap, wait_limit_cycles=wait_limit_cycles, stream=stream)
            self._decoded[i].record(torch.cuda.current_stream(self.device))
            self._ahead_cur, self._ahead_ready = i, None
        else:
            self.planner.plan(stream)
            self.planner.decode(self.pools, q_lat, q_rope, new_latent, new_rope, out, softmax_scale=softmax_scale,
                                logit_softcap=logit_softcap, wait_limit_cycles=wait_limit_cycles, stream=stream)
        d = self.planner.desc
        _lib.check(_lib.load().asterq_batch_append(
            ctypes.byref(d), self.tables.dev["hot_tokens"].data_ptr(), new_latent.data_ptr(), new_rope.data_ptr(),
            int(new_latent.shape[0]), self.pools.hot_latent.data_ptr(), self.pools.hot_rope.data_ptr(), int(self.pools.hot_latent.shape[0]),
            self.append_status.data_ptr(), stream))

    def _check_step_inputs(self, q_lat, q_rope, new_latent, new_rope, out) -> None:
        rows = self.max_seqs * self.q_len
        H = self.n_heads
        for name, t, shape in (("q_lat", q_lat, (rows, H, LATENT_DIM)), ("q_rope", q_rope, (rows, H, ROPE_DIM)),
                               ("new_latent", new_latent, (rows, LATENT_DIM)), ("new_rope", new_rope, (rows, ROPE_DIM))):
            if t.dtype != torch.bfloat16 or tuple(t.shape) != shape or not t.is_contiguous() or not t.is_cuda:
                raise ValueError(f"{name} must be a contiguous bfloat16 CUDA tensor of shape {shape}")
        if out.dtype not in (torch.float32, torch.bfloat16) or tuple(out.shape) != (rows, H, LATENT_DIM):
            raise ValueError(f"out must be float32/bfloat16 [{rows}, {H}, {LATENT_DIM}]")

    def step(self, q_lat, q_rope, new_latent, new_rope, out=None, *, softmax_scale: float | None = None,
             logit_softcap: float | None = None) -> torch.Tensor:
        """One decode step of every active slot: context latents [max_seqs * q_len, H, 512] of
        the step's queries over each cache plus the step's own tokens, which are then appended."""
        if out is None:
            out = torch.empty(q_lat.shape[0], self.n_heads, LATENT_DIM, dtype=torch.bfloat16, device=self.device)
        if self._provisional:
            raise RuntimeError("accept() the pending verification step first")
        self._check_step_inputs(q_lat, q_rope, new_latent, new_rope, out)
        self.enqueue_step(q_lat, q_rope, new_latent, new_rope, out, softmax_scale=softmax_scale,
                          logit_softcap=logit_softcap)
        self.advance()
        if self.plan_ahead:  # the next step's schedule, built while this step decodes
            nxt = self._ahead_cur ^ 1
            self._plan_into(nxt)
            self._ahead_ready = nxt
        return out

    def verify(self, q_lat, q_rope, new_latent, new_rope, out=None, *, softmax_scale: float | None = None,
               logit_softcap: float | None = None) -> torch.Tensor:
        """A cache-aware verification step for multi-token prediction: the ``q_len`` tokens of every
        active slot (the last accepted token, then the drafts) attend to the cache and causally to
        each other, as ``step`` does, and are appended provisionally.  ``accept`` must follow: it
        keeps a prefix of them per slot and only then flushes, so the cache ends exactly as if
        only the accepted tokens had been appended (cache.py:186-201).

        The reference verifier re-runs the model over the whole prefix each round
        (speculative.py:45-60); here the prefix is read from the cache once."""
        if out is None:
            out = torch.empty(q_lat.shape[0], self.n_heads, LATENT_DIM, dtype=torch.bfloat16, device=self.device)
        if self._provisional:
            raise RuntimeError("accept() the previous verification step first")
        self._check_step_inputs(q_lat, q_rope, new_latent, new_rope, out)
        self.enqueue_step(q_lat, q_rope, new_latent, new_rope, out, softmax_scale=softmax_scale,
                          logit_softcap=logit_softcap)
        h = self.tables.host
        h["hot_tokens"][h["q_len"] > 0] += self.q_len
        self._provisional = True
        self._invalidate_plan()
        return out

    def accept(self, keep) -> None:
        """After ``verify``: keep the first ``keep[s]`` (1 .. q_len) of slot s's provisional tokens
        and drop the rest from its hot window (entries of empty slots are ignored); then flush and
        hand out pages as after a ``step``."""
        if not self._provisional:
            raise RuntimeError("accept() follows a verify() step")
        h = self.tables.host
        act = h["q_len"] > 0
        keep = np.asarray(keep, dtype=np.int64).reshape(-1)
        if keep.shape[0] != self.max_seqs:
            raise ValueError(f"keep must have one entry per slot ({self.max_seqs})")
        if ((keep[act] < 1) | (keep[act] > self.q_len)).any():
            raise ValueError(f"keep must be in 1..{self.q_len} for every active slot")
        h["hot_tokens"][act] -= (self.q_len - keep[act]).astype(np.int32)
        self._provisional = False
        self._settle(force_upload=True)
        self._invalidate_plan()

    def advance(self) -> None:
        """Host bookkeeping after a step's launches: advance the mirror's hot lengths, flush the
        sequences over the threshold and hand out pages the next step's tokens need."""
        h = self.tables.host
        h["hot_tokens"][h["q_len"] > 0] += self.q_len
        self._settle()

    def _settle(self, force_upload: bool = False) -> None:
        h, P = self.tables.host, self.page_tokens
        act = h["q_len"] > 0
        changed = force_upload
        over = np.nonzero(h["hot_tokens"] > self.threshold)[0]
        if over.size:
            self._flush(over)
            changed = True
        if self.window_size is not None and self._trim_windows():
            changed = True
        need = (h["hot_tokens"] + self.q_len + P - 1) // P
        have = (h["hot_pages"] >= 0).sum(axis=1)
        short = np.nonzero(act & (need > have))[0]
        for s in short:
            pages = self._hot_free.alloc(int(need[s] - have[s]))
            h["hot_pages"][s, have[s] : need[s]] = pages
            changed = True
        if changed:
            self.tables.upload()

    def _trim_windows(self) -> bool:
        """Drop the cold pages between each over-long sequence's sink and recent tokens."""
        from .cache import trim_page_range

        h, P, W = self.tables.host, self.page_tokens, self.window_size
        slack = P if W > 2 * P else 0
        trimmed = False
        for s in np.nonzero(h["q_len"] > 0)[0]:
            n = int(h["n_cold"][s])
            if self.length(s) <= W + slack or n == 0:
                continue
            rng = trim_page_range(n, h["cold_tokens"][s, :n], int(h["hot_tokens"][s]), P, W, self.sink_tokens)
            if rng is None:
                continue
            a, b = rng
            self._cold_free.release(h["cold_pages"][s, a:b])
            keep = n - (b - a)
            for name in ("cold_pages", "cold_tokens"):
                row = h[name][s]
                row[a:keep] = row[b:n].copy()
                row[keep:n] = 0
            h["n_cold"][s] = keep
            self.pages_trimmed += b - a
            trimmed = True
        return trimmed

    def _flush(self, seqs: np.ndarray) -> None:
        """cache.py:167-177 for the given slots: the oldest hot page (full) of each is encoded
        into a new cold page and released."""
        h, P = self.tables.host, self.page_tokens
        full = h["n_cold"][seqs] >= self.tables.max_cold_pages
        if full.any():
            raise RuntimeError("a sequence has no free cold-page slot (raise max_cold_pages)")
        src = h["hot_pages"][seqs, 0].astype(np.int64)
        dst = self._cold_free.alloc(len(seqs))
        si = _pinned(src).to(self.device, non_blocking=True)
        lat = self.pools.hot_latent.index_select(0, si).reshape(-1, LATENT_DIM)
        rope = self.pools.hot_rope.index_select(0, si).reshape(-1, ROPE_DIM)
        self._encode_into(lat, rope, dst)
        for i, s in enumerate(seqs):
            c = h["n_cold"][s]
            h["cold_pages"][s, c] = dst[i]
            h["cold_tokens"][s, c] = P
            h["n_cold"][s] = c + 1
            h["hot_pages"][s, :-1] = h["hot_pages"][s, 1:].copy()
            h["hot_pages"][s, -1] = -1
            h["hot_tokens"][s] -= P
        self._hot_free.release(src)
        self.flushes += len(seqs)
        self.flush_launches += 1

    def capture(self, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float | None = None,
                logit_softcap: float | None = None) -> "StepGraph":
        """Record plan + decode + append on these fixed buffers as a CUDA graph (refill the
        buffers in place between replays; ``StepGraph.replay`` also does the host bookkeeping)."""
        if self.plan_ahead:
            raise NotImplementedError("a captured step plans in-line: build the batch without plan_ahead")
        self._check_step_inputs(q_lat, q_rope, new_latent, new_rope, out)
        return StepGraph(self, (q_lat, q_rope, new_latent, new_rope, out), softmax_scale, logit_softcap)

    @property
    def last_planner(self) -> DevicePlanner:
        """The planner whose schedule the latest step decoded."""
        return self._ahead[self._ahead_cur] if (self.plan_ahead and self._ahead) else self.planner

    def raise_if_failed(self) -> None:
        """Synchronize; raise if the planner, a decode wait or an append failed."""
        self.planner.raise_if_failed()
        for pl in self._ahead:
            pl.raise_if_failed()
        if int(self.append_status.item()) != 0:
            self.append_status.zero_()
            raise RuntimeError("asterq batch_append: a sequence's hot page was missing")


class StepGraph:
    """A captured decode step of a ``PagedLatentBatch`` (plan + decode + append)."""

    def __init__(self, batch: PagedLatentBatch, buffers, softmax_scale, logit_softcap) -> None:
        self.batch, self.buffers = batch, buffers
        self.generation = batch.tables.generation
        # one eager plan + decode first (sets the kernels' launch attributes outside the capture;
        # appends nothing)
        scale = 1.0 / math.sqrt(LATENT_DIM + ROPE_DIM) if softmax_scale is None else softmax_scale
        batch.planner.plan()
        batch.planner.decode(batch.pools, *buffers, softmax_scale=scale, logit_softcap=logit_softcap)
        torch.cuda.synchronize(batch.device)
        self.graph = torch.cuda.CUDAGraph()
        # the launches are recorded but not run; the tables are left as they were
        with torch.cuda.graph(self.graph):
            batch.enqueue_step(*buffers, softmax_scale=softmax_scale, logit_softcap=logit_softcap)

    def replay(self) -> torch.Tensor:
        if self.generation != self.batch.tables.generation:
            raise RuntimeError("the batch's tables were reallocated since capture: capture the step again")
        self.graph.replay()
        self.batch.advance()
        return self.buffers[4]
