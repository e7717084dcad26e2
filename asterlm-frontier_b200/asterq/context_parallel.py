"""Context-parallel decode of long sequences (config C4) across ranks.

The cold chunks of a sequence are split into contiguous ranges, one per rank,
balanced by the bytes a decode step streams (the last rank also holds the hot
window and the step's new tokens, so it takes fewer chunks).  Each rank:

1. runs the split-KV decode over its own pages, every work item writing an
   (m, l, o) partial record (``build_plan(..., force_partial=True)``);
2. merges its records into one record per 16-row block with
   ``asterq_splitkv_merge`` (about 33 KB per row block);
3. exchanges the merged records with one ``all_gather`` over the process group
   (NCCL on GPUs; the records are fp32 in the workspace layout);
4. combines the gathered records where they landed with
   ``asterq_splitkv_combine_ranks`` into the context latents, identically on
   every rank.

``capture`` records the four steps as one CUDA graph per rank.

With a ``PeerExchange`` (``use_peer_exchange``), steps 2-4 become two kernels and no
collective: ``asterq_cp_merge_push`` merges the rank's records and stores the merged record
into every rank's mailbox (device memory mapped between the rank processes through CUDA IPC,
written with plain stores over NVLink), then raises the rank's flag in each; and
``asterq_cp_combine_wait`` waits (bounded) for every rank's flag and combines the records from
local memory.

The merge rule is the reference's online softmax (latent_attention.py:212-220)
applied across ranks instead of across chunks.  No TMA or library kernel reads
another GPU's memory: the records arrive by NCCL into local buffers.
"""
from __future__ import annotations

import ctypes
from dataclasses import replace

import torch

from . import _lib
from .decode import COLD_TILE_TOKENS, LATENT_DIM, DeviceDecodePlan, LatentPools, capture_step, make_params
from .plan import ROWS_PER_BLOCK, SequenceLayout, build_plan
from .sharding import COLD_TOKEN_BYTES, HOT_TOKEN_BYTES

RECORD_FLOATS = ROWS_PER_BLOCK * (LATENT_DIM + 2)


def split_chunks(chunk_tokens: list[int], hot_tokens: int, world: int, q_len: int = 1) -> list[tuple[int, int]]:
    """Contiguous [begin, end) ranges of cold chunks per rank; the hot window and new tokens go to the last rank.

    Ranges are cut at equal shares of the step's total bytes, counting the last
    rank's hot window and new tokens as part of its share.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    n = len(chunk_tokens)
    costs = [t * COLD_TOKEN_BYTES for t in chunk_tokens]
    total = sum(costs) + (hot_tokens + q_len) * HOT_TOKEN_BYTES
    share = total / world
    bounds = [0]
    acc = 0.0
    i = 0
    for r in range(world - 1):
        target = share * (r + 1)
        while i < n and acc + costs[i] / 2 <= target:
            acc += costs[i]
            i += 1
        bounds.append(i)
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def rank_layout(layout: SequenceLayout, rank: int, world: int) -> SequenceLayout:
    """The part of one sequence's layout that `rank` reads."""
    ranges = split_chunks([c[2] for c in layout.cold], layout.hot_tokens, world, layout.q_len)
    a, b = ranges[rank]
    last = rank == world - 1
    return replace(layout, cold=list(layout.cold[a:b]), hot=list(layout.hot) if last else [], attend_new=last)


class PeerExchange:
    """Mailboxes for exchanging merged records between the ranks of one process group.

    Every rank allocates one mailbox in its own device memory (``asterq_mailbox_create``),
    the ranks swap CUDA IPC handles over the group (``all_gather_object``), and each maps its
    peers' mailboxes.  ``close`` must run on every rank after all ranks have finished their
    last step (a barrier first), or a peer could still be writing into a freed mailbox.
    """

    def __init__(self, n_blocks: int, rank: int, world: int, device, *, group=None,
                 wait_limit_cycles: int = 0) -> None:
        import torch.distributed as dist

        lib = _lib.load()
        self.rank, self.world, self.n_blocks = rank, world, n_blocks
        self.device = torch.device(device)
        self.group = group
        self.wait_limit_cycles = int(wait_limit_cycles)
        nbytes = lib.asterq_mailbox_bytes(world, n_blocks, LATENT_DIM)
        if nbytes <= 0:
            raise ValueError(f"no mailbox for world {world}, {n_blocks} blocks")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check(lib.asterq_mailbox_create(nbytes, ctypes.byref(own), handle))
        self.own = own.value
        handles: list = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers: list[int] = []
        ptrs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == rank:
                    ptrs.append(self.own)
                    continue
                buf = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
                peer = ctypes.c_void_p()
                _lib.check(lib.asterq_mailbox_open(buf, ctypes.byref(peer)))
                self.peers.append(peer.value)
                ptrs.append(peer.value)
        self.table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def raise_if_failed(self) -> None:
        """Synchronize; raise if a combine gave up waiting for a rank's records."""
        if int(self.status.item()) != 0:
            self.status.zero_()
            raise RuntimeError("asterq context parallel: a rank's records did not arrive in time")

    def close(self) -> None:
        import torch.distributed as dist

        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank writes into a mailbox any more
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for peer in self.peers:
                _lib.check(lib.asterq_mailbox_close(peer))
            _lib.check(lib.asterq_mailbox_destroy(self.own))
        self.peers, self.own = [], None


class ContextParallelDecoder:
    """One rank's share of a context-parallel decode step for one sequence (B = 1)."""

    def __init__(self, pools: LatentPools, layout: SequenceLayout, n_heads: int, rank: int, world: int,
                 device, **plan_kw) -> None:
        self.pools, self.rank, self.world, self.n_heads = pools, rank, world, n_heads
        self.device = torch.device(device)
        self.local = rank_layout(replace(layout, q_start=0), rank, world)
        plan_kw.setdefault("cold_tile", COLD_TILE_TOKENS.get(pools.cold_scheme, 128))
        self.plan = build_plan([self.local], n_heads, force_partial=True, **plan_kw)
        self.dplan = DeviceDecodePlan(self.plan, self.device)
        self.n_rb = int(self.plan.combine.shape[0])
        self.q_len = layout.q_len
        self.merged = torch.empty(self.n_rb * RECORD_FLOATS, dtype=torch.float32, device=self.device)
        self.gathered = torch.empty(world * self.n_rb * RECORD_FLOATS, dtype=torch.float32, device=self.device)
        # job rb merges record rb of every rank (asterq_splitkv_combine_ranks)
        jobs = [(0, world, int(self.plan.combine[rb, 2]), int(self.plan.combine[rb, 3])) for rb in range(self.n_rb)]
        self.final_jobs = torch.tensor(jobs, dtype=torch.int32, device=self.device).reshape(-1, 4)
        self.exchange: PeerExchange | None = None
        # the decode's own output rows stay unwritten (every item writes partial records)
        self._unused_out = torch.empty(layout.q_len, n_heads, LATENT_DIM, dtype=torch.float32, device=self.device)

    def partial(self, q_lat, q_rope, new_latent, new_rope, *, softmax_scale: float,
                logit_softcap: float | None = None) -> torch.Tensor:
        """Steps 1-2: this rank's merged (m, l, o) records, [n_rb * 16 * 514] fp32."""
        stream = self._decode_records(q_lat, q_rope, new_latent, new_rope, softmax_scale=softmax_scale,
                                      logit_softcap=logit_softcap)
        lib = _lib.load()
        _lib.check(lib.asterq_splitkv_merge(self.dplan.workspace.data_ptr(), self.plan.n_slots,
                                            self.dplan.combine.data_ptr(), self.n_rb, LATENT_DIM,
                                            self.merged.data_ptr(), stream))
        return self.merged

    def _decode_records(self, q_lat, q_rope, new_latent, new_rope, *, softmax_scale: float,
                        logit_softcap: float | None = None) -> int:
        """Step 1: this rank's split-KV partial records into the workspace; returns the stream."""
        out = self._unused_out
        if out.shape[0] != q_lat.shape[0]:
            out = torch.empty(q_lat.shape[0], self.n_heads, LATENT_DIM, dtype=torch.float32, device=self.device)
        p = make_params(self.pools, self.dplan, q_lat, q_rope, new_latent, new_rope, out, n_heads=self.n_heads,
                        softmax_scale=softmax_scale, logit_softcap=logit_softcap)
        p.n_combine = 0  # the records are merged later, not combined
        stream = _lib.stream_handle(self.device)
        _lib.check(_lib.load().asterq_latent_decode(ctypes.byref(p), stream))
        return stream

    def use_peer_exchange(self, group=None, *, wait_limit_cycles: int = 0) -> "PeerExchange":
        """Set up mailboxes with the other ranks of `group` (collective: every rank calls it);
        ``step`` then exchanges records by peer stores instead of ``all_gather``."""
        self.exchange = PeerExchange(self.n_rb, self.rank, self.world, self.device, group=group,
                                     wait_limit_cycles=wait_limit_cycles)
        return self.exchange

    def step_peer(self, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float,
                  logit_softcap: float | None = None) -> torch.Tensor:
        """Steps 1-4 with the peer exchange: decode, merge + push to every rank, wait + combine."""
        ex = self.exchange
        stream = self._decode_records(q_lat, q_rope, new_latent, new_rope, softmax_scale=softmax_scale,
                                      logit_softcap=logit_softcap)
        lib = _lib.load()
        _lib.check(lib.asterq_cp_merge_push(self.dplan.workspace.data_ptr(), self.plan.n_slots,
                                            self.dplan.combine.data_ptr(), self.n_rb, LATENT_DIM,
                                            ex.table.data_ptr(), self.world, self.rank, stream))
        dtype = _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16
        _lib.check(lib.asterq_cp_combine_wait(ex.own, self.world, self.n_rb, self.final_jobs.data_ptr(), LATENT_DIM,
                                              out.data_ptr(), dtype, ex.wait_limit_cycles, ex.status.data_ptr(),
                                              stream))
        return out

    def finish(self, gathered: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Step 4: combine the records of all ranks (rank-major as all_gather leaves them) into `out`.

        ``asterq_splitkv_combine_ranks`` reads the gathered records in place.
        """
        dtype = _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16
        lib = _lib.load()
        _lib.check(lib.asterq_splitkv_combine_ranks(gathered.data_ptr(), self.world, self.n_rb,
                                                    self.final_jobs.data_ptr(), LATENT_DIM, out.data_ptr(), dtype,
                                                    _lib.stream_handle(self.device)))
        return out

    def step(self, q_lat, q_rope, new_latent, new_rope, out, *, group=None, softmax_scale: float,
             logit_softcap: float | None = None) -> torch.Tensor:
        """Steps 1-4 with ``torch.distributed.all_gather_into_tensor`` over `group`."""
        import torch.distributed as dist

        rec = self.partial(q_lat, q_rope, new_latent, new_rope, softmax_scale=softmax_scale,
                           logit_softcap=logit_softcap)
        dist.all_gather_into_tensor(self.gathered, rec, group=group)
        return self.finish(self.gathered, out)

    def capture(self, q_lat, q_rope, new_latent, new_rope, out, *, group=None, softmax_scale: float,
                logit_softcap: float | None = None) -> torch.cuda.CUDAGraph:
        """``step`` recorded as one CUDA graph (decode, merge, all-gather, combine) on these buffers.

        Each ``replay()`` is one context-parallel step with no Python between the
        launches; every rank must capture and replay in the same order.  Refill the
        inputs in place between replays, and release the graph before the process
        group is destroyed (it holds an NCCL collective).
        """
        return capture_step(lambda: self.step(q_lat, q_rope, new_latent, new_rope, out, group=group,
                                              softmax_scale=softmax_scale, logit_softcap=logit_softcap),
                            self.device)

    def capture_peer(self, q_lat, q_rope, new_latent, new_rope, out, *, softmax_scale: float,
                     logit_softcap: float | None = None) -> torch.cuda.CUDAGraph:
        """``step_peer`` recorded as one CUDA graph (decode, merge-push, combine-wait); every rank
        replays its graph once per step, in the same order.  The step number lives in the
        mailbox, so replays need no host bookkeeping."""
        return capture_step(lambda: self.step_peer(q_lat, q_rope, new_latent, new_rope, out,
                                                   softmax_scale=softmax_scale, logit_softcap=logit_softcap),
                            self.device)
