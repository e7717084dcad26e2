"""Batched split-KV decode over paged latent pools (the ``asterq_latent_decode`` C ABI).

``LatentPools`` holds the five device pools of one global-attention layer;
``DeviceDecodePlan`` uploads a ``DecodePlan`` and owns the partial-record
workspace, so that a decode step is one C call with no allocation (and can be
captured in a CUDA graph by the caller).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from .plan import DecodePlan

LATENT_DIM = 512
ROPE_DIM = 64
GROUP_SIZE = 64
COLD_SCHEMES = {"hadamard_int4": _lib.SCHEME_HADAMARD_INT4, "int4": _lib.SCHEME_INT4, "int8": _lib.SCHEME_INT8,
                "float8": _lib.SCHEME_FLOAT8}
# tokens of a cold tile per scheme (the host and device planners cut pages into such tiles)
COLD_TILE_TOKENS = {"hadamard_int4": 128, "int4": 128, "int8": 64, "float8": 64}
# one code byte a dim (512 a token) for these schemes, two dims a byte for the INT4 ones
BYTE_SCHEMES = ("int8", "float8")


@dataclass
class LatentPools:
    """Device pools (layout documented in include/asterq.h)."""

    cold_codes: torch.Tensor  # uint8 [Pc, page, 256] INT4 codes, or [Pc, page, 512] int8 codes / e4m3 bytes
    cold_scales: torch.Tensor  # fp16 [Pc, page, 8] (float8: [Pc, page, 0], no scales)
    cold_rope: torch.Tensor  # bf16 [Pc, page, 64], or uint8 [Pc, page, 32] INT4 codes (quantized RoPE keys)
    hot_latent: torch.Tensor  # bf16 [Ph, page, 512]
    hot_rope: torch.Tensor  # bf16 [Ph, page, 64]
    cold_scheme: str = "hadamard_int4"  # or "int4": plain groupwise codes, same layout
    # fp16 [Pc, page]: one scale per token of quantized cold RoPE keys (quantize_rope=True,
    # cache.py:160-164), whose codes (cold scheme, one group of 64) are in cold_rope
    cold_rope_scales: torch.Tensor | None = None

    @property
    def page_tokens(self) -> int:
        return int(self.cold_codes.shape[1] if self.cold_codes.numel() else self.hot_latent.shape[1])

    @property
    def rope_quantized(self) -> bool:
        return self.cold_rope.element_size() == 1

    @staticmethod
    def empty(n_cold_pages: int, n_hot_pages: int, page_tokens: int, device, *,
              quantize_rope: bool = False, cold_scheme: str = "hadamard_int4") -> "LatentPools":
        if cold_scheme not in COLD_SCHEMES:
            raise NotImplementedError(f"cold scheme {cold_scheme!r}: the decode kernels read {tuple(COLD_SCHEMES)}")
        n_scales = LATENT_DIM // GROUP_SIZE
        if cold_scheme == "int8":
            codes = torch.empty(n_cold_pages, page_tokens, LATENT_DIM, dtype=torch.int8, device=device)
        elif cold_scheme == "float8":
            codes = torch.empty(n_cold_pages, page_tokens, LATENT_DIM, dtype=torch.uint8, device=device)  # e4m3 bytes
            n_scales = 0
        else:
            codes = torch.empty(n_cold_pages, page_tokens, LATENT_DIM // 2, dtype=torch.uint8, device=device)
        if quantize_rope:
            # RoPE codes of the cold scheme: 32 bytes a token (INT4) or 64 (int8, float8); one fp16
            # scale a token but for float8
            width = ROPE_DIM if cold_scheme in BYTE_SCHEMES else ROPE_DIM // 2
            rdt = torch.int8 if cold_scheme == "int8" else torch.uint8
            cold_rope = torch.empty(n_cold_pages, page_tokens, width, dtype=rdt, device=device)
            rope_scales = (None if cold_scheme == "float8"
                           else torch.empty(n_cold_pages, page_tokens, dtype=torch.float16, device=device))
        else:
            cold_rope = torch.empty(n_cold_pages, page_tokens, ROPE_DIM, dtype=torch.bfloat16, device=device)
            rope_scales = None
        return LatentPools(
            cold_codes=codes,
            cold_scales=torch.empty(n_cold_pages, page_tokens, n_scales, dtype=torch.float16, device=device),
            cold_rope=cold_rope,
            hot_latent=torch.empty(n_hot_pages, page_tokens, LATENT_DIM, dtype=torch.bfloat16, device=device),
            hot_rope=torch.empty(n_hot_pages, page_tokens, ROPE_DIM, dtype=torch.bfloat16, device=device),
            cold_rope_scales=rope_scales,
            cold_scheme=cold_scheme,
        )

    @property
    def num_bytes(self) -> int:
        parts = [self.cold_codes, self.cold_scales, self.cold_rope, self.hot_latent, self.hot_rope]
        if self.cold_rope_scales is not None:
            parts.append(self.cold_rope_scales)
        return sum(t.numel() * t.element_size() for t in parts)


def set_cold_pools(p: _lib.DecodeParams, pools: LatentPools) -> None:
    """The cold-pool fields of ``asterq_decode_params``: codes, scales, RoPE keys (bf16, or
    quantized codes with their scales) and the cold scheme."""
    p.n_cold_pages = int(pools.cold_codes.shape[0])
    p.cold_codes = pools.cold_codes.data_ptr() if pools.cold_codes.numel() else None
    p.cold_scales = pools.cold_scales.data_ptr() if pools.cold_scales.numel() else None
    p.cold_rope = pools.cold_rope.data_ptr() if pools.cold_rope.numel() else None
    if pools.rope_quantized:
        width = ROPE_DIM if pools.cold_scheme in BYTE_SCHEMES else ROPE_DIM // 2
        if pools.cold_rope.shape[-1] != width:
            raise ValueError(f"quantized cold RoPE keys of scheme {pools.cold_scheme!r}: cold_rope [Pc, page, {width}]")
        if pools.cold_scheme == "float8":
            p.cold_rope_scales = None
        else:
            if pools.cold_rope_scales is None or pools.cold_rope_scales.dtype != torch.float16:
                raise ValueError("quantized cold RoPE keys need cold_rope_scales fp16 [Pc, page]")
            p.cold_rope_scales = pools.cold_rope_scales.data_ptr() if pools.cold_rope_scales.numel() else None
        p.rope_scheme = _lib.ROPE_QUANTIZED
    else:
        p.rope_scheme = _lib.ROPE_BF16
        p.cold_rope_scales = None
    if pools.cold_scheme not in COLD_SCHEMES:
        raise NotImplementedError(f"cold scheme {pools.cold_scheme!r}: the decode kernels read {COLD_SCHEMES}")
    width = LATENT_DIM if pools.cold_scheme in BYTE_SCHEMES else LATENT_DIM // 2
    if pools.cold_codes.numel() and (pools.cold_codes.shape[-1] != width or pools.cold_codes.element_size() != 1):
        raise ValueError(f"cold_codes of scheme {pools.cold_scheme!r} must be one-byte [Pc, page, {width}]")
    p.cold_scheme = COLD_SCHEMES[pools.cold_scheme]


class DeviceDecodePlan:
    """A ``DecodePlan`` resident on the device plus its workspace."""

    def __init__(self, plan: DecodePlan, device) -> None:
        self.plan = plan
        self.device = torch.device(device)

        def up(a):
            t = torch.from_numpy(a.copy()) if a.size else torch.zeros(1, 4, dtype=torch.int32)
            return t.to(self.device)

        self.tiles = up(plan.tiles)
        self.items = up(plan.items)
        self.combine = up(plan.combine)
        self.units = up(plan.units)
        self.workers = None if plan.workers is None else torch.from_numpy(plan.workers.copy()).to(self.device)
        self.unit_jobs = None if plan.unit_jobs is None else torch.from_numpy(plan.unit_jobs.copy()).to(self.device)
        self.workspace = torch.empty(max(4, plan.workspace_bytes // 4), dtype=torch.float32, device=self.device)
        # set nonzero by the kernel when one of its bounded pipeline waits ran out
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def n_items(self) -> int:
        return int(self.plan.items.shape[0])

    def raise_if_failed(self) -> None:
        """Synchronize and raise ``RuntimeError`` if a decode on this plan timed out in a pipeline
        wait (the kernel stopped instead of hanging; its output is not valid).  Clears the status."""
        if int(self.status.item()) != 0:
            self.status.zero_()
            raise RuntimeError("asterq decode: a pipeline wait timed out on the device (output not valid)")


def make_params(
    pools: LatentPools,
    dplan: DeviceDecodePlan,
    q_lat: torch.Tensor,
    q_rope: torch.Tensor,
    new_latent: torch.Tensor,
    new_rope: torch.Tensor,
    out: torch.Tensor,
    *,
    n_heads: int,
    softmax_scale: float,
    logit_softcap: float | None = None,
    wait_limit_cycles: int = 0,
) -> _lib.DecodeParams:
    plan = dplan.plan
    want = COLD_TILE_TOKENS.get(pools.cold_scheme, 128)
    if pools.cold_codes.numel() and plan.cold_tile != want:
        raise ValueError(f"the plan cuts cold tiles of {plan.cold_tile} tokens; scheme {pools.cold_scheme!r} "
                         f"needs {want} (build_plan(..., cold_tile={want}))")
    p = _lib.DecodeParams()
    p.n_heads = n_heads
    p.latent_dim = LATENT_DIM
    p.rope_dim = ROPE_DIM
    p.group_size = GROUP_SIZE
    p.page_tokens = int(pools.cold_codes.shape[1] if pools.cold_codes.dim() == 3 and pools.cold_codes.shape[0] else pools.hot_latent.shape[1])
    p.out_dtype = _lib.DTYPE_F32 if out.dtype == torch.float32 else _lib.DTYPE_BF16
    p.softmax_scale = float(softmax_scale)
    p.logit_softcap = float(logit_softcap) if logit_softcap else 0.0
    set_cold_pools(p, pools)
    p.n_hot_pages = int(pools.hot_latent.shape[0])
    p.total_q = int(q_lat.shape[0])
    p.n_tiles = int(plan.tiles.shape[0])
    p.n_items = int(plan.items.shape[0])
    p.n_combine = plan.n_separate  # jobs for the combine launch; the rest run inside the decode kernel
    p.n_combine_total = int(plan.combine.shape[0])
    p.n_slots = int(plan.n_slots)
    p.q_lat = q_lat.data_ptr()
    p.q_rope = q_rope.data_ptr()
    p.new_latent = new_latent.data_ptr()
    p.new_rope = new_rope.data_ptr()
    p.hot_latent = pools.hot_latent.data_ptr() if pools.hot_latent.numel() else None
    p.hot_rope = pools.hot_rope.data_ptr() if pools.hot_rope.numel() else None
    p.tiles = dplan.tiles.data_ptr()
    p.items = dplan.items.data_ptr()
    p.combine = dplan.combine.data_ptr()
    p.out = out.data_ptr()
    p.workspace = dplan.workspace.data_ptr()
    p.workspace_bytes = dplan.workspace.numel() * 4
    p.units = dplan.units.data_ptr()
    p.n_units = int(plan.n_units)
    if dplan.workers is not None and plan.n_workers > 0:
        p.workers = dplan.workers.data_ptr()
        p.n_workers = plan.n_workers
    if dplan.unit_jobs is not None:
        p.unit_jobs = dplan.unit_jobs.data_ptr()
    p.device_status = dplan.status.data_ptr()
    p.wait_limit_cycles = int(wait_limit_cycles)
    return p


def _check_inputs(q_lat, q_rope, new_latent, new_rope, n_heads):
    for name, t in (("q_lat", q_lat), ("q_rope", q_rope), ("new_latent", new_latent), ("new_rope", new_rope)):
        if not t.is_cuda:
            raise RuntimeError(f"{name}: asterq kernels need CUDA tensors; there is no CPU path")
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bfloat16 (got {t.dtype})")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if q_lat.dim() != 3 or q_lat.shape[1:] != (n_heads, LATENT_DIM):
        raise ValueError(f"q_lat must be [total_q, {n_heads}, {LATENT_DIM}] (got {tuple(q_lat.shape)})")
    if q_rope.shape != (q_lat.shape[0], n_heads, ROPE_DIM):
        raise ValueError(f"q_rope must be [total_q, {n_heads}, {ROPE_DIM}] (got {tuple(q_rope.shape)})")
    if new_latent.shape != (q_lat.shape[0], LATENT_DIM) or new_rope.shape != (q_lat.shape[0], ROPE_DIM):
        raise ValueError("new_latent / new_rope must be [total_q, 512] / [total_q, 64]")


def capture_step(fn, device, warmup: int = 3) -> "torch.cuda.CUDAGraph":
    """Record `fn` (a decode step on fixed buffers) as a CUDA graph; replay it with ``.replay()``.

    `fn` runs `warmup` times eagerly on a side stream first (NCCL collectives
    need that before capture).  Every tensor `fn` reads or writes must stay
    allocated while the graph lives; refill inputs in place between replays.
    A graph holding an NCCL collective must be released before the process
    group is destroyed.
    """
    dev = torch.device(device)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def latent_decode(
    pools: LatentPools,
    dplan: DeviceDecodePlan,
    q_lat: torch.Tensor,
    q_rope: torch.Tensor,
    new_latent: torch.Tensor,
    new_rope: torch.Tensor,
    *,
    softmax_scale: float | None = None,
    logit_softcap: float | None = None,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    wait_limit_cycles: int = 0,
) -> torch.Tensor:
    """Context latents [total_q, H, 512] for every query row of the batch.

    ``softmax_scale`` defaults to 1/sqrt(512 + 64) (latent_attention.py:189 with
    head_dim = latent_dim under absorption).  Nothing synchronizes the host: a decode whose
    pipeline wait ran out (after ``wait_limit_cycles`` SM cycles, 0: about 2 s) leaves the
    plan's status set, which ``dplan.raise_if_failed()`` turns into ``RuntimeError``.
    """
    n_heads = dplan.plan.n_heads
    _check_inputs(q_lat, q_rope, new_latent, new_rope, n_heads)
    if q_lat.shape[0] < dplan.plan.total_q:
        raise ValueError("q arrays are shorter than the plan's total_q")
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(LATENT_DIM + ROPE_DIM)
    if out is None:
        out = torch.empty(q_lat.shape[0], n_heads, LATENT_DIM, dtype=out_dtype, device=q_lat.device)
    elif out.dtype not in (torch.float32, torch.bfloat16) or out.shape != (q_lat.shape[0], n_heads, LATENT_DIM):
        raise ValueError("out must be float32/bfloat16 [total_q, H, 512]")
    p = make_params(pools, dplan, q_lat, q_rope, new_latent, new_rope, out, n_heads=n_heads,
                    softmax_scale=softmax_scale, logit_softcap=logit_softcap, wait_limit_cycles=wait_limit_cycles)
    lib = _lib.load()
    _lib.check(lib.asterq_latent_decode(ctypes.byref(p), _lib.stream_handle(q_lat.device)))
    return out
