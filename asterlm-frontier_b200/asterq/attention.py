"""Drop-in for the attention side of AsterLM's global layer (src/asterlm/layers/latent_attention.py).

``latent_attention`` is the kernel call both reference code paths reduce to once
the key/value up-projections are absorbed into the query and the output
(latent_attention.py:186-188 and :231):

* ``_absorbed_decode`` (:177-231, T = 1): online softmax over the cold chunks,
  the hot window, then the new token itself;
* ``_full_attention`` (:116-175, T > 1): the whole cache plus the T new tokens,
  new token i seeing new tokens 0..i (mask ``k <= past_len + i``, :151-153).

Scores are ``(q_latent . latent + q_rope . rope) * scale`` with
``scale = 1 / sqrt(head_dim + rope_dim)`` (:189), optional ``logit_softcap``
(:200-201), and the result is ``context / max(sum, 1e-20)`` (:229).

``LatentAttentionKernels`` keeps the reference method names and arguments for a
module that owns the ``k_up`` / ``v_up`` weights; the absorption einsums are
plain library GEMMs around the decode kernel.
"""
from __future__ import annotations

import math

import torch

from .cache import LatentLayerCache
from .decode import COLD_TILE_TOKENS, LATENT_DIM, ROPE_DIM, DeviceDecodePlan, LatentPools, latent_decode
from .plan import MAX_Q_LEN, SequenceLayout, build_plan


def _empty_pools(device) -> LatentPools:
    return LatentPools.empty(0, 0, 16, device)


def latent_attention(
    q_latent: torch.Tensor,
    q_rope: torch.Tensor,
    latent: torch.Tensor,
    k_rope: torch.Tensor,
    cache: LatentLayerCache | None,
    *,
    softmax_scale: float,
    logit_softcap: float | None = None,
    out_dtype: torch.dtype | None = None,
    **plan_kw,
) -> torch.Tensor:
    """Context latents [B, T, H, 512] of T new tokens per batch row over ``cache`` plus themselves.

    q_latent [B, T, H, 512], q_rope [B, T, H, 64], latent [B, T, 512] and k_rope
    [B, T, 64] are the step's absorbed queries and new cache entries (RoPE
    already applied).  The cache is read in place; it is not modified.
    """
    if q_latent.dim() != 4 or q_latent.shape[-1] != LATENT_DIM:
        raise ValueError("q_latent must be [B, T, H, 512]")
    bsz, t, n_heads, _ = q_latent.shape
    if q_rope.shape != (bsz, t, n_heads, ROPE_DIM):
        raise ValueError("q_rope must be [B, T, H, 64]")
    if latent.shape != (bsz, t, LATENT_DIM) or k_rope.shape != (bsz, t, ROPE_DIM):
        raise ValueError("latent / k_rope must be [B, T, 512] / [B, T, 64]")
    if not 0 < t <= MAX_Q_LEN:
        raise ValueError(f"the decode kernels take 1..{MAX_Q_LEN} new tokens per step (got {t})")
    dev = q_latent.device
    bf = torch.bfloat16
    args = (q_latent.reshape(bsz * t, n_heads, LATENT_DIM).to(bf).contiguous(),
            q_rope.reshape(bsz * t, n_heads, ROPE_DIM).to(bf).contiguous(),
            latent.reshape(bsz * t, LATENT_DIM).to(bf).contiguous(),
            k_rope.reshape(bsz * t, ROPE_DIM).to(bf).contiguous())
    kernel_dtype = torch.float32 if out_dtype in (None, torch.float32) else torch.bfloat16
    if cache is not None and cache.length:
        if cache.batch_size != bsz:
            raise ValueError(f"cache holds {cache.batch_size} rows, the step has {bsz}")
        pools = cache.pools()
        if not plan_kw:
            # the step planned on the GPU from the cache's device page tables (kept across calls)
            planner = cache.device_planner(n_heads, t)
            planner.plan()
            out = torch.empty(bsz * t, n_heads, LATENT_DIM, dtype=kernel_dtype, device=dev)
            planner.decode(pools, *args, out, softmax_scale=softmax_scale, logit_softcap=logit_softcap)
            out = out.view(bsz, t, n_heads, LATENT_DIM)
            return out if out_dtype is None else out.to(out_dtype)
        layouts = cache.decode_layouts(t)
    else:
        pools = _empty_pools(dev)
        layouts = [SequenceLayout(q_start=b * t, q_len=t) for b in range(bsz)]
    # host-built schedule: an empty cache, or explicit planner options (plan_kw)
    plan_kw.setdefault("cold_tile", COLD_TILE_TOKENS.get(pools.cold_scheme, 128))
    plan = build_plan(layouts, n_heads, **plan_kw)
    dplan = DeviceDecodePlan(plan, dev)
    out = latent_decode(pools, dplan, *args, softmax_scale=softmax_scale, logit_softcap=logit_softcap,
                        out_dtype=kernel_dtype)
    out = out.view(bsz, t, n_heads, LATENT_DIM)
    return out if out_dtype is None else out.to(out_dtype)


class LatentAttentionKernels:
    """Kernel-backed ``_absorbed_decode`` / ``_full_attention`` for one layer's weights.

    ``k_up_weight`` / ``v_up_weight`` are the reference's ``k_up.weight`` /
    ``v_up.weight`` ([H * head_dim, 512]); they are viewed as [H, head_dim, 512]
    exactly as latent_attention.py:186-187 does.
    """

    def __init__(self, k_up_weight: torch.Tensor, v_up_weight: torch.Tensor, n_heads: int, head_dim: int,
                 rope_dim: int = ROPE_DIM, logit_softcap: float | None = None) -> None:
        if rope_dim != ROPE_DIM:
            raise NotImplementedError(f"rope_dim {rope_dim}: the kernels use {ROPE_DIM}")
        self.n_heads, self.head_dim, self.rope_dim = n_heads, head_dim, rope_dim
        self.wk = k_up_weight.view(n_heads, head_dim, LATENT_DIM)
        self.wv = v_up_weight.view(n_heads, head_dim, LATENT_DIM)
        self.logit_softcap = logit_softcap
        self.scale = 1.0 / math.sqrt(head_dim + rope_dim)

    def _context(self, q_content, q_rope, latent, k_rope, previous) -> torch.Tensor:
        q_latent = torch.einsum("bthd,hdl->bthl", q_content, self.wk)
        ctx = latent_attention(q_latent, q_rope, latent, k_rope, previous, softmax_scale=self.scale,
                               logit_softcap=self.logit_softcap, out_dtype=q_content.dtype)
        return torch.einsum("bthl,hdl->bthd", ctx, self.wv)

    def _absorbed_decode(self, q_content, q_rope, latent, k_rope, previous: LatentLayerCache) -> torch.Tensor:
        """latent_attention.py:177-231 (one new token per row)."""
        if q_content.shape[1] != 1:
            raise ValueError("_absorbed_decode takes one token per row")
        return self._context(q_content, q_rope, latent, k_rope, previous)

    def _full_attention(self, q_content, q_rope, latent, k_rope, previous: LatentLayerCache | None) -> torch.Tensor:
        """latent_attention.py:116-175 for T <= 2048 new tokens (MTP verification, prefill chunks)."""
        return self._context(q_content, q_rope, latent, k_rope, previous)
