"""The drop-in inside the reference model itself.

AsterLM (the unmodified reference package installed under ``baseline/_ref``) runs with
its global-attention layers' cache and attention replaced by asterq's, the way the
integration notes show a maintainer doing it: ``asterlm.cache.LatentLayerCache`` becomes
the paged ``asterq.cache.LatentLayerCache`` and ``LatentAttention._absorbed_decode`` /
``_full_attention`` call ``asterq.attention.LatentAttentionKernels``.  Checked on a
small model with the kernels' geometry (latent rank 512, RoPE 64, 16 heads):

* cached decode equals the full forward (the reference's own pin, tests/test_model.py:41-50),
  now with both paths on the kernels;
* with the Hadamard-INT4 cache and flushes happening during the run, the patched model's
  logits follow the unpatched reference model's at every step of ``generate_tokens``
  (decode.py:95-129), and greedy generation produces the same tokens.

The kernels take bf16 queries and latents (the reference's production dtype), so logits of
an fp32 model differ from the fp32 reference by bf16 rounding of those operands; the
tolerances below are stated for that.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REF_DIR = Path(__file__).resolve().parent.parent / "baseline" / "_ref"

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not (REF_DIR / "asterlm").is_dir(),
                       reason="the reference package is not installed under baseline/_ref"),
]


@pytest.fixture(scope="module")
def ref():
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import asterlm
    import asterlm.cache
    import asterlm.generation.decode
    import asterlm.layers.latent_attention

    return asterlm


def tiny_config(ref, **changes):
    values = dict(vocab_size=96, d_model=512, n_layers=4, n_heads=16, head_dim=32, ffn_hidden=1024, max_seq_len=256,
                  kda_ratio=1, kda_backend="torch", latent_rank=512, rope_dim=64, attention_window=None,
                  sink_tokens=0, mtp_depth=0, gradient_checkpointing=False)
    values.update(changes)
    return ref.AsterConfig(**values)


class _Patched:
    """Context manager: route the reference's global-attention cache and attention to asterq."""

    def __init__(self, ref):
        self.ref = ref

    def __enter__(self):
        from asterq.attention import LatentAttentionKernels
        from asterq.cache import LatentLayerCache

        la = self.ref.layers.latent_attention.LatentAttention
        self.saved = (self.ref.cache.LatentLayerCache, la._absorbed_decode, la._full_attention)

        def kernels(module):
            return LatentAttentionKernels(module.k_up.weight, module.v_up.weight, module.n_heads, module.head_dim,
                                          module.rope_dim, module.logit_softcap)

        def absorbed(module, q_content, q_rope, latent, k_rope, previous):
            return kernels(module)._absorbed_decode(q_content, q_rope, latent, k_rope, previous)

        def full(module, q_content, q_rope, latent, k_rope, previous):
            return kernels(module)._full_attention(q_content, q_rope, latent, k_rope, previous)

        self.ref.cache.LatentLayerCache = LatentLayerCache
        la._absorbed_decode = absorbed
        la._full_attention = full
        return self

    def __exit__(self, *exc):
        la = self.ref.layers.latent_attention.LatentAttention
        self.ref.cache.LatentLayerCache, la._absorbed_decode, la._full_attention = self.saved


def test_cached_decode_matches_full_forward_on_the_kernels(cuda, ref):
    torch.manual_seed(4)
    model = ref.AsterLM(tiny_config(ref)).to(cuda).eval()
    ids = torch.randint(0, 96, (1, 40), device=cuda)
    with _Patched(ref), torch.no_grad():
        full = model(ids).logits[:, -1]
        cache = model.make_cache()
        model(ids[:, :-1], cache=cache, use_cache=True)
        layer = next(iter(cache.latent.values()))
        assert type(layer).__module__ == "asterq.cache"  # the paged cache is the one in use
        cached = model(ids[:, -1:], cache=cache, use_cache=True).logits[:, -1]
    # both paths read the same bf16 latents; they differ by fp32 accumulation order only
    torch.testing.assert_close(cached, full, rtol=1e-3, atol=1e-3)


def test_generation_follows_the_reference_with_int4_flushes(cuda, ref):
    """Hadamard-INT4 cache with recent 64 / chunk 64: a chunk is flushed once the hot window
    exceeds 128 tokens (cache.py:167-176), which the 96-token prompt reaches at decode step 33.
    The patched model's next-token logits stay within bf16-operand distance of the unpatched
    reference model's at every step, before and after the flush, and greedy tokens agree."""
    torch.manual_seed(7)
    cfg = tiny_config(ref, cache_dtype="hadamard_int4", cache_recent_tokens=64, cache_chunk_tokens=64)
    model = ref.AsterLM(cfg).to(cuda).eval()
    ids = torch.randint(0, 96, (1, 96), device=cuda)
    steps = 40

    def run():
        out = []
        with torch.no_grad():
            cache = model.make_cache()
            logits = model(ids, cache=cache, use_cache=True).logits[:, -1]
            for _ in range(steps):
                out.append(logits.float().clone())
                tok = logits.argmax(dim=-1, keepdim=True)
                logits = model(tok, cache=cache, use_cache=True).logits[:, -1]
            layer = next(iter(cache.latent.values()))
        return torch.cat(out), layer

    want, ref_layer = run()
    with _Patched(ref):
        got, our_layer = run()
    assert type(our_layer).__module__ == "asterq.cache" and our_layer.cold_chunks > 0
    assert our_layer.length == ref_layer.length and our_layer.cold_length == ref_layer.cold_length
    err = (got - want).abs().max() / want.abs().max()
    assert float(err) < 2e-2, f"max logit error {float(err):.3e} of the logit range"
    assert torch.equal(got.argmax(dim=-1), want.argmax(dim=-1))

    # the reference's own generation loop (decode.py:95-129), greedy, on the patched model
    gen = ref.generation.decode
    config = gen.GenerationConfig(max_new_tokens=16, temperature=0.0, repetition_penalty=1.0)
    with _Patched(ref):
        patched_tokens = list(gen.generate_tokens(model, ids, config))
    reference_tokens = list(gen.generate_tokens(model, ids, config))
    assert patched_tokens == reference_tokens
