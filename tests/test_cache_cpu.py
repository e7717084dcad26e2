"""Host-side behaviour of the drop-in cache that needs no GPU: argument checks and error types."""
from __future__ import annotations

import pytest
import torch


def test_unsupported_configurations_raise():
    from asterq.cache import LatentLayerCache

    with pytest.raises(NotImplementedError):
        LatentLayerCache("int2")
    with pytest.raises(NotImplementedError):
        LatentLayerCache("hadamard_int4", group_size=32)
    with pytest.raises(ValueError):
        LatentLayerCache("hadamard_int4", chunk_tokens=100)


def test_quantize_rope_is_accepted_for_every_kernel_scheme():
    """quantize_rope=True (cache.py:64, :160-164) is served: the integer schemes store codes, bfloat16
    never flushes, so its RoPE keys stay bf16 as in the reference."""
    from asterq.cache import LatentLayerCache

    for scheme in ("hadamard_int4", "int4", "int8", "float8", "bfloat16"):
        c = LatentLayerCache(scheme, quantize_rope=True, chunk_tokens=512)
        assert c.quantize_rope and c._rope_quantized == (scheme != "bfloat16")
        assert c.num_bytes == 0


def test_empty_cache_reports_nothing():
    from asterq.cache import LatentLayerCache

    c = LatentLayerCache("hadamard_int4", chunk_tokens=512)
    assert c.length == 0 and c.cold_length == 0 and c.num_bytes == 0
    assert c.latent is None and c.materialize_latent() is None
    assert list(c.iter_chunks(dtype=torch.float32, device=torch.device("cpu"))) == []


def test_cpu_tensors_are_rejected():
    from asterq.cache import LatentLayerCache

    c = LatentLayerCache("hadamard_int4", chunk_tokens=512)
    with pytest.raises(RuntimeError):
        c.append(torch.zeros(1, 4, 512), torch.zeros(1, 4, 64), None, 0)
    with pytest.raises(ValueError):
        c.append(torch.zeros(1, 4, 256), torch.zeros(1, 4, 64), None, 0)


def test_aster_cache_builds_layers_from_its_settings():
    from asterq.cache import AsterCache

    cache = AsterCache(cache_dtype="hadamard_int4", cache_recent_tokens=256, cache_chunk_tokens=512)
    layer = cache.latent_layer(3)
    assert layer is cache.latent_layer(3)
    assert (layer.cache_dtype, layer.recent_tokens, layer.chunk_tokens) == ("hadamard_int4", 256, 512)
    assert cache.num_bytes == 0
    cache.reset()
    assert not cache.latent


def test_trim_page_range_keeps_sink_and_recent_pages():
    """Whole-page window trim: pages holding the first min(sink, window) tokens and the newest
    pages that, with the hot window, hold window - sink tokens survive; the rest go."""
    from asterq.cache import trim_page_range

    P = 256
    # 10 full cold pages + 440 hot tokens, window 1500 with 4 sink tokens: page 0 holds the sink,
    # the hot window plus the 5 newest pages hold >= 1496 tokens, pages 1-4 are dropped
    assert trim_page_range(10, [P] * 10, 440, P, 1500, 4) == (1, 5)
    # no sink: only the recent side is kept
    assert trim_page_range(10, [P] * 10, 440, P, 1500, 0) == (0, 5)
    # a sink longer than the window is clipped to the window (recent = 0)
    assert trim_page_range(10, [P] * 10, 440, P, 700, 5000) == (3, 10)
    # nothing between sink and recent pages: no trim
    assert trim_page_range(3, [P] * 3, 440, P, 1500, 4) is None
    # partial cold pages count their own tokens
    assert trim_page_range(5, [100, 256, 256, 256, 30], 10, P, 300, 150) == (2, 3)
    assert trim_page_range(4, [100, 256, 256, 30], 10, P, 300, 150) is None
