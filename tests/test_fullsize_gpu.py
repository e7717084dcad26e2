"""Parity at the BASELINE configurations' full sizes (GPU against the CPU oracle).

* C2: every one of the 64 x 4096 tokens' codes and scales bit-exact.
* C3: every one of the 64 sequences of the batch ``bench.py`` times (data seed 1000),
  float32 and bfloat16 outputs.
* C4: the 131,072-token sequence on one GPU, and split into 2, 4 and 8 context-parallel
  ranks (emulated in turn on one GPU, records combined rank-major).
* C5: all 32 sequences of one rank's shard of the 8-GPU split (q_len 3, causal).

Tolerance (north_star): rel-L2 <= 1e-3 and max-abs <= 2e-2 (float32 output against the
float32 oracle); bfloat16 output: rel-L2 <= 1e-3 and every element within
max(2e-2, one bf16 ulp) of the bfloat16-rounded oracle.  The oracle runs on the host
in a process pool started with ``spawn``.
"""
from __future__ import annotations

import math
import multiprocessing as mp
import os
from concurrent.futures import ProcessPoolExecutor

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)
MAX_ABS = 2e-2
REL_L2 = 1e-3


def assert_close(out: np.ndarray, ref: np.ndarray, what: str) -> None:
    rel, mab = O.rel_l2(out, ref), O.max_abs(out, ref)
    assert rel <= REL_L2 and mab <= MAX_ABS, f"{what}: rel-L2 {rel:.3e} max-abs {mab:.3e}"


def assert_close_bf16(out_bf16: np.ndarray, ref_fp32: np.ndarray, what: str) -> None:
    ref = O.round_bf16(ref_fp32)
    rel = O.rel_l2(out_bf16, ref)
    ax = np.maximum(np.abs(ref_fp32), np.float32(2.0 ** -126))
    ulp = np.exp2(np.floor(np.log2(ax)) - 7).astype(np.float32)
    worst = float(np.max(np.abs(out_bf16.astype(np.float64) - ref) - np.maximum(MAX_ABS, ulp)))
    assert rel <= REL_L2 and worst <= 0.0, f"{what}: rel-L2 {rel:.3e}, worst excess over bound {worst:.3e}"


def oracle_batch(host: dict, lengths, hot, scheme: str = "hadamard_int4", quantize_rope: bool = False) -> dict:
    """Oracle outputs of the sequences in ``host`` (position -> CPU bf16 tensors), in parallel."""
    jobs = {k: (h["latent"].float().numpy(), h["rope"].float().numpy(), h["q_lat"].float().numpy(),
                h["q_rope"].float().numpy(), lengths[k], hot[k], SCALE, 512, scheme, quantize_rope)
            for k, h in host.items()}
    workers = max(1, min(16, (os.cpu_count() or 2) // 2, len(jobs)))
    with ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")) as ex:
        futs = {k: ex.submit(O.decode_sequence, *args) for k, args in jobs.items()}
        return {k: f.result() for k, f in futs.items()}


def run_decode(wl, out_dtype):
    from asterq.decode import COLD_TILE_TOKENS, DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan

    plan = build_plan(wl.layouts, wl.n_heads, cold_tile=COLD_TILE_TOKENS[wl.pools.cold_scheme])
    dplan = DeviceDecodePlan(plan, wl.q_lat.device)
    out = latent_decode(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                        out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out


def test_c2_every_code_and_scale(cuda):
    """Config 2: 64 x 4096 bf16 latent tokens through the write path, all codes and scales."""
    from asterq.kv import quantize_tensor
    from asterq.synth import outlier_channels

    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(64 * 4096, 512, generator=g, device=cuda)
    x[:, outlier_channels(2).to(cuda)] *= 20
    x = x.to(torch.bfloat16)
    q = quantize_tensor(x, "hadamard_int4", group_size=64)
    codes, scales = q.data.cpu().numpy(), q.scale.reshape(-1, 8).cpu().numpy()
    xs = x.float().cpu().numpy()
    for r0 in range(0, xs.shape[0], 65536):
        ref = O.quantize(xs[r0:r0 + 65536], "hadamard_int4", 64)
        np.testing.assert_array_equal(codes[r0:r0 + 65536], ref.data)
        np.testing.assert_array_equal(scales[r0:r0 + 65536].view(np.uint16),
                                      ref.scale.reshape(-1, 8).view(np.uint16))


def test_c3_every_sequence_of_the_benched_batch(cuda):
    """Config 3: the 64-sequence batch bench.py times (lengths seed 0, data seed 1000)."""
    from asterq.synth import c3_lengths, make_shard_workload

    lens = c3_lengths(0, 64)
    hot = [min(n, 2048) for n in lens]
    wl = make_shard_workload("C3", lens, hot, list(range(64)), q_len=1, seed=1000, device=cuda,
                             keep_host=set(range(64)))
    out32 = run_decode(wl, torch.float32).cpu().numpy()
    out16 = run_decode(wl, torch.bfloat16).float().cpu().numpy()
    refs = oracle_batch(wl.host, wl.lengths, wl.hot)
    for i in range(64):
        assert_close(out32[i:i + 1], refs[i], f"C3 seq {i} (len {lens[i]}) fp32")
        assert_close_bf16(out16[i:i + 1], refs[i], f"C3 seq {i} bf16")


@pytest.mark.parametrize("scheme,qrope", [("int8", False), ("float8", False), ("hadamard_int4", True),
                                          ("int8", True)])
def test_c3_batch_other_cache_schemes(cuda, scheme, qrope):
    """The benched C3 batch (64 sequences, 948k cached tokens) stored with the other cache schemes
    the reference offers (int8, float8, quantized RoPE keys); every 4th sequence checked against
    the oracle (16 sequences from 1k to 32k tokens), fp32 output."""
    from asterq.synth import c3_lengths, make_shard_workload

    lens = c3_lengths(0, 64)
    hot = [min(n, 2048) for n in lens]
    keep = set(range(0, 64, 4))
    wl = make_shard_workload("C3", lens, hot, list(range(64)), q_len=1, seed=1000, device=cuda, keep_host=keep,
                             scheme=scheme, quantize_rope=qrope)
    out32 = run_decode(wl, torch.float32).cpu().numpy()
    refs = oracle_batch(wl.host, wl.lengths, wl.hot, scheme, qrope)
    for i in sorted(keep):
        assert_close(out32[i:i + 1], refs[i], f"C3 {scheme} qrope={qrope} seq {i} (len {lens[i]})")


def test_c4_full_length_one_gpu_and_context_parallel(cuda):
    """Config 4: 131,072 tokens (248 cold chunks + 4096 hot) on one GPU, then split over 2/4/8 ranks."""
    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import c4_workload

    wl = c4_workload(cuda, seed=0, keep_host={0})
    assert wl.lengths == [131072] and len(wl.layouts[0].cold) == 248
    ref = oracle_batch(wl.host, wl.lengths, wl.hot)[0]
    assert_close(run_decode(wl, torch.float32).cpu().numpy(), ref, "C4 one GPU")
    for world in (2, 4, 8):
        decs = [ContextParallelDecoder(wl.pools, wl.layouts[0], 16, r, world, cuda) for r in range(world)]
        recs = [d.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE).clone() for d in decs]
        out = torch.empty(1, 16, 512, dtype=torch.float32, device=cuda)
        decs[world // 2].finish(torch.cat(recs), out)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref, f"C4 over {world} ranks")


def test_c5_one_shard_of_eight(cuda):
    """Config 5: rank 0's 32 of the 256 sequences split over 8 GPUs, q_len 3 with the causal mask."""
    from asterq.sharding import shard_sequences
    from asterq.synth import c5_lengths, make_shard_workload

    lens = c5_lengths(0, 256)
    hot = [min(n, 2048) for n in lens]
    shard = shard_sequences(lens, hot, 8, q_len=3)[0]
    assert len(shard) == 32
    wl = make_shard_workload("C5 shard", lens, hot, shard, q_len=3, seed=0, device=cuda, keep_host=set(shard))
    out = run_decode(wl, torch.float32).cpu().numpy()
    refs = oracle_batch(wl.host, wl.lengths, wl.hot)
    for k in range(len(shard)):
        assert_close(out[3 * k:3 * k + 3], refs[k], f"C5 seq {shard[k]} (len {lens[shard[k]]})")
