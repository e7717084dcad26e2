"""``asterq_latent_decode_noalloc`` against ``asterq_latent_decode``, through the C ABI.

The allocation-free entry point keeps its split-KV partial records in an array
inside the library instead of a caller-provided workspace.  It must give the
same context latents as the ordinary entry point (same tolerance as the other
decode tests: rel-L2 <= 1e-3 and max-abs <= 2e-2; the schedule and kernels are
the same, so the results are expected to be identical) on consecutive calls,
including a call whose schedule differs from the one before it (the shared
array still holds the previous call's records); the second call is also checked
against the CPU oracle directly.

Kept in a file of its own that pytest collects last, so that it runs both after
every other test and alone in a fresh process.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import hq4_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / math.sqrt(512 + 64)
MAX_ABS = 2e-2
REL_L2 = 1e-3
MAX_SLOTS = 256  # size of the library's built-in partial-record array


def _workload(seed, lengths, device):
    from asterq.synth import make_workload

    return make_workload("no-alloc", lengths, [min(n, 700) for n in lengths], q_len=1, seed=seed, device=device,
                         keep_host=set(range(len(lengths))))


def _oracle(wl):
    """The oracle's context latents for every sequence of the workload, [total_q, H, 512]."""
    rows = []
    for i, (n, hot) in enumerate(zip(wl.lengths, wl.hot)):
        h = wl.host[i]
        rows.append(O.decode_sequence(h["latent"].float().numpy(), h["rope"].float().numpy(),
                                      h["q_lat"].float().numpy(), h["q_rope"].float().numpy(), n, hot, SCALE))
    return np.concatenate(rows)


def _params(wl, plan_kw, out_dtype):
    from asterq.decode import DeviceDecodePlan, make_params
    from asterq.plan import build_plan

    plan = build_plan(wl.layouts, wl.n_heads, **plan_kw)
    dplan = DeviceDecodePlan(plan, wl.q_lat.device)
    out = torch.empty(wl.q_lat.shape[0], wl.n_heads, 512, dtype=out_dtype, device=wl.q_lat.device)
    p = make_params(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, n_heads=wl.n_heads,
                    softmax_scale=SCALE)
    return p, dplan, out


def _decode_both(wl, plan_kw, out_dtype=torch.float32):
    """(ordinary entry point's output, no-alloc entry point's output, n_slots, combine jobs the decode
    kernel runs itself with the counters that live in the built-in array)."""
    from asterq import _lib

    lib = _lib.load()
    stream = _lib.stream_handle(wl.q_lat.device)
    p, dplan, out_ref = _params(wl, plan_kw, out_dtype)
    _lib.check(lib.asterq_latent_decode(ctypes.byref(p), stream))
    out_na = torch.full_like(out_ref, float("nan"))
    p.out = out_na.data_ptr()
    p.workspace = None  # the no-alloc entry point ignores these
    p.workspace_bytes = 0
    _lib.check(lib.asterq_latent_decode_noalloc(ctypes.byref(p), stream))
    torch.cuda.synchronize()
    return (out_ref.float().cpu().numpy(), out_na.float().cpu().numpy(), int(p.n_slots),
            int(p.n_combine_total) - int(p.n_combine))


def _assert_same(got, want, what):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    rel, mab = O.rel_l2(got, want), O.max_abs(got, want)
    assert rel <= REL_L2 and mab <= MAX_ABS, f"{what}: rel-L2 {rel:.3e} max-abs {mab:.3e}"


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda):
    wl_a = _workload(11, [9000, 3000, 700, 40], cuda)
    wl_b = _workload(12, [5000, 12000], cuda)
    split = dict(n_sms=32, ctas_per_sm=2, waves=4)
    calls = [(wl_a, split, torch.float32), (wl_a, split, torch.float32), (wl_b, split, torch.bfloat16),
             (wl_a, dict(max_items_per_seq=1), torch.float32)]
    fused_calls = 0
    for i, (wl, kw, dt) in enumerate(calls):
        ref, got, n_slots, n_fused = _decode_both(wl, kw, dt)
        if kw is split:
            assert 0 < n_slots <= MAX_SLOTS, n_slots
        fused_calls += n_fused > 0
        _assert_same(got, ref, f"call {i} ({wl.lengths}, {dt})")
        if i == 1:  # a second call in a row: also against the oracle directly
            _assert_same(got, _oracle(wl), f"call {i} against the oracle")
    # the in-kernel merge (whose per-block counters sit in the built-in array, zeroed every call)
    # ran on consecutive calls
    assert fused_calls >= 2


def test_noalloc_rejects_schedules_beyond_its_array(cuda):
    from asterq import _lib

    lib = _lib.load()
    wl = _workload(13, [700], cuda)
    p, _, _ = _params(wl, dict(max_items_per_seq=1), torch.float32)
    p.n_slots = MAX_SLOTS + 1
    assert lib.asterq_latent_decode_noalloc(ctypes.byref(p), _lib.stream_handle(cuda)) == _lib.ASTERQ_ERR_WORKSPACE
    assert b"no-alloc" in lib.asterq_last_error()
    p.n_slots = 0
    p.n_units = MAX_SLOTS + 1  # the array also holds one prepared query block and one counter per 16-row block
    assert lib.asterq_latent_decode_noalloc(ctypes.byref(p), _lib.stream_handle(cuda)) == _lib.ASTERQ_ERR_WORKSPACE
    assert b"no-alloc" in lib.asterq_last_error()
