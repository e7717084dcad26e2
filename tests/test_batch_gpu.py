"""The device-built schedule (asterq_plan_batch), the in-place append (asterq_batch_append)
and the continuous-batching loop built on them (asterq.batch.PagedLatentBatch).

* The planner's tables for a ragged batch: the tile and unit tables equal the host planner's
  (asterq.plan) exactly; every query block's work items cover its visible tiles once, in
  order; slots, combine jobs and the workers table are consistent.
* Decoding on those tables gives the oracle's context latents (rel-L2 <= 1e-3, max-abs
  <= 2e-2, as every decode test) and agrees with decoding on the host-built schedule.
* A decode loop with appends, flushes and sequences leaving and joining: at every checked
  step each sequence's context latents match the oracle over its whole token history split
  as the loop's cache holds it, the hot pages hold the appended tokens bit-exactly and the
  cold pages the oracle's codes and scales; a captured step replays bit-identically to the
  eager one.
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


def _close(got, want, what):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    rel, mab = O.rel_l2(got, want), O.max_abs(got, want)
    assert rel <= REL_L2 and mab <= MAX_ABS, f"{what}: rel-L2 {rel:.3e} max-abs {mab:.3e}"


def _ragged(cuda, q_len, seed=3):
    """Lengths with partial last cold pages, an all-hot sequence, a tiny one, a long one."""
    from asterq.synth import make_workload

    lengths = [9000, 700, 40, 20000, 3333, 512, 1, 6100]
    hot = [2048, 700, 40, 2048, 1000, 512, 1, 1536]
    keep = set(range(len(lengths)))
    return make_workload("ragged", lengths, hot, q_len=q_len, seed=seed, device=cuda, keep_host=keep)


def _oracle(wl, i):
    h = wl.host[i]
    n, hot = wl.lengths[i], wl.hot[i]
    return O.decode_sequence(h["latent"].float().numpy(), h["rope"].float().numpy(), h["q_lat"].float().numpy(),
                             h["q_rope"].float().numpy(), n, hot, SCALE)


def _check_tables(planner, plan, n_workers):
    """Device tables vs the host plan of the same layouts."""
    c = planner.host_counts()
    assert c["status"] == 0
    nt, nu, ni = c["n_tiles"], c["n_units"], c["n_items"]
    tiles = planner.tiles[:nt].cpu().numpy()
    np.testing.assert_array_equal(tiles, plan.tiles)
    np.testing.assert_array_equal(planner.units[:nu].cpu().numpy(), plan.units)
    items = planner.items[:ni].cpu().numpy()
    workers = planner.workers.cpu().numpy()
    assert workers[0] == 0 and workers[n_workers] == ni and (np.diff(workers) >= 0).all()
    # each unit: its items cover the host plan's tile range of that unit, contiguously, once
    want = {}
    for it in plan.items:
        lo, hi = want.get(int(it[0]), (1 << 30, -1))
        want[int(it[0])] = (min(lo, int(it[2])), max(hi, int(it[3])))
    by_unit = {}
    for it in items:
        by_unit.setdefault(int(it[0]), []).append(it)
    assert sorted(by_unit) == list(range(nu))
    combine = planner.combine.cpu().numpy()
    unit_jobs = planner.unit_jobs[:nu].cpu().numpy()
    slots_seen = []
    for u, its in by_unit.items():
        its = sorted(its, key=lambda r: r[2])
        assert (its[0][2], its[-1][3]) == want[u], f"unit {u}"
        for a, b in zip(its[:-1], its[1:]):
            assert a[3] == b[2] and a[2] < a[3], f"unit {u}: pieces not contiguous"
        assert all((r[5], r[6]) == tuple(plan.units[u]) for r in its)
        if len(its) == 1:
            assert its[0][4] == -1 and unit_jobs[u] == -1
        else:
            slots = sorted(int(r[4]) for r in its)
            assert slots == list(range(slots[0], slots[0] + len(its)))
            slots_seen += slots
            if len(its) <= 16:
                job = unit_jobs[u]
                assert c["n_separate"] <= job < c["n_jobs"]
            else:
                assert unit_jobs[u] == -1
                job = next(j for j in range(c["n_separate"]) if combine[j][0] == slots[0])
            np.testing.assert_array_equal(combine[job], [slots[0], slots[0] + len(its), *plan.units[u]])
    assert len(set(slots_seen)) == len(slots_seen) == c["n_slots"]
    return c


@pytest.mark.parametrize("q_len", [1, 3])
def test_device_plan_matches_host_tables_and_the_oracle(cuda, q_len):
    from asterq.batch import DevicePlanner, tables_from_layouts
    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan

    wl = _ragged(cuda, q_len)
    tables = tables_from_layouts(wl.layouts, 512, cuda)
    for n_workers in (148, 19):
        planner = DevicePlanner(tables, wl.n_heads, 512, max_q_len=q_len, n_workers=n_workers)
        planner.plan()
        out = torch.full((wl.total_q, wl.n_heads, 512), float("nan"), device=cuda)
        planner.decode(wl.pools, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
        planner.raise_if_failed()
        c = _check_tables(planner, build_plan(wl.layouts, wl.n_heads, n_sms=n_workers), n_workers)
        assert c["n_items"] > c["n_units"]  # the long sequences were cut
        got = out.cpu().numpy()
        host_out = latent_decode(wl.pools, DeviceDecodePlan(build_plan(wl.layouts, wl.n_heads), cuda), wl.q_lat,
                                 wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SCALE,
                                 out_dtype=torch.float32).cpu().numpy()
        # different cut points: each piece rounds p relative to its own running max (fp16 p x scale
        # operands), so the two schedules differ by ~1e-5, far inside the oracle tolerance
        assert O.rel_l2(got, host_out) <= 1e-4
        for i in range(len(wl.lengths)):
            rows = slice(i * q_len, (i + 1) * q_len)
            _close(got[rows], _oracle(wl, i), f"seq {i} (W={n_workers}, q_len {q_len})")


def test_device_plan_one_long_sequence_uses_the_combine_launch(cuda):
    """One 60k-token sequence over 148 workers: its single block is cut into more than 16
    pieces, so its merge goes to the combine launch (jobs [0, counts[6]))."""
    from asterq.batch import DevicePlanner, tables_from_layouts
    from asterq.synth import make_workload

    wl = make_workload("long", [60000], [2048], q_len=1, seed=5, device=cuda, keep_host={0})
    planner = DevicePlanner(tables_from_layouts(wl.layouts, 512, cuda), wl.n_heads, 512, n_workers=148)
    planner.plan()
    out = torch.empty(1, wl.n_heads, 512, device=cuda)
    planner.decode(wl.pools, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
    planner.raise_if_failed()
    c = planner.host_counts()
    assert c["n_items"] > 16 and c["n_separate"] == 1
    _close(out.cpu().numpy(), _oracle(wl, 0), "60k tokens")


def test_empty_slots_and_capacity_overflow(cuda):
    """Slots with q_len 0 plan nothing and their output rows stay untouched; a plan that does
    not fit its buffers reports status 1, plans nothing, and the decode then writes nothing."""
    from asterq import _lib
    from asterq.batch import DevicePlanner, tables_from_layouts

    wl = _ragged(cuda, 1)
    tables = tables_from_layouts(wl.layouts, 512, cuda)
    tables.host["q_len"][[1, 4]] = 0
    tables.upload()
    planner = DevicePlanner(tables, wl.n_heads, 512)
    planner.plan()
    out = torch.full((wl.total_q, wl.n_heads, 512), 7.0, device=cuda)
    planner.decode(wl.pools, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
    planner.raise_if_failed()
    got = out.cpu().numpy()
    assert (got[[1, 4]] == 7.0).all()
    for i in (0, 2, 3, 5, 6, 7):
        _close(got[i : i + 1], _oracle(wl, i), f"seq {i} beside empty slots")

    b = _lib.PlanBuffers.from_buffer_copy(planner.buffers)
    b.cap_tiles = 5
    _lib.check(_lib.load().asterq_plan_batch(ctypes.byref(planner.desc), ctypes.byref(b), _lib.stream_handle(cuda)))
    counts = planner.counts.cpu().numpy()
    assert counts[5] == 1 and counts[2] == 0
    assert (planner.workers.cpu().numpy() == 0).all()
    out.fill_(7.0)
    planner.decode(wl.pools, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SCALE)
    torch.cuda.synchronize()
    assert (out.cpu().numpy() == 7.0).all()
    with pytest.raises(RuntimeError, match="capacities"):
        planner.raise_if_failed()


def test_append_without_a_page_fails_that_sequence_only(cuda):
    from asterq import _lib
    from asterq.batch import PagedLatentBatch

    batch = PagedLatentBatch(16, max_seqs=2, q_len=1, page_tokens=128, recent_tokens=128, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(1)
    for n in (128, 50):  # slot 0 ends exactly on a page boundary
        batch.add_sequence(torch.randn(n, 512, generator=g, device=cuda).bfloat16(),
                           torch.randn(n, 64, generator=g, device=cuda).bfloat16())
    h = batch.tables.host
    page = int(h["hot_pages"][0, 1])
    h["hot_pages"][0, 1] = -1  # the page position 128 needs
    batch.tables.upload()
    new_lat = torch.randn(2, 512, generator=g, device=cuda).bfloat16()
    new_rope = torch.randn(2, 64, generator=g, device=cuda).bfloat16()
    d = batch.planner.desc
    _lib.check(_lib.load().asterq_batch_append(
        ctypes.byref(d), batch.tables.dev["hot_tokens"].data_ptr(), new_lat.data_ptr(), new_rope.data_ptr(), 2,
        batch.pools.hot_latent.data_ptr(), batch.pools.hot_rope.data_ptr(), int(batch.pools.hot_latent.shape[0]),
        batch.append_status.data_ptr(), _lib.stream_handle(cuda)))
    torch.cuda.synchronize()
    assert batch.tables.dev["hot_tokens"].cpu().tolist() == [128, 51]
    assert int(batch.append_status.item()) == 1
    p1 = int(h["hot_pages"][1, 0])
    assert torch.equal(batch.pools.hot_latent[p1, 50], new_lat[1]) and torch.equal(batch.pools.hot_rope[p1, 50], new_rope[1])
    assert page >= 0


class _History:
    """Every slot's token history (CPU bf16) and its step queries, to rebuild the oracle."""

    def __init__(self):
        self.lat, self.rope = {}, {}

    def start(self, slot, lat, rope):
        self.lat[slot], self.rope[slot] = [lat.cpu()], [rope.cpu()]

    def extend(self, slot, lat, rope):
        self.lat[slot].append(lat.cpu())
        self.rope[slot].append(rope.cpu())

    def tokens(self, slot):
        return torch.cat(self.lat[slot]).float().numpy(), torch.cat(self.rope[slot]).float().numpy()


@pytest.mark.parametrize("q_len,scheme,qrope", [(1, "hadamard_int4", False), (3, "hadamard_int4", False),
                                                (1, "int8", False), (3, "float8", False), (1, "hadamard_int4", True),
                                                (1, "int8", True), (1, "float8", True)])
def test_decode_loop_with_flushes_and_turnover_matches_the_oracle(cuda, q_len, scheme, qrope):
    """The serving loop with flushes and a sequence replaced mid-run, for INT4 pages and for the
    one-byte schemes (int8, float8: 64-token cold tiles planned on the GPU), with bf16 or
    quantized cold RoPE keys."""
    from asterq.batch import PagedLatentBatch

    P, recent = 128, 64  # a page is flushed whenever a hot window passes 192 tokens
    batch = PagedLatentBatch(16, max_seqs=5, q_len=q_len, page_tokens=P, recent_tokens=recent,
                             max_cold_pages=40, cache_dtype=scheme, quantize_rope=qrope, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(11 + q_len)
    hist = _History()

    def admit(n):
        lat = torch.randn(n, 512, generator=g, device=cuda)
        lat[:, :5] *= 20.0
        lat, rope = lat.bfloat16(), torch.randn(n, 64, generator=g, device=cuda).bfloat16()
        slot = batch.add_sequence(lat, rope)
        hist.start(slot, lat, rope)
        return slot

    for n in (1, 100, 300, 777, 1500):
        admit(n)
    rows = 5 * q_len
    steps = 140 if q_len == 1 else 60
    checked = 0
    for step in range(steps):
        if step == 45:
            batch.remove_sequence(2)
            hist.lat.pop(2)
            admit(260)  # takes the freed slot
        q_lat = torch.randn(rows, 16, 512, generator=g, device=cuda).bfloat16()
        q_rope = torch.randn(rows, 16, 64, generator=g, device=cuda).bfloat16()
        new_lat = torch.randn(rows, 512, generator=g, device=cuda).bfloat16()
        new_rope = torch.randn(rows, 64, generator=g, device=cuda).bfloat16()
        # lengths and hot windows as the cache holds them before this step
        before = {s: (batch.length(s), batch.hot_length(s)) for s in batch.active()}
        out = batch.step(q_lat, q_rope, new_lat, new_rope, torch.empty(rows, 16, 512, device=cuda))
        if step % 23 == 0 or step == steps - 1:
            got = out.cpu().numpy()
            for s, (n, hot) in before.items():
                lat, rope = hist.tokens(s)
                r = slice(s * q_len, (s + 1) * q_len)
                lat = np.concatenate([lat, new_lat[r].float().cpu().numpy()])
                rope = np.concatenate([rope, new_rope[r].float().cpu().numpy()])
                want = O.decode_sequence(lat, rope, q_lat[r].float().cpu().numpy(), q_rope[r].float().cpu().numpy(),
                                         n, hot, SCALE, chunk=P, scheme=scheme, quantize_rope=qrope)
                _close(got[r], want, f"step {step} slot {s} (n {n}, hot {hot})")
                checked += 1
        for s in before:
            r = slice(s * q_len, (s + 1) * q_len)
            hist.extend(s, new_lat[r], new_rope[r])
    batch.raise_if_failed()
    assert checked >= 20 and batch.flushes >= 4

    # the cache's pages hold exactly the history: hot tokens bit-exact, cold codes = the oracle's
    h = batch.tables.host
    for s in batch.active():
        lat, rope = hist.tokens(s)
        n_cold = int(h["n_cold"][s])
        cold = int(h["cold_tokens"][s, :n_cold].sum())
        assert cold + int(h["hot_tokens"][s]) == lat.shape[0] == batch.length(s)
        hot_pages = [int(p) for p in h["hot_pages"][s] if p >= 0]
        hot = torch.cat([batch.pools.hot_latent[p] for p in hot_pages])[: h["hot_tokens"][s]].float().cpu().numpy()
        np.testing.assert_array_equal(hot, lat[cold:])
        if n_cold:
            pages = [int(p) for p in h["cold_pages"][s, :n_cold]]
            codes = torch.cat([batch.pools.cold_codes[p] for p in pages]).cpu().numpy()
            q = O.quantize(lat[:cold], scheme, 64)
            np.testing.assert_array_equal(codes.view(np.uint8), q.data.reshape(cold, -1).view(np.uint8))
            if q.scale is not None:
                scales = torch.cat([batch.pools.cold_scales[p] for p in pages]).cpu().numpy()
                np.testing.assert_array_equal(scales.view(np.uint16), q.scale.reshape(cold, 8).view(np.uint16))


def test_captured_step_replays_like_the_eager_step(cuda):
    from asterq.batch import PagedLatentBatch

    def make():
        b = PagedLatentBatch(16, max_seqs=4, q_len=1, page_tokens=128, recent_tokens=128, device=cuda)
        g = torch.Generator(device=cuda).manual_seed(21)
        for n in (90, 250, 400, 1000):
            b.add_sequence(torch.randn(n, 512, generator=g, device=cuda).bfloat16(),
                           torch.randn(n, 64, generator=g, device=cuda).bfloat16())
        return b

    eager, graphed = make(), make()
    bufs = [torch.zeros(4, 16, 512, dtype=torch.bfloat16, device=cuda),
            torch.zeros(4, 16, 64, dtype=torch.bfloat16, device=cuda),
            torch.zeros(4, 512, dtype=torch.bfloat16, device=cuda),
            torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda),
            torch.zeros(4, 16, 512, dtype=torch.float32, device=cuda)]
    graph = graphed.capture(*bufs)
    g = torch.Generator(device=cuda).manual_seed(5)
    for step in range(70):  # crosses page boundaries and flushes
        inputs = [torch.randn(b.shape, generator=g, device=cuda).to(b.dtype) for b in bufs[:4]]
        want = eager.step(*inputs, torch.empty_like(bufs[4]))
        for b, x in zip(bufs[:4], inputs):
            b.copy_(x)
        got = graph.replay()
        assert torch.equal(got, want), f"step {step}"
    graphed.raise_if_failed()
    assert graphed.flushes == eager.flushes > 0
    for name in ("hot_tokens", "n_cold", "hot_pages", "cold_pages"):
        assert torch.equal(graphed.tables.dev[name], eager.tables.dev[name]), name


def test_mtp_verification_keeps_only_accepted_tokens(cuda):
    """Cache-aware verification (q_len 3: the last accepted token and two drafts): every step's
    three tokens attend to the cache and causally to each other (checked against the oracle over
    the accepted history), then a random prefix of them is accepted.  Flushes follow the accepted
    history only (the reference's rule, cache.py:167-177, replayed on it), and at the end the pages
    hold exactly that history: hot tokens bit-exact, cold codes and scales the oracle's."""
    from asterq.batch import PagedLatentBatch

    q_len, P, recent = 3, 128, 64
    threshold = recent + P
    batch = PagedLatentBatch(16, max_seqs=4, q_len=q_len, page_tokens=P, recent_tokens=recent,
                             max_cold_pages=24, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(17)
    rng = np.random.default_rng(17)
    hist = _History()
    sim = {}  # the reference's (cold, hot) lengths, replayed on the accepted tokens
    for n in (5, 150, 191, 900):
        lat = torch.randn(n, 512, generator=g, device=cuda)
        lat[:, :5] *= 20.0
        lat, rope = lat.bfloat16(), torch.randn(n, 64, generator=g, device=cuda).bfloat16()
        s = batch.add_sequence(lat, rope)
        hist.start(s, lat, rope)
        cold = 0
        while n - cold > threshold:
            cold += P
        sim[s] = [cold, n - cold]
    rows = 4 * q_len
    checked = 0
    for step in range(70):
        q_lat = torch.randn(rows, 16, 512, generator=g, device=cuda).bfloat16()
        q_rope = torch.randn(rows, 16, 64, generator=g, device=cuda).bfloat16()
        new_lat = torch.randn(rows, 512, generator=g, device=cuda).bfloat16()
        new_rope = torch.randn(rows, 64, generator=g, device=cuda).bfloat16()
        before = {s: (batch.length(s), batch.hot_length(s)) for s in batch.active()}
        for s, (n, hot) in before.items():
            assert (n, hot) == (sum(sim[s]), sim[s][1]), f"step {step} slot {s}"
        out = batch.verify(q_lat, q_rope, new_lat, new_rope, torch.empty(rows, 16, 512, device=cuda))
        with pytest.raises(RuntimeError):
            batch.step(q_lat, q_rope, new_lat, new_rope)
        if step % 9 == 0 or step == 69:
            got = out.cpu().numpy()
            for s, (n, hot) in before.items():
                lat, rope = hist.tokens(s)
                r = slice(s * q_len, (s + 1) * q_len)
                lat = np.concatenate([lat, new_lat[r].float().cpu().numpy()])
                rope = np.concatenate([rope, new_rope[r].float().cpu().numpy()])
                want = O.decode_sequence(lat, rope, q_lat[r].float().cpu().numpy(), q_rope[r].float().cpu().numpy(),
                                         n, hot, SCALE, chunk=P)
                _close(got[r], want, f"step {step} slot {s} (n {n}, hot {hot})")
                checked += 1
        keep = rng.integers(1, q_len + 1, size=4)
        batch.accept(keep)
        for s in before:
            k = int(keep[s])
            r = slice(s * q_len, s * q_len + k)
            hist.extend(s, new_lat[r], new_rope[r])
            sim[s][1] += k
            if sim[s][1] > threshold:
                sim[s][0] += P
                sim[s][1] -= P
    batch.raise_if_failed()
    assert checked >= 30 and batch.flushes >= 4
    h = batch.tables.host
    for s in batch.active():
        lat, rope = hist.tokens(s)
        n_cold = int(h["n_cold"][s])
        cold = int(h["cold_tokens"][s, :n_cold].sum())
        assert [cold, int(h["hot_tokens"][s])] == sim[s] and cold + sim[s][1] == lat.shape[0]
        assert batch.tables.dev["hot_tokens"][s].item() == sim[s][1]
        hot_pages = [int(p) for p in h["hot_pages"][s] if p >= 0]
        hot = torch.cat([batch.pools.hot_latent[p] for p in hot_pages])[: sim[s][1]].float().cpu().numpy()
        np.testing.assert_array_equal(hot, lat[cold:])
        if n_cold:
            pages = [int(p) for p in h["cold_pages"][s, :n_cold]]
            codes = torch.cat([batch.pools.cold_codes[p] for p in pages]).cpu().numpy()
            q = O.quantize(lat[:cold], "hadamard_int4", 64)
            np.testing.assert_array_equal(codes, q.data.reshape(cold, 256))


def test_planning_ahead_gives_the_same_steps(cuda):
    """With ``plan_ahead`` each step's schedule is built on a side stream while the step before it
    decodes, from a copy of the page tables taken after that step's bookkeeping.  Against a batch
    that plans in line with the same worker count (so the same schedule), every step's output is
    bit-identical, through flushes, a sequence leaving and one joining (which replan in line)."""
    from asterq.batch import PagedLatentBatch

    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    g0 = torch.Generator(device=cuda).manual_seed(33)
    prompts = [(torch.randn(n, 512, generator=g0, device=cuda).bfloat16(),
                torch.randn(n, 64, generator=g0, device=cuda).bfloat16()) for n in (60, 300, 1000, 2500)]

    def make(ahead):
        b = PagedLatentBatch(16, max_seqs=5, q_len=1, page_tokens=128, recent_tokens=64, max_cold_pages=40,
                             n_workers=sms - 1, plan_ahead=ahead, device=cuda)
        for lat, rope in prompts:
            b.add_sequence(lat, rope)
        return b

    ahead, inline = make(True), make(False)
    g = torch.Generator(device=cuda).manual_seed(34)
    for step in range(150):  # every hot window passes recent + page tokens at least once
        if step == 50:
            for b in (ahead, inline):
                b.remove_sequence(1)
        if step == 90:
            for b in (ahead, inline):
                b.add_sequence(*prompts[2])
        inputs = [torch.randn(5, 16, 512, generator=g, device=cuda).bfloat16(),
                  torch.randn(5, 16, 64, generator=g, device=cuda).bfloat16(),
                  torch.randn(5, 512, generator=g, device=cuda).bfloat16(),
                  torch.randn(5, 64, generator=g, device=cuda).bfloat16()]
        got = ahead.step(*inputs, torch.empty(5, 16, 512, device=cuda))
        want = inline.step(*inputs, torch.empty(5, 16, 512, device=cuda))
        for s in inline.active():
            assert torch.equal(got[s], want[s]), f"step {step} slot {s}"
    ahead.raise_if_failed()
    inline.raise_if_failed()
    assert ahead.flushes == inline.flushes > 0
    for name in ("hot_tokens", "n_cold", "hot_pages", "cold_pages", "cold_tokens"):
        assert torch.equal(ahead.tables.dev[name], inline.tables.dev[name]), name


def test_sliding_window_drops_whole_pages_and_decodes_the_kept_tokens(cuda):
    """A batch with a window of 600 tokens and 10 sink tokens: once a sequence is longer than the
    window plus a page of slack, the cold pages between its sink and its recent tokens are
    released (no re-quantization).  Every kept cold page still holds the chunk of the history it
    was flushed from, the kept chunks are the sink pages plus the newest ones, and each checked
    step matches the oracle over exactly the kept tokens."""
    from asterq.batch import PagedLatentBatch

    P, recent, W, sink = 128, 64, 600, 10
    batch = PagedLatentBatch(16, max_seqs=3, q_len=1, page_tokens=P, recent_tokens=recent, max_cold_pages=40,
                             window_size=W, sink_tokens=sink, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(23)
    hist = _History()
    chunk_of = {}  # live cold page id -> index of the history chunk it holds
    flushed = {}
    for n in (100, 900, 2000):
        lat = torch.randn(n, 512, generator=g, device=cuda)
        lat[:, :5] *= 20.0
        lat, rope = lat.bfloat16(), torch.randn(n, 64, generator=g, device=cuda).bfloat16()
        s = batch.add_sequence(lat, rope)
        hist.start(s, lat, rope)
        h = batch.tables.host
        flushed[s] = int(h["n_cold"][s])
        for j in range(flushed[s]):
            chunk_of[int(h["cold_pages"][s, j])] = j

    def kept_tokens(s):
        h = batch.tables.host
        lat, rope = hist.tokens(s)
        chunks = [chunk_of[int(p)] for p in h["cold_pages"][s, : h["n_cold"][s]]]
        hot = int(h["hot_tokens"][s])
        sel = np.concatenate([np.arange(c * P, (c + 1) * P) for c in chunks] + [np.arange(lat.shape[0] - hot, lat.shape[0])])
        return lat[sel], rope[sel], chunks, hot

    checked = 0
    for step in range(160):
        q_lat = torch.randn(3, 16, 512, generator=g, device=cuda).bfloat16()
        q_rope = torch.randn(3, 16, 64, generator=g, device=cuda).bfloat16()
        new_lat = torch.randn(3, 512, generator=g, device=cuda).bfloat16()
        new_rope = torch.randn(3, 64, generator=g, device=cuda).bfloat16()
        before = {s: kept_tokens(s) for s in batch.active()}
        out = batch.step(q_lat, q_rope, new_lat, new_rope, torch.empty(3, 16, 512, device=cuda))
        if step % 31 == 0 or step == 159:
            got = out.cpu().numpy()
            for s, (klat, krope, _, hot) in before.items():
                lat = np.concatenate([klat, new_lat[s : s + 1].float().cpu().numpy()])
                rope = np.concatenate([krope, new_rope[s : s + 1].float().cpu().numpy()])
                want = O.decode_sequence(lat, rope, q_lat[s : s + 1].float().cpu().numpy(),
                                         q_rope[s : s + 1].float().cpu().numpy(), klat.shape[0], hot, SCALE, chunk=P)
                _close(got[s : s + 1], want, f"step {step} slot {s}")
                checked += 1
        for s in before:
            hist.extend(s, new_lat[s : s + 1], new_rope[s : s + 1])
        h = batch.tables.host
        live_all = {int(p) for s in before for p in h["cold_pages"][s, : h["n_cold"][s]]}
        for p in [p for p in chunk_of if p not in live_all]:  # released by a trim (ids are reused later)
            del chunk_of[p]
        for s in before:  # a page flushed this step holds the next chunk of the history
            n_cold = int(h["n_cold"][s])
            for p in [int(p) for p in h["cold_pages"][s, :n_cold]]:
                if p not in chunk_of:
                    chunk_of[p] = flushed[s]
                    flushed[s] += 1
    batch.raise_if_failed()
    assert checked >= 15 and batch.pages_trimmed > 0
    for s in batch.active():
        _, _, chunks, hot = kept_tokens(s)
        n_sink = -(-min(sink, W) // P)
        assert chunks[:n_sink] == list(range(n_sink)), chunks
        rest = chunks[n_sink:]
        assert rest == list(range(flushed[s] - len(rest), flushed[s])), chunks  # the newest chunks
        assert batch.length(s) <= W + P + 2 * P
        # the kept pages hold their chunks' codes (flushed once, never re-quantized)
        lat, _ = hist.tokens(s)
        pages = [int(p) for p in batch.tables.host["cold_pages"][s, : len(chunks)]]
        for p, c in zip(pages, chunks):
            q = O.quantize(lat[c * P : (c + 1) * P], "hadamard_int4", 64)
            np.testing.assert_array_equal(batch.pools.cold_codes[p].cpu().numpy(), q.data.reshape(P, 256))
