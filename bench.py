"""Decode-attention benchmark (one JSON line on rank 0).

Workload: BASELINE config 3, ragged continuous-batching decode -- one batch of
64 sequences with seeded context lengths U[1024, 32768], the newest
min(len, 2048) tokens hot BF16, the rest INT4 chunks of 512, 16 heads, latent
512 + RoPE 64, q_len 1.  With N GPUs the batch is split longest-first by step
bytes (asterq.sharding): every rank decodes its own sequences, no collective
(strong scaling: the whole job is always the same 64 sequences).

  value  device-timed whole-job seq-steps/s: 64 sequences / the max over ranks
         of the per-step decode time (CUDA events around each step's launches;
         a 256 MB write flushes L2 between steps, outside the events)
  e2e    the same metric through the serving API (asterq.batch.PagedLatentBatch):
         every step copies its queries and new tokens from pinned host memory,
         plans on the GPU, decodes, appends the new tokens (the cache grows one
         token per sequence per step, flushing pages as they fill) and copies the
         context latents back
  roofline  achieved HBM GB/s of rank 0's decode kernel = algorithmic bytes per
         launch / its CUDA-event duration, against MEASURED_PEAKS.json
  cpu_baseline  the reference's own decode (LatentAttention._absorbed_decode of
         the unmodified AsterLM package installed under baseline/_ref) on the
         host cores, over 8 of the same 64 sequences, plus a one-thread figure

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "asterlm-frontier_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] if (ROOT / "BASELINE.json").exists() else \
    "decode-attn seq-steps/s per GPU and % of HBM peak, 1/2/4/8 B200 vs host CPU"
UNIT = "seq-steps/s"
SOFTMAX_SCALE = 1.0 / math.sqrt(512 + 64)
WORKLOAD = ("C3 ragged continuous-batching decode: one batch of 64 seqs, ctx U[1024,32768] (seed 0), hot min(len,2048) "
            "BF16 + INT4 chunks of 512, 16 heads, latent 512 + RoPE 64, q_len 1")


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks() -> tuple[float, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic() -> float | None:
    """dram bytes per decode launch from the committed ncu summary, if any."""
    f = ROOT / "profiles" / "decode_kernel_c3.md"
    if not f.exists():
        return None
    m = re.search(r"dram_bytes_per_launch\s*=\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region.

    NVML is polled from a thread every ~0.5 ms (read-only queries) from the
    warm-up through the end-to-end loop, so even a timed region of a few
    milliseconds yields samples.  Falls back to
    ``nvidia-smi -lms 100`` when NVML cannot be opened.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80))

    def __init__(self, gpu_index: int, torch_device=None):
        self.gpu = gpu_index
        self.torch_device = torch_device
        self.proc = None
        self.lines: list[str] = []
        self.samples: list[tuple[float, float, int]] = []  # (sm MHz, max sm MHz, reason bits)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        self._nvml = pynvml
        if self.torch_device is not None:
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(self.torch_device).uuid)
                return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                pass
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        idx = self.gpu
        if vis and all(x.strip().isdigit() for x in vis.split(",")):
            idx = int(vis.split(",")[self.gpu])
        return pynvml.nvmlDeviceGetHandleByIndex(idx)

    def _poll_nvml(self, h):
        nv = self._nvml
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((sm, mx, bits))
            except Exception:
                break
            time.sleep(0.0005)

    def __enter__(self):
        try:
            h = self._nvml_handle()
            self._t = threading.Thread(target=self._poll_nvml, args=(h,), daemon=True)
            self._t.start()
            return self
        except Exception:
            self._nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        if self.samples:
            for sm, mx, bits in self.samples:
                sms.append(sm)
                maxes.append(mx)
                for name, attr, default in self.REASONS:
                    if bits & int(getattr(self._nvml, attr, default) if self._nvml else default):
                        reasons.add(name)
            source = "nvml"
        else:
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for ln in self.lines:
                parts = [x.strip() for x in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    maxes.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
            source = "nvidia-smi"
        return {
            "sm_mhz": statistics.median(sms) if sms else None,
            "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": sorted(reasons),
            "samples": len(sms),
            "source": source,
        }


C3_SEQS = 64
C3_DATA_SEED = 1000
REF_SAMPLE = list(range(0, C3_SEQS, 8))  # the sequences the CPU baselines decode (every 8th)
REF_DIR = ROOT / "baseline" / "_ref"
L2_FLUSH_BYTES = 256 << 20


def c3_batch() -> tuple[list[int], list[int]]:
    from asterq.synth import c3_lengths

    lens = c3_lengths(0, C3_SEQS)
    return lens, [min(n, 2048) for n in lens]


def run_config(world: int) -> dict:
    """The workload description both arms print (the same for --impl asterq and reference)."""
    lens, hot = c3_batch()
    return {
        "workload": WORKLOAD,
        "seqs": C3_SEQS,
        "cached_tokens": int(sum(lens)),
        "q_len": 1,
        "n_heads": 16,
        "data_seed": C3_DATA_SEED,
        "parallelism": f"sequence sharding over {world} GPU(s): the one batch split longest-first by step bytes, "
                       "no collective",
        "l2": f"flushed between steps ({L2_FLUSH_BYTES >> 20} MB write, outside the per-step events)",
    }


# ---------------------------------------------------------------------------
# the reference's own CPU path (baseline/_ref: the unmodified AsterLM package)
# ---------------------------------------------------------------------------
def load_reference():
    """(modules, None) or (None, reason): LatentAttention, LatentLayerCache and quantize_tensor
    imported from the reference package installed under baseline/_ref."""
    if not (REF_DIR / "asterlm").is_dir():
        return None, "the reference is not installed under baseline/_ref"
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    try:
        from asterlm.cache import LatentLayerCache
        from asterlm.layers.latent_attention import LatentAttention
        from asterlm.quantization.kv import quantize_tensor
    except Exception as exc:  # a broken install is reported, not hidden
        return None, f"importing the reference failed: {exc!r}"
    import types

    return types.SimpleNamespace(LatentLayerCache=LatentLayerCache, LatentAttention=LatentAttention,
                                 quantize_tensor=quantize_tensor), None


def reference_cases(ref, host: dict, lengths: list[int], hot: list[int]) -> list:
    """One (attention module, decode arguments) per sampled sequence, in the reference's production
    dtype (bf16): the cache is the reference's own LatentLayerCache holding the C3 split (newest
    min(len, 2048) tokens hot, older tokens in 512-token chunks encoded by the reference quantizer,
    the newest chunk possibly partial), and the attention module is a duck-typed LatentAttention
    with identity absorption (head_dim = latent_rank = 512), as the golden fixtures use."""
    import types

    import torch

    def linear():
        m = torch.nn.Linear(512, 16 * 512, bias=False)
        m.weight.data = torch.eye(512).repeat(16, 1).to(torch.bfloat16)
        return m

    attn = types.SimpleNamespace(n_heads=16, head_dim=512, latent_rank=512, rope_dim=64, logit_softcap=None,
                                 training=False, dropout_p=0.0, k_up=linear(), v_up=linear())
    cases = []
    for i, h in sorted(host.items()):
        n, hn = lengths[i], hot[i]
        lat, rope = h["latent"], h["rope"]
        cache = ref.LatentLayerCache(cache_dtype="hadamard_int4", group_size=64, recent_tokens=hn, chunk_tokens=512)
        cold = n - hn
        for s0 in range(0, cold, 512):
            e0 = min(cold, s0 + 512)
            cache.cold_latent.append(ref.quantize_tensor(lat[None, s0:e0].contiguous(), "hadamard_int4", group_size=64))
            cache.cold_rope.append(rope[None, s0:e0].contiguous())
        cache.latent = lat[None, cold:n].contiguous()
        cache.rope_key = rope[None, cold:n].contiguous()
        args = (h["q_lat"][None], h["q_rope"][None], lat[None, n:], rope[None, n:], cache)
        cases.append((attn, args, n))
    return cases


def reference_rate(ref, cases, threads: int, budget_s: float, min_rounds: int = 1):
    """seq-steps/s of the reference decode (LatentAttention._absorbed_decode) on `threads` host
    threads: whole rounds over the sampled sequences until `budget_s` is spent."""
    import torch

    old = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        done, t0 = 0, time.perf_counter()
        rounds = 0
        with torch.inference_mode():
            while rounds < min_rounds or time.perf_counter() - t0 < budget_s:
                for attn, args, _ in cases:
                    ref.LatentAttention._absorbed_decode(attn, *args)
                    done += 1
                rounds += 1
        dt = time.perf_counter() - t0
    finally:
        torch.set_num_threads(old)
    return done / dt, done, dt


def reference_host_sample(dev):
    """CPU copies of the sampled C3 sequences, drawn exactly as the GPU arm draws its batch
    (on the GPU's generator when there is one)."""
    import torch

    from asterq.synth import host_sequences

    lens, _ = c3_batch()
    gen_dev = dev if (dev is not None and torch.cuda.is_available()) else "cpu"
    return host_sequences(lens, REF_SAMPLE, seed=C3_DATA_SEED, device=gen_dev), str(gen_dev)


def cpu_baseline_block(ref, host, lengths, hot, budget_s: float, one_thread_s: float) -> dict:
    cores = host_cores()
    cases = reference_cases(ref, host, lengths, hot)
    rate, done, dt = reference_rate(ref, cases, cores, budget_s)
    rate1, done1, dt1 = reference_rate(ref, cases[:2], 1, one_thread_s)
    toks = sum(n for _, _, n in cases)
    return {
        "value": rate, "unit": UNIT, "cores": cores, "kind": "reference",
        "sample": (f"{len(cases)} of the 64 C3 sequences (every 8th, {toks} cached tokens), {done} decodes in "
                   f"{dt:.1f} s by LatentAttention._absorbed_decode of the unmodified reference (baseline/_ref), "
                   "bf16 cache built by its own quantizer"),
        "one_thread": {"value": rate1, "unit": UNIT, "cores": 1,
                       "sample": f"sequences {REF_SAMPLE[:2]}, {done1} decodes in {dt1:.1f} s"},
    }


def run_reference_arm(args) -> None:
    """--impl reference: the reference's own CPU decode path (baseline/_ref) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    ref, why = load_reference()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    import torch

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    host, gen_dev = reference_host_sample(dev)
    lens, hot = c3_batch()
    cases = reference_cases(ref, host, lens, hot)
    cores = host_cores()
    torch.set_num_threads(cores)
    with torch.inference_mode():
        for _ in range(max(0, args.warmup)):
            for attn, a, _ in cases:
                ref.LatentAttention._absorbed_decode(attn, *a)
    # one step = one decode of each sampled sequence (all host threads)
    steps = max(1, args.steps)
    t0 = time.perf_counter()
    with torch.inference_mode():
        for _ in range(steps):
            for attn, a, _ in cases:
                ref.LatentAttention._absorbed_decode(attn, *a)
    elapsed = time.perf_counter() - t0
    value = steps * len(cases) / elapsed
    rate1, done1, dt1 = reference_rate(ref, cases[:2], 1, 4.0)
    sample = (f"{len(cases)} of the 64 C3 sequences (every 8th, {sum(n for _, _, n in cases)} cached tokens, drawn on "
              f"{gen_dev}); each step decodes each of them once with LatentAttention._absorbed_decode of the "
              "unmodified reference (baseline/_ref), bf16 cache built by its own quantizer")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": run_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference", "sample": sample,
                         "one_thread": {"value": rate1, "unit": UNIT, "cores": 1,
                                        "sample": f"sequences {REF_SAMPLE[:2]}, {done1} decodes in {dt1:.1f} s"}},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="asterq", choices=["asterq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--write-path-only", action="store_true",
                    help="time only the config-2 encode (3 + --steps launches per entry point) and print it")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.write_path_only:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"c2_write_path": write_path_rate(torch.device("cuda", 0), measured_peaks()[0],
                                                            iters=args.steps)}), flush=True)
        return

    import torch
    import torch.distributed as dist

    from asterq import _lib
    from asterq.decode import DeviceDecodePlan, latent_decode, make_params
    from asterq.plan import build_plan
    from asterq.sharding import shard_sequences
    from asterq.synth import make_shard_workload

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    args.warmup = max(args.warmup, 3)

    # the one C3 batch, split over the ranks (every rank computes the same split)
    lens, hot = c3_batch()
    shard = shard_sequences(lens, hot, world)[rank]
    keep = set(REF_SAMPLE) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    wl = make_shard_workload("C3", lens, hot, shard, q_len=1, n_heads=16, seed=C3_DATA_SEED, device=dev,
                             keep_host=keep)
    plan = build_plan(wl.layouts, wl.n_heads)
    dplan = DeviceDecodePlan(plan, dev)
    out = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    # decode-only and combine-only parameter blocks (same kernels as latent_decode)
    p_dec = make_params(wl.pools, dplan, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out,
                        n_heads=wl.n_heads, softmax_scale=SOFTMAX_SCALE)
    n_combine = p_dec.n_combine
    p_dec.n_combine = 0
    ws = dplan.workspace

    def step_device():
        _lib.check(lib.asterq_latent_decode(ctypes.byref(p_dec), sh))
        if n_combine:
            _lib.check(lib.asterq_splitkv_combine(ws.data_ptr(), plan.n_slots, dplan.combine.data_ptr(), n_combine,
                                                  512, out.data_ptr(), _lib.DTYPE_BF16, sh))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with ClockSampler(local, dev) as clocks:
        for _ in range(args.warmup):
            flush_buf.zero_()
            step_device()
        torch.cuda.synchronize()

        # ---- device-timed steps (events around each step's launches; the L2 flush between) ----
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
               torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        for e0, e1, e2 in ev:
            flush_buf.zero_()
            e0.record(stream)
            _lib.check(lib.asterq_latent_decode(ctypes.byref(p_dec), sh))
            e1.record(stream)
            if n_combine:  # blocks cut into more pieces than the decode kernel merges itself
                _lib.check(lib.asterq_splitkv_combine(ws.data_ptr(), plan.n_slots, dplan.combine.data_ptr(),
                                                      n_combine, 512, out.data_ptr(), _lib.DTYPE_BF16, sh))
            e2.record(stream)
        torch.cuda.synchronize()
        barrier()
        dec_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1, _ in ev)
        step_ms_local = statistics.mean(e0.elapsed_time(e2) for e0, _, e2 in ev)
        comb_ms = statistics.mean(e1.elapsed_time(e2) for _, e1, e2 in ev) if n_combine else 0.0
        ms_per_step = max_over_ranks(step_ms_local)
        value = C3_SEQS / (ms_per_step / 1e3)

        # ---- end-to-end through the public API with host buffers ----
        e2e = e2e_measure(wl, dev, stream, args, barrier, max_over_ranks)

    peak, peak_kind = measured_peaks()
    alg_bytes = wl.algorithmic_bytes()
    achieved = alg_bytes / (dec_ms / 1e3) / 1e9
    traffic = profiled_traffic() if world == 1 else None
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int4 codes + bf16/fp16 tensor-core operands, fp32 accumulate",
        "data": "synthetic",
        "config": run_config(world),
        "shard": {"rank0_seqs": len(shard), "rank0_cached_tokens": int(sum(wl.lengths)),
                  "rank0_work_items": int(plan.items.shape[0])},
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_kind": peak_kind,
            "traffic": traffic,
            "kernel": "asterq::dec::decode_kernel (timed with its query-preparation launch), rank 0",
            "algorithmic_bytes_per_launch": alg_bytes,
            "kernel_ms": dec_ms,
            "combine_ms": comb_ms,
        },
        "e2e": e2e,
        # per step: query preparation + decode_kernel, then combine_kernel when items were split
        # device-timed steps: query preparation + decode_kernel (+ combine_kernel when blocks were cut
        # into more pieces than the kernel merges); e2e steps: plan_batch, query preparation, decode,
        # append (+ combine), and any flush's encode
        "gpu_launches": args.steps * (3 if n_combine else 2) + args.steps * e2e["launches_per_step"]
        + e2e["flush_launches_timed"],
        "clocks": clocks.summary(),
    }

    if rank == 0 and world == 1 and not args.no_extras:
        line["extras"] = extras(dev, args)
    if world > 1 and not args.no_extras:
        ex = multi_gpu_extras(dev, rank, world, args, max_over_ranks, barrier)
        if rank == 0:
            line["extras"] = ex

    if keep:
        ref, why = load_reference()
        if ref is not None:
            line["cpu_baseline"] = cpu_baseline_block(ref, {g: wl.host[k] for k, g in enumerate(shard) if k in wl.host},
                                                      lens, hot, budget_s=10.0, one_thread_s=4.0)
        else:
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": host_cores(), "kind": "reference",
                                    "sample": f"not measured: {why}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def e2e_measure(wl, dev, stream, args, barrier, max_over_ranks) -> dict:
    """The same metric end to end through the serving API (``asterq.batch.PagedLatentBatch``),
    with the cache growing by one token per sequence every step, as in a decode loop
    (generate_tokens, decode.py:113-129, with LatentLayerCache.append, cache.py:186-201):

    each step copies its queries and new tokens from pinned host memory, plans the step on the
    GPU from the device page tables (``asterq_plan_batch``), decodes, appends the new tokens to
    the hot windows in place, flushes a sequence's oldest hot page into a cold page once its
    window passes recent + page tokens (cache.py:167-177), and copies the context latents back
    to pinned host memory.  The copies run on a second stream, double-buffered, so step k + 1's
    inputs and step k - 1's result move while step k decodes."""
    import torch

    from asterq.batch import PagedLatentBatch

    n, P = len(wl.lengths), wl.pools.page_tokens
    warm = max(args.warmup, 2)
    max_cold = max(len(lay.cold) for lay in wl.layouts) + (warm + args.steps) // P + 2
    # A large per-GPU batch plans each step on a side stream while the one before decodes (the
    # planner would otherwise add its time to the step); a small one replays the whole step
    # (plan, decode, append) as a CUDA graph, since there the host's per-step Python would
    # outlast the step's GPU time.
    use_graph = n <= 32
    batch = PagedLatentBatch(wl.n_heads, max_seqs=n, q_len=1, page_tokens=P, recent_tokens=2048 - P,
                             max_cold_pages=max_cold, plan_ahead=not use_graph, cache_dtype=wl.pools.cold_scheme,
                             quantize_rope=wl.pools.rope_quantized, device=dev)
    for lay in wl.layouts:  # slot s = shard position s: the step's row s
        batch.add_layout(wl.pools, lay.cold, lay.hot)
    inputs = (wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope)
    host_in = [t.cpu().pin_memory() for t in inputs]
    dev_in = [[torch.empty_like(t) for t in inputs] for _ in range(2)]
    out_shape = (wl.total_q, wl.n_heads, 512)
    dev_out = [torch.empty(out_shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    host_out = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out[0].numel() * host_out[0].element_size()
    copy_stream = torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    dec_done = [torch.cuda.Event() for _ in range(2)]
    host_s = []
    if use_graph:
        graphs = [batch.capture(*dev_in[b], dev_out[b], softmax_scale=SOFTMAX_SCALE) for b in range(2)]

        def one_step(b):
            graphs[b].replay()
    else:
        def one_step(b):
            batch.step(*dev_in[b], dev_out[b], softmax_scale=SOFTMAX_SCALE)

    def copy_in(b):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(dec_done[b])  # the step that last read buffer b is done
            for d, h in zip(dev_in[b], host_in):
                d.copy_(h, non_blocking=True)
            in_ready[b].record(copy_stream)

    def run(n_steps, start_ev=None, end_ev=None):
        for b in range(2):
            dec_done[b].record(stream)
        if start_ev is not None:
            start_ev.record(copy_stream)
        copy_in(0)
        for k in range(n_steps):
            b = k & 1
            stream.wait_event(in_ready[b])
            if k + 1 < n_steps:
                copy_in(1 - b)
            t0 = time.perf_counter()
            one_step(b)
            host_s.append(time.perf_counter() - t0)
            dec_done[b].record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(dec_done[b])
                host_out[b].copy_(dev_out[b], non_blocking=True)
        if end_ev is not None:
            end_ev.record(copy_stream)

    run(warm)
    torch.cuda.synchronize()
    batch.raise_if_failed()
    barrier()
    host_s.clear()
    flushes0, flush_launches0 = batch.flushes, batch.flush_launches
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(args.steps, e_s, e_e)
    torch.cuda.synchronize()
    batch.raise_if_failed()
    barrier()
    e2e_ms = max_over_ranks(e_s.elapsed_time(e_e)) / args.steps
    counts = batch.last_planner.host_counts()
    host_ms = statistics.mean(host_s) * 1e3
    how = ("the step (plan, decode, append) replayed as one CUDA graph (PagedLatentBatch.capture), host bookkeeping "
           "between replays" if use_graph else
           "each step's schedule planned on a side stream while the step before it decodes (one SM left to the planner)")
    res = {"value": C3_SEQS / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "ms_per_step": e2e_ms,
           "api": "asterq.batch.PagedLatentBatch." + ("capture + StepGraph.replay" if use_graph else "step"),
           "per_step": "H2D of queries and new tokens, plan on the GPU, decode, append (cache grows one token per "
                       "sequence), flushes as they fall due, D2H of the context latents; " + how,
           "host_ms_per_step": host_ms, "host_frac_of_step": host_ms / e2e_ms,
           "flushes_timed": batch.flushes - flushes0, "flush_launches_timed": batch.flush_launches - flush_launches0,
           "launches_per_step": 4 + (1 if counts["n_separate"] else 0),
           "per_rank": "h2d/d2h bytes are rank 0's"}
    if use_graph:
        del graphs
    del batch
    return res


def multi_gpu_extras(dev, rank, world, args, max_over_ranks, barrier) -> dict:
    """N > 1: weak scaling (every rank its own 64-sequence C3 batch), C5 sharded by sequence, and
    C4 context-parallel over the ranks."""
    import torch

    from asterq.decode import DeviceDecodePlan, latent_decode
    from asterq.plan import build_plan
    from asterq.sharding import shard_sequences
    from asterq.synth import c5_lengths, make_shard_workload, make_workload

    res = {}

    def timed_decode(wl, iters):
        plan = build_plan(wl.layouts, wl.n_heads)
        dp = DeviceDecodePlan(plan, dev)
        o = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)
        fn = lambda: latent_decode(wl.pools, dp, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope,  # noqa: E731
                                   softmax_scale=SOFTMAX_SCALE, out=o)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / iters)

    lens, hot = c3_batch()
    wl = make_workload("C3 weak", lens, hot, q_len=1, seed=C3_DATA_SEED + rank, device=dev)
    ms = timed_decode(wl, 20)
    res["c3_weak_scaling"] = {"seqs_per_gpu": C3_SEQS, "ms": ms, "seq_steps_per_s": world * C3_SEQS / ms * 1e3,
                              "scaling": "weak (every rank its own 64-sequence batch, seed 1000 + rank)"}
    del wl
    lens5 = c5_lengths(0, 256)
    hot5 = [min(n, 2048) for n in lens5]
    shard5 = shard_sequences(lens5, hot5, world, q_len=3)[rank]
    wl = make_shard_workload("C5", lens5, hot5, shard5, q_len=3, n_heads=16, seed=0, device=dev)
    ms = timed_decode(wl, 5)
    res["c5_sharded"] = {"seqs": 256, "q_len": 3, "ms": ms, "seq_steps_per_s": 256 / ms * 1e3,
                         "scaling": f"strong (256 sequences split over {world} GPUs)"}
    del wl
    torch.cuda.empty_cache()
    res["c4_context_parallel"] = context_parallel_extra(dev, rank, world, args, max_over_ranks, barrier)
    return res


def context_parallel_extra(dev, rank, world, args, max_over_ranks, barrier) -> dict:
    """C4 (one 131,072-token sequence) split by cold chunk over the ranks, partials gathered over NCCL."""
    import torch

    from asterq.context_parallel import ContextParallelDecoder
    from asterq.synth import c4_workload

    wl = c4_workload(dev, seed=4)
    dec = ContextParallelDecoder(wl.pools, wl.layouts[0], wl.n_heads, rank, world, dev)
    out = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)

    def step():
        dec.step(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SOFTMAX_SCALE)

    def timed(fn, iters=20):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / iters)

    ms_eager = timed(step)
    # the phases on their own (eager): decode + rank-local merge, the all-gather, the combine
    import torch.distributed as dist

    rec = dec.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, softmax_scale=SOFTMAX_SCALE)
    ms_partial = timed(lambda: dec.partial(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope,
                                           softmax_scale=SOFTMAX_SCALE))
    ms_gather = timed(lambda: dist.all_gather_into_tensor(dec.gathered, rec))
    ms_finish = timed(lambda: dec.finish(dec.gathered, out))
    # the same step as one CUDA graph per rank (decode, merge, NCCL all-gather, combine)
    graph = dec.capture(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SOFTMAX_SCALE)
    ms = timed(graph.replay)
    torch.cuda.synchronize()
    del graph  # released before the process group is destroyed
    # the records exchanged by peer stores into CUDA IPC mailboxes (no collective in the step)
    ex = dec.use_peer_exchange()
    try:
        ms_peer_eager = timed(lambda: dec.step_peer(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out,
                                                    softmax_scale=SOFTMAX_SCALE))
        graph = dec.capture_peer(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SOFTMAX_SCALE)
        ms_peer = timed(graph.replay)
        torch.cuda.synchronize()
        del graph
        ex.raise_if_failed()
    finally:
        ex.close()
    alg = wl.algorithmic_bytes()
    return {"seqs": 1, "cached_tokens": int(wl.lengths[0]), "ranks": world, "ms": ms, "ms_eager": ms_eager,
            "phases_ms_eager": {"decode_and_merge": ms_partial, "all_gather": ms_gather, "combine": ms_finish,
                                "rank0_pieces": int(dec.plan.n_slots)},
            "seq_steps_per_s": 1e3 / ms, "GB/s_total": alg / (ms / 1e3) / 1e9,
            "launch": "CUDA graph replay per step (ms_eager: the same step launched from Python)",
            "collective": "one all_gather_into_tensor of 32,896 B per rank per step (NCCL)",
            "peer_exchange": {"ms": ms_peer, "ms_eager": ms_peer_eager, "seq_steps_per_s": 1e3 / ms_peer,
                              "exchange": "merged records stored into every rank's CUDA IPC mailbox over NVLink, "
                                          "bounded wait on per-rank flags, combine from local memory"}}


def timed_ms(fn, iters: int) -> float:
    """Average device time of `fn` over `iters` calls after 3 warm-up calls (CUDA events, current stream)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def write_path_rate(dev, peak: float, iters: int = 20) -> dict:
    """Config 2: encode 64 x 4096 bf16 latent rows (hadamard_int4, groups of 64)."""
    import torch

    from asterq import _lib
    from asterq.kv import quantize_tensor
    from asterq.synth import outlier_channels

    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(64 * 4096, 512, generator=g, device=dev)
    x[:, outlier_channels(2).to(dev)] *= 20
    x = x.to(torch.bfloat16)
    ms_api = timed_ms(lambda: quantize_tensor(x, "hadamard_int4", group_size=64), iters)
    # the kernel alone: the C entry point into preallocated codes and scales
    lib = _lib.load()
    codes = torch.empty(64 * 4096, 256, dtype=torch.uint8, device=dev)
    scales = torch.empty(64 * 4096, 8, dtype=torch.float16, device=dev)
    stream = _lib.stream_handle(dev)
    ms = timed_ms(lambda: lib.asterq_quantize(x.data_ptr(), _lib.DTYPE_BF16, 64 * 4096, 512, 512,
                                              _lib.SCHEME_HADAMARD_INT4, 64, codes.data_ptr(), scales.data_ptr(),
                                              stream), iters)
    b = 64 * 4096 * (1024 + 256 + 16)
    res = {"tokens": 64 * 4096, "ms": ms, "ms_quantize_tensor": ms_api, "tokens_per_s": 64 * 4096 / ms * 1e3,
           "GB/s": b / ms / 1e6, "frac_hbm": b / ms / 1e6 / peak}
    del codes, scales, x
    return res


def extras(dev, args) -> dict:
    """Secondary single-GPU measurements: the write path (config 2) and configs 1, 4, 5."""
    import torch

    from asterq.decode import COLD_TILE_TOKENS, DeviceDecodePlan, capture_step, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import c1_inputs, c3_workload, c4_workload, c5_workload, PoolBuilder

    peak, _ = measured_peaks()
    res = {}
    timed = timed_ms
    res["c2_write_path"] = write_path_rate(dev, peak)

    def decode_rate(wl, name, iters):
        plan = build_plan(wl.layouts, wl.n_heads, cold_tile=COLD_TILE_TOKENS[wl.pools.cold_scheme])
        dp = DeviceDecodePlan(plan, dev)
        out = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)
        fn = lambda: latent_decode(wl.pools, dp, wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope,  # noqa: E731
                                   softmax_scale=SOFTMAX_SCALE, out=out)
        ms = timed(fn, iters)
        graph = capture_step(fn, dev)
        ms_graph = timed(graph.replay, iters)
        del graph
        b = wl.algorithmic_bytes()
        res[name] = {"seqs": len(wl.lengths), "q_len": wl.q_len, "ms": ms, "seq_steps_per_s": len(wl.lengths) / ms * 1e3,
                     "GB/s": b / ms / 1e6, "frac_hbm": b / ms / 1e6 / peak, "TFLOP/s": wl.flops() / ms / 1e9,
                     "ms_graph": ms_graph, "seq_steps_per_s_graph": len(wl.lengths) / ms_graph * 1e3}

    # chunked prefill (decode.py:105-108, prefill_chunk_size 2048): 2048 new tokens attending to an
    # 8k-token cache and causally to each other, through the decode kernel (one 16-row block per
    # new token); FLOPs counted over each token's visible keys
    T, ctx = 2048, 8192
    inp = c1_inputs(seed=0, ctx=ctx, q_len=T)
    bp = PoolBuilder([ctx], [1024], q_len=T, n_heads=16, device=dev)
    bp.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    decode_rate(bp.finish("prefill"), "prefill_2048_over_8k", 5)
    pf = res["prefill_2048_over_8k"]
    pf_flops = 2 * 16 * (512 + 64 + 512) * sum(ctx + t + 1 for t in range(T))
    pf.update({"TFLOP/s": pf_flops / pf["ms"] / 1e9, "tokens_per_s": T / pf["ms"] * 1e3,
               "note": "TFLOP/s over the causally visible keys; seq_steps_per_s counts chunks"})
    del bp, inp
    inp = c1_inputs(seed=0)
    b1 = PoolBuilder([8192], [1024], q_len=1, n_heads=16, device=dev)
    b1.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    decode_rate(b1.finish("C1"), "c1_single_sequence", 50)
    # C3 with quantize_rope=True: cold RoPE keys as INT4 codes (306 instead of 400 bytes a cold token)
    wl = c3_workload(dev, seed=1000, quantize_rope=True)
    decode_rate(wl, "c3_quantize_rope_1gpu", 20)
    del wl
    # C3 with cache_dtype="int8": 512 code bytes a cold token (656 B with scales and RoPE key)
    wl = c3_workload(dev, seed=1000, scheme="int8")
    decode_rate(wl, "c3_int8_1gpu", 20)
    # the same batch end to end through the serving loop (int8 flushes, 64-token tiles planned on
    # the GPU)
    e2e_args = argparse.Namespace(warmup=3, steps=20)
    res["c3_int8_1gpu"]["e2e"] = e2e_measure(wl, dev, torch.cuda.current_stream(dev), e2e_args, lambda: None,
                                             lambda x: x)
    del wl
    # C3 with cache_dtype="float8": 512 e4m3 bytes a cold token, no scales (640 B with the RoPE key)
    wl = c3_workload(dev, seed=1000, scheme="float8")
    decode_rate(wl, "c3_float8_1gpu", 20)
    del wl
    wl = c4_workload(dev)
    decode_rate(wl, "c4_long_context_1gpu", 30)
    del wl
    wl = c5_workload(dev)
    decode_rate(wl, "c5_mtp_verification_1gpu", 10)
    res["c5_mtp_verify_loop"] = mtp_verify_loop(wl, dev, iters=10)
    del wl
    torch.cuda.empty_cache()
    return res


def mtp_verify_loop(wl, dev, iters: int) -> dict:
    """C5 as a multi-token-prediction serving loop: the 256 sequences in a PagedLatentBatch with
    q_len 3 (the last accepted token and two drafts), each step ``verify`` (the three tokens
    attend to the cache and causally to each other, and are appended provisionally) then
    ``accept`` with a seeded random number of kept tokens per sequence (1-3), flushes after
    acceptance.  The inputs are already on the device; the host's accept bookkeeping and the
    device-side planning are inside the timed region."""
    import numpy as np
    import torch

    from asterq.batch import PagedLatentBatch

    n, P = len(wl.lengths), wl.pools.page_tokens
    max_cold = max(len(lay.cold) for lay in wl.layouts) + 4
    batch = PagedLatentBatch(wl.n_heads, max_seqs=n, q_len=wl.q_len, page_tokens=P, recent_tokens=2048 - P,
                             max_cold_pages=max_cold, device=dev)
    for lay in wl.layouts:
        batch.add_layout(wl.pools, lay.cold, lay.hot)
    out = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)
    rng = np.random.default_rng(5)
    keeps = [rng.integers(1, wl.q_len + 1, size=n) for _ in range(iters + 3)]

    def step(k):
        batch.verify(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SOFTMAX_SCALE)
        batch.accept(keeps[k])

    for k in range(3):
        step(k)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for k in range(iters):
        step(3 + k)
    e.record()
    torch.cuda.synchronize()
    batch.raise_if_failed()
    ms = s.elapsed_time(e) / iters
    accepted = float(np.mean([kp.mean() for kp in keeps[3:]]))
    res = {"seqs": n, "q_len": wl.q_len, "ms": ms, "seq_steps_per_s": n / ms * 1e3,
           "tokens_per_s": n * accepted / ms * 1e3, "mean_tokens_kept": accepted,
           "api": "asterq.batch.PagedLatentBatch.verify + accept"}
    del batch
    return res


if __name__ == "__main__":
    main()
