"""Decode-attention benchmark (one JSON line on rank 0).

Workload (per GPU): BASELINE config 3, ragged continuous-batching decode --
64 sequences with seeded context lengths U[1024, 32768], the newest
min(len, 2048) tokens hot BF16, the rest INT4 chunks of 512, 16 heads, latent
512 + RoPE 64, q_len 1.  Sequences are sharded across GPUs: every rank owns its
own 64-sequence batch (weak scaling, no collective in the timed step).

  value  device-timed whole-job seq-steps/s (CUDA events, max over ranks),
         inputs resident in HBM (0.53 GB per GPU, larger than the 126 MB L2)
  e2e    the same metric through the public API (asterq.decode.latent_decode)
         with the step's query/new-token inputs copied from pinned host memory
         and the context latents copied back, every step
  roofline  achieved HBM GB/s of the decode kernel = algorithmic bytes per
         launch / its CUDA-event duration, against MEASURED_PEAKS.json
  cpu_baseline  the CPU oracle port on the host cores (bounded sample)

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
WORKLOAD = ("C3 ragged continuous-batching decode: 64 seqs/GPU, ctx U[1024,32768] (seed 0), hot min(len,2048) "
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

    NVML is polled from a thread every ~2 ms (read-only queries), so even a
    timed region of a few tens of milliseconds yields samples.  Falls back to
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
            time.sleep(0.002)

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


def build_workload(device, rank: int, n_seqs: int = 64, keep_host=None):
    from asterq.synth import c3_lengths, make_workload

    lens = c3_lengths(0, n_seqs)
    return make_workload("C3", lens, [min(n, 2048) for n in lens], q_len=1, seed=1000 + rank, device=device,
                         keep_host=keep_host)


def oracle_caches(host_seqs: dict, lengths, hot) -> list:
    """The sampled sequences' caches in the oracle's form (built once, outside any timing)."""
    from oracle import hq4_oracle as O

    caches = []
    for i, h in sorted(host_seqs.items()):
        lat = h["latent"].float().numpy()
        rope = h["rope"].float().numpy()
        n = lengths[i]
        caches.append((O.build_cache_split(lat[:n], rope[:n], hot[i], 512), h, lat[n:], rope[n:]))
    return caches


def cpu_oracle_rate(caches: list, budget_s: float = 12.0):
    """Oracle decode (numpy port of the reference path) on host cores over prebuilt caches; seq-steps/s."""
    from oracle import hq4_oracle as O

    done, t0 = 0, time.perf_counter()
    tokens = 0
    while True:
        for cache, h, nl, nr in caches:
            O.absorbed_decode(h["q_lat"].float().numpy(), h["q_rope"].float().numpy(), nl, nr, cache, SOFTMAX_SCALE)
            done += 1
            tokens += cache.length
            if time.perf_counter() - t0 > budget_s:
                break
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, tokens, dt


def run_reference_arm(args) -> None:
    """--impl reference: the CPU oracle port of the reference path, all host threads."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from asterq.synth import c3_lengths

    lens = c3_lengths(0, 64)
    hot = [min(n, 2048) for n in lens]
    # the sample: 8 sequences of the config-3 batch, generated on the CPU
    pick = list(range(0, 64, 8))
    host = {}
    g = torch.Generator().manual_seed(7)
    from asterq.synth import outlier_channels

    oc = outlier_channels(7)
    for i in pick:
        n = lens[i]
        lat = torch.randn(n + 1, 512, generator=g)
        lat[:, oc] *= 20
        host[i] = {"latent": lat.to(torch.bfloat16), "rope": torch.randn(n + 1, 64, generator=g).to(torch.bfloat16),
                   "q_lat": torch.randn(1, 16, 512, generator=g).to(torch.bfloat16),
                   "q_rope": torch.randn(1, 16, 64, generator=g).to(torch.bfloat16)}
    cores = host_cores()
    caches = oracle_caches(host, lens, hot)
    for _ in range(max(0, args.warmup)):
        cpu_oracle_rate(caches, budget_s=0.5)
    rates = []
    t0 = time.perf_counter()
    # each step is a bounded sample; the whole timed run stays near one minute
    step_budget = min(2.0, 60.0 / max(1, args.steps))
    for _ in range(max(1, args.steps)):
        r, _, _, _ = cpu_oracle_rate(caches, budget_s=step_budget)
        rates.append(r)
    elapsed = time.perf_counter() - t0
    value = statistics.median(rates)
    sample = f"{len(pick)} config-3 sequences (every 8th), each step = {step_budget:.2f} s of oracle decodes"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / max(1, args.steps) * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
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

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    args.warmup = max(args.warmup, 3)

    keep = set(range(0, 64, 16)) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    wl = build_workload(dev, rank, keep_host=keep)
    plan = build_plan(wl.layouts, wl.n_heads)
    dplan = DeviceDecodePlan(plan, dev)
    out = torch.empty(wl.total_q, wl.n_heads, 512, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

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

    for _ in range(args.warmup):
        step_device()
    torch.cuda.synchronize()

    # ---- device-timed steps ----
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local, dev) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for e0, e1, e2 in ev:
            e0.record(stream)
            _lib.check(lib.asterq_latent_decode(ctypes.byref(p_dec), sh))
            e1.record(stream)
            if n_combine:  # blocks cut into more pieces than the decode kernel merges itself
                _lib.check(lib.asterq_splitkv_combine(ws.data_ptr(), plan.n_slots, dplan.combine.data_ptr(),
                                                      n_combine, 512, out.data_ptr(), _lib.DTYPE_BF16, sh))
                e2.record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = max_over_ranks(t_start.elapsed_time(t_end))
    dec_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1, _ in ev)
    comb_ms = statistics.mean(e1.elapsed_time(e2) for _, e1, e2 in ev) if n_combine else 0.0
    ms_per_step = total_ms / args.steps
    n_seqs = len(wl.lengths)
    value = world * n_seqs / (ms_per_step / 1e3)

    # ---- end-to-end through the public API with host buffers ----
    # A serving loop's shape: every step copies its inputs from pinned host memory and
    # reads its result back; the copies run on a second stream, double-buffered, so
    # step k + 1's inputs and step k - 1's result move while step k decodes.
    host_in = [t.cpu().pin_memory() for t in (wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope)]
    dev_in = [[torch.empty_like(t) for t in (wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope)] for _ in range(2)]
    dev_out = [torch.empty_like(out) for _ in range(2)]
    host_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out[0].numel() * host_out[0].element_size()
    copy_stream = torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    dec_done = [torch.cuda.Event() for _ in range(2)]

    def copy_in(b):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(dec_done[b])  # the decode that last read buffer b is done
            for d, h in zip(dev_in[b], host_in):
                d.copy_(h, non_blocking=True)
            in_ready[b].record(copy_stream)

    def run_e2e(n_steps, start_ev=None, end_ev=None):
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
            latent_decode(wl.pools, dplan, *dev_in[b], softmax_scale=SOFTMAX_SCALE, out=dev_out[b])
            dec_done[b].record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(dec_done[b])
                host_out[b].copy_(dev_out[b], non_blocking=True)
        if end_ev is not None:
            end_ev.record(copy_stream)

    run_e2e(max(args.warmup, 2))
    torch.cuda.synchronize()
    barrier()
    e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run_e2e(args.steps, e_s, e_e)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e_s.elapsed_time(e_e)) / args.steps
    e2e_value = world * n_seqs / (e2e_ms / 1e3)

    peak, peak_kind = measured_peaks()
    alg_bytes = wl.algorithmic_bytes()
    achieved = alg_bytes / (dec_ms / 1e3) / 1e9
    traffic = profiled_traffic()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4 codes + bf16/fp16 tensor-core operands, fp32 accumulate",
        "data": "synthetic",
        "config": {
            "workload": WORKLOAD,
            "seqs_per_gpu": n_seqs,
            "cached_tokens_per_gpu": int(sum(wl.lengths)),
            "q_len": 1,
            "n_heads": wl.n_heads,
            "parallelism": f"sequence sharding x{world} (independent batches, no collective)",
            "l2": f"no flush: {alg_bytes / 1e9:.2f} GB read per step per GPU > 126 MB L2",
            "work_items": int(plan.items.shape[0]),
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_kind": peak_kind,
            "traffic": traffic,
            "kernel": "asterq::dec::decode_kernel (timed with its query-preparation launch)",
            "algorithmic_bytes_per_launch": alg_bytes,
            "kernel_ms": dec_ms,
            "combine_ms": comb_ms,
        },
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms},
        # per step: query preparation + decode_kernel, then combine_kernel when items were split
        "gpu_launches": args.steps * (3 if n_combine else 2),
        "clocks": clocks.summary(),
    }

    if rank == 0 and world == 1 and not args.no_extras:
        line["extras"] = extras(dev, args)
    if world > 1 and not args.no_extras:
        cp = context_parallel_extra(dev, rank, world, args, max_over_ranks, barrier)
        if rank == 0:
            line["extras"] = {"c4_context_parallel": cp}

    if keep:
        rate, done, toks, dt = cpu_oracle_rate(oracle_caches(wl.host, wl.lengths, wl.hot))
        line["cpu_baseline"] = {
            "value": rate, "unit": UNIT, "cores": host_cores(), "kind": "port",
            "sample": f"{len(keep)} of the 64 sequences, {done} oracle decodes ({toks} cached tokens) in {dt:.1f} s",
        }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    # the same step as one CUDA graph per rank (decode, merge, NCCL all-gather, combine)
    graph = dec.capture(wl.q_lat, wl.q_rope, wl.new_latent, wl.new_rope, out, softmax_scale=SOFTMAX_SCALE)
    ms = timed(graph.replay)
    torch.cuda.synchronize()
    del graph  # released before the process group is destroyed
    alg = wl.algorithmic_bytes()
    return {"seqs": 1, "cached_tokens": int(wl.lengths[0]), "ranks": world, "ms": ms, "ms_eager": ms_eager,
            "seq_steps_per_s": 1e3 / ms, "GB/s_total": alg / (ms / 1e3) / 1e9,
            "launch": "CUDA graph replay per step (ms_eager: the same step launched from Python)",
            "collective": "one all_gather_into_tensor of 32,896 B per rank per step (NCCL)"}


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

    from asterq.decode import DeviceDecodePlan, capture_step, latent_decode
    from asterq.plan import build_plan
    from asterq.synth import c1_inputs, c4_workload, c5_workload, PoolBuilder

    peak, _ = measured_peaks()
    res = {}
    timed = timed_ms
    res["c2_write_path"] = write_path_rate(dev, peak)

    def decode_rate(wl, name, iters):
        plan = build_plan(wl.layouts, wl.n_heads)
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

    inp = c1_inputs(seed=0)
    b1 = PoolBuilder([8192], [1024], q_len=1, n_heads=16, device=dev)
    b1.add(inp["latent"], inp["rope"], inp["q_lat"], inp["q_rope"])
    decode_rate(b1.finish("C1"), "c1_single_sequence", 50)
    wl = c4_workload(dev)
    decode_rate(wl, "c4_long_context_1gpu", 30)
    del wl
    wl = c5_workload(dev)
    decode_rate(wl, "c5_mtp_verification_1gpu", 10)
    del wl
    torch.cuda.empty_cache()
    return res


if __name__ == "__main__":
    main()
