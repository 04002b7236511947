#!/usr/bin/env python
"""Attention forward throughput on B200: the BASELINE metric, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the box-scale sharded config): B=16, H=32, N=8192,
D=128, BF16 in / FP32 accumulate, scale 1/sqrt(D). One step = one dense forward
plus one causal forward over all 512 (batch, head) slabs. With N GPUs (one
process each, torchrun) the slabs are split into N contiguous ranges and each
rank runs the same kernel on its own range -- no collective on the data path
(total work fixed: strong scaling). Time is CUDA events on the launching stream,
max over ranks. TFLOP/s uses the reference's FLOP count (kernels/v0_unfused.cu:
118-126: causal pairs N(N+1)/2).

After W warm-up steps the GPU arm runs untimed steps for --soak-s seconds, so the
timed steps see the clock the GPU holds under its power limit at every N.

The reference arm (--impl reference) times the reference's CPU FP64 oracle
(benchmarks/bench_flash_attention.cu:105-145, as the oracle port that is pinned to
it bit for bit) on all host cores over a bounded, balanced sample of the same
workload: the same dense and causal rows of an (8192 x 128) slab on every thread.
"""
import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "attn fwd TFLOP/s per B200 (D=128, N=8192, dense+causal) and % of BF16 peak"
CONFIG = {"batch": 16, "heads": 32, "seq_len": 8192, "head_dim": 128}
FALLBACK_PEAK_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--shape", default=None,
                    help="B,H,N,D instead of config 5 (profiling and exploration; not the headline)")
    ap.add_argument("--mask", choices=["both", "dense", "causal"], default="both",
                    help="forwards per step (default: one dense + one causal)")
    ap.add_argument("--soak-s", type=float, default=3.0,
                    help="untimed seconds of steps after the warm-up, so the timed steps run at the "
                         "power-limited steady-state clock (0 = time right after the warm-up)")
    ap.add_argument("--gather", action="store_true",
                    help="with N > 1, also time the optional all-gather of the O slices (NCCL), "
                         "separately from the forward; reported under \"gather\"")
    return ap.parse_args()


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def slab_range(total, rank, world):
    """Contiguous, near-equal ranges of the flattened batch*heads axis."""
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            peaks = json.load(fh)
        return float(peaks["bf16_tflops"]), "measured burst cuBLAS bf16 (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s"


def measured_sustained_peak():
    """cuBLAS bf16 run back to back under the 1000 W power cap (MEASURED_PEAKS.json), or None."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        return None


def profile_traffic():
    """Per-launch DRAM bytes of the kernel from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "fa_fwd_kernel_traffic.json")
    try:
        with open(path) as fh:
            return json.load(fh)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_id), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def summary(self, since=None):
        """Median SM clock, power and the limit reasons seen, over the samples read at or after
        `since` (time.monotonic(); None = all samples)."""
        sm, mx, reasons, power = [], None, set(), []
        names = self.REASONS
        for stamp, line in self.lines:
            if since is not None and stamp < since:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            try:
                power.append(float(parts[2]))
            except ValueError:
                pass
            for name, flag in zip(names, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w": statistics.median(power) if power else None,
                "power_max_w": max(power) if power else None}


# ----------------------------------------------------------------------------- CPU legs
def cpu_slab_step(threads, seq_len, head_dim, causal):
    """One bounded, balanced sample of the workload on the host: every host thread computes one
    whole (seq_len x head_dim) slab with the same mask, so no thread idles while another
    finishes. The function timed is the reference's own reference_attention
    (benchmarks/bench_flash_attention.cu:105-145), compiled from its sources into oracle/_ref;
    where that library is absent, the oracle port pinned to it bit for bit
    (oracle/fa_oracle.cpp). Returns (flops, seconds, kind) with kind "reference" or "port"."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import fa_oracle
    ref = fa_oracle.load_reference()
    fn, kind = (ref.ref_reference_attention, "reference") if ref is not None else \
        (fa_oracle.load().fa_oracle_attention, "port")
    q, k, v = fa_oracle.make_inputs(1, 1, seq_len, head_dim)
    # A private copy of the slab and its output per thread, so no two threads share cache lines.
    slabs = [tuple(np.copy(x) for x in (q, k, v)) for _ in range(threads)]
    outs = [np.empty(seq_len * head_dim, np.float64) for _ in range(threads)]
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)

    def work(i):
        q_, k_, v_ = slabs[i]
        fn(P(q_), P(k_), P(v_), P(outs[i]), 1, 1, seq_len, head_dim, int(causal))

    pool = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    for t in pool:
        t.start()
    for t in pool:
        t.join()
    seconds = time.perf_counter() - t0
    flops = threads * fa_oracle.attention_flops(1, 1, seq_len, head_dim, causal)
    return flops, seconds, kind


def cpu_sample(threads, steps, seq_len, head_dim):
    """`steps` reference-arm steps, dense and causal alternating (dense first):
    {"tflops", "flops", "seconds", "kind", "per_mask"}."""
    flops = secs = 0.0
    kind = None
    per_mask = {"dense": [], "causal": []}
    for step in range(steps):
        causal = step % 2
        f, s_, kind = cpu_slab_step(threads, seq_len, head_dim, causal)
        flops += f
        secs += s_
        per_mask["causal" if causal else "dense"].append(f / s_ / 1e12)
    return {"tflops": flops / secs / 1e12, "flops": flops, "seconds": secs, "kind": kind,
            "per_mask": {m: spread(r) for m, r in per_mask.items() if r}}


def cpu_single_thread_configs():
    """The reference's reference_attention on one host thread at BASELINE configs 1 and 2
    (dense), whole problems: {name: {"ms": ..., "gflops": ...}}, or None without oracle/_ref."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import fa_oracle
    ref = fa_oracle.load_reference()
    if ref is None:
        return None
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    out = {}
    for name, (b, h, n, d) in (("config1", (1, 2, 128, 64)), ("config2", (2, 8, 2048, 64))):
        q, k, v = fa_oracle.make_inputs(b, h, n, d)
        o = np.empty(b * h * n * d, np.float64)
        t0 = time.perf_counter()
        ref.ref_reference_attention(P(q), P(k), P(v), P(o), b, h, n, d, 0)
        sec = time.perf_counter() - t0
        out[name] = {"ms": sec * 1e3, "gflops": fa_oracle.attention_flops(b, h, n, d, 0) / sec / 1e9,
                     "shape": [b, h, n, d], "causal": 0, "threads": 1}
    return out


def cpu_extrapolation(tflops):
    """One bench step (all slabs of config 5, one dense + one causal forward) at the sampled host
    rate. Every slab of a mask is the same work, so this is exact by slab count, but it is an
    extrapolation, not a measurement."""
    b, h, n, d = (CONFIG[key] for key in ("batch", "heads", "seq_len", "head_dim"))
    step_flops = 4.0 * b * h * d * (n * n + n * (n + 1) / 2.0)   # attention_flops, dense + causal
    return {"step_s": step_flops / (tflops * 1e12), "step_flops": step_flops,
            "note": "extrapolated by slab count from the sample (identical work per slab), not measured"}


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def spread(rates):
    return {"min": min(rates), "max": max(rates),
            "stdev": statistics.stdev(rates) if len(rates) > 1 else 0.0}


def run_reference_arm(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0   # the CPU reference runs once, on rank 0
    threads = host_threads()
    n, d = CONFIG["seq_len"], CONFIG["head_dim"]
    for step in range(args.warmup):   # warm-up on (1024 x D) slabs: the CPU has nothing to warm
        cpu_slab_step(threads, 1024, d, step % 2)
    sample = cpu_sample(threads, args.steps, n, d)
    value = sample["tflops"]
    secs = sample["seconds"]
    function = ("the reference's own reference_attention (bench_flash_attention.cu:105-145) from oracle/_ref"
                if sample["kind"] == "reference" else "the oracle port of reference_attention (no oracle/_ref)")
    description = (f"per step: every host thread computes one whole (N={n}, D={d}) slab, all threads the same "
                   f"mask, dense and causal alternating between steps; {function}; warm-up steps on "
                   f"(1024 x {d}) slabs")
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic N(0,1) bf16 (reference generator, seeds 11/22/33)",
        "impl": "reference",
        "config": {"workload": "BASELINE config 5 (16,32,8192,128) dense+causal, CPU sample", **CONFIG},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": sample["kind"],
                         "sample": description, "spread_over_steps": sample["per_mask"],
                         "extrapolated": cpu_extrapolation(value),
                         "single_thread": cpu_single_thread_configs()},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


# ----------------------------------------------------------------------------- GPU arm
def gpu_index(local_rank):
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    return visible.split(",")[local_rank] if visible else str(local_rank)


def clock_fields(summary):
    """A clock summary as a fixed-length float list (for an all-gather across ranks)."""
    bits = sum(1 << i for i, name in enumerate(ClockSampler.REASONS) if name in summary.get("reasons", []))
    return [summary.get("sm_mhz") or 0.0, summary.get("sm_max_mhz") or 0.0, summary.get("power_w") or 0.0,
            summary.get("power_max_w") or 0.0, float(summary.get("samples") or 0), float(bits)]


def clock_summary_from_fields(fields):
    sm, mx, power, power_max, samples, bits = fields
    return {"sm_mhz": sm or None, "sm_max_mhz": mx or None, "power_w": power or None,
            "power_max_w": power_max or None, "samples": int(samples),
            "reasons": [name for i, name in enumerate(ClockSampler.REASONS) if int(bits) >> i & 1]}


def run_ours(args):
    import torch
    import torch.distributed as dist
    from cuda_fused_attention_b200 import AttentionShape, attention_flops, device_status
    from cuda_fused_attention_b200 import _lib

    rank, world, local_rank = env_rank()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        # Communicator set-up lines (rank, nranks, transport) go to stderr, as the record of
        # which ranks took part; nothing of NCCL runs in the timed region. (The environment may
        # already set NCCL_DEBUG to VERSION, which prints only the banner.)
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT,ENV")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(values):
        t = torch.tensor(values, dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def gather_rows(values):
        t = torch.tensor(values, dtype=torch.float64, device=device)
        if world == 1:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [x.tolist() for x in out]

    lib = _lib.load()
    config = dict(CONFIG)
    if args.shape:
        b_, h_, n_, d_ = (int(x) for x in args.shape.split(","))
        config = {"batch": b_, "heads": h_, "seq_len": n_, "head_dim": d_}
    masks = {"both": (0, 1), "dense": (0,), "causal": (1,)}[args.mask]
    full = AttentionShape(**config)
    s0, s1 = slab_range(full.slabs, rank, world)
    local = s1 - s0
    n, d = full.seq_len, full.head_dim
    numel = local * n * d
    g = torch.Generator(device=device)
    tensors = []
    for seed in (11, 22, 33):
        g.manual_seed(seed * 1000 + rank)
        tensors.append(torch.randn(numel, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16))
    q, k, v = tensors
    o = torch.empty_like(q)
    stream = torch.cuda.current_stream(device)
    handle = ctypes.c_void_p(stream.cuda_stream)

    def launch(causal):
        st = lib.fa_sm100_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), local, 1, n, d,
                              causal, handle)
        if st != 0:
            raise RuntimeError(f"fa_sm100_fwd status {st}")

    flops_dense_local = attention_flops(AttentionShape(local, 1, n, d), False) if 0 in masks else 0.0
    flops_causal_local = attention_flops(AttentionShape(local, 1, n, d), True) if 1 in masks else 0.0
    flops_step_total = sum(attention_flops(full, bool(c)) for c in masks)

    def step():
        for c in masks:
            launch(c)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    status, word = device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} ({word:#x}) after warm-up")
    # The first collective sets up the NCCL communicator (about a second at 8 ranks). Done here,
    # before the soak, it cannot leave the GPUs idle between the soak and the timed steps.
    barrier()

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_index(local_rank)) as clocks:
        # Heat soak (untimed): keep stepping until the GPU has run for soak_s seconds, so that
        # the timed steps run in the power-limited steady state at every N. Without it a rank's
        # share of the timed steps can be shorter than the power limit's response (at N=8 the
        # timed region is ~60 ms), and N would compare burst clocks against capped ones.
        # The soak has to keep the GPU as busy as the timed steps do. It therefore keeps one batch
        # of ~50 ms of steps queued behind the one running, and waits for the older batch only.
        # Synchronising every few steps would leave the GPU idle while the host catches up: with
        # 8 ranks on one host that was 11 % of the soak at N=8, and the GPU then stayed below its
        # power limit.
        # Every rank runs the same number of soak steps (from the slowest rank's estimate), so
        # that the ranks finish the soak together and the barrier before the timed steps is
        # short: an idle gap there lets the clock return to its maximum before the timing starts.
        soak_steps = 0
        t_soak = time.monotonic()
        if args.soak_s > 0:
            step()
            step()
            torch.cuda.synchronize()
            soak_steps = 2
            per_step = max((time.monotonic() - t_soak) / 2, 1e-5)
            total, batch = max_over_ranks([float(args.soak_s / per_step), float(max(1, int(0.05 / per_step)))])
            total, batch = int(total), int(batch)
            pending = None
            while soak_steps < total:
                n_batch = min(batch, total - soak_steps)
                for _ in range(n_batch):
                    step()
                soak_steps += n_batch
                queued = torch.cuda.Event()
                queued.record(stream)
                if pending is not None:
                    pending.synchronize()
                pending = queued
        torch.cuda.synchronize()
        soak_s = time.monotonic() - t_soak
        barrier()
        torch.cuda.synchronize()
        t_timed = time.monotonic()
        start.record(stream)
        for a, b, c in ev:
            a.record(stream)
            if 0 in masks:
                launch(0)
            b.record(stream)
            if 1 in masks:
                launch(1)
            c.record(stream)
        end.record(stream)
        torch.cuda.synchronize()
        t_timed_end = time.monotonic()
    barrier()
    # Clock samples from the last second of the soak through the end of the timed region: the
    # timed region alone can be shorter than the 200 ms sampling period.
    clock_window = max(t_soak, t_timed - 1.0)
    my_clocks = clocks.summary(since=clock_window)
    total_ms = start.elapsed_time(end)
    dense_ms = statistics.mean(a.elapsed_time(b) for a, b, _ in ev)
    causal_ms = statistics.mean(b.elapsed_time(c) for _, b, c in ev)
    status, word = device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} ({word:#x}) after timing")
    ms_step, dense_ms_max, causal_ms_max = max_over_ranks([total_ms / args.steps, dense_ms, causal_ms])
    per_rank_clocks = [clock_summary_from_fields(f) for f in gather_rows(clock_fields(my_clocks))]
    value = flops_step_total / (ms_step * 1e-3) / 1e12
    peak, peak_src = measured_peak()
    sustained = measured_sustained_peak()
    # Dominant (only) kernel: the row-pair kernel fa_fwd_kernel<128, false, false>; per-launch algorithmic
    # FLOPs / mean launch time.
    achieved = (flops_dense_local + flops_causal_local) / ((dense_ms + causal_ms) * 1e-3) / 1e12
    traffic = profile_traffic()
    rank_mhz = [c["sm_mhz"] for c in per_rank_clocks if c["sm_mhz"]]
    mean_mhz = statistics.mean(rank_mhz) if rank_mhz else None
    clock_norm = None if mean_mhz is None else {
        "sm_mhz_mean_of_rank_medians": mean_mhz,
        "tflops_per_ghz_per_gpu": value / world / (mean_mhz / 1e3),
        "ms_per_step_x_ghz": ms_step * mean_mhz / 1e3,
        "note": "value and step time normalised by the SM clock the ranks ran at: compare these across N "
                "to separate the design's scaling from clock differences"}

    # ---- end-to-end through the host-buffer C ABI (pinned host memory) --------------------
    e2e = None
    if not args.no_e2e:
        hq = torch.empty(numel, dtype=torch.bfloat16, pin_memory=True)
        hk = torch.empty_like(hq, pin_memory=True)
        hv = torch.empty_like(hq, pin_memory=True)
        ho = torch.empty_like(hq, pin_memory=True)
        hq.copy_(q)
        hk.copy_(k)
        hv.copy_(v)

        # The PCIe link's rate for one tensor each way (pinned, CUDA events), for the bound below.
        def link_gbs(dst, src):
            dst.copy_(src, non_blocking=True)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dst.copy_(src, non_blocking=True)
            b.record(stream)
            b.synchronize()
            return src.numel() * src.element_size() / (a.elapsed_time(b) * 1e-3) / 1e9
        h2d_gbs = link_gbs(o, hq)
        d2h_gbs = link_gbs(ho, o)

        def host_step():
            for causal in masks:
                st = lib.fa_sm100_fwd_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(),
                                           local, 1, n, d, causal)
                if st != 0:
                    raise RuntimeError(f"fa_sm100_fwd_host status {st}")
        for _ in range(max(1, args.warmup)):
            host_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host_step()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        barrier()
        (e2e_ms, h2d_min, d2h_min) = max_over_ranks([e2e_ms, -h2d_gbs, -d2h_gbs])
        h2d_min, d2h_min = -h2d_min, -d2h_min
        tensor_bytes = full.numel * 2
        h2d_bytes = len(masks) * 3 * tensor_bytes
        d2h_bytes = len(masks) * tensor_bytes
        # H2D and D2H overlap (separate copy engines), so the link bound of a step is the
        # slower direction's bytes per GPU over that direction's measured rate.
        link_ms = max(h2d_bytes / world / (h2d_min * 1e9), d2h_bytes / world / (d2h_min * 1e9)) * 1e3
        e2e = {"value": flops_step_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d_bytes,
               "d2h_bytes_per_step": d2h_bytes,
               "api": "fa_sm100_fwd_host (C ABI, pinned host buffers, H2D+forward+D2H per call; "
                      "one dense and one causal call per step; bytes summed over ranks)",
               "link": {"h2d_gbs": h2d_min, "d2h_gbs": d2h_min, "bound_ms_per_step": link_ms,
                        "bound_tflops": flops_step_total / (link_ms * 1e-3) / 1e12,
                        "note": "pinned copy rate of one tensor each way on this GPU's PCIe link (slowest rank); "
                                "the step cannot beat its H2D bytes at that rate"}}
        lib.fa_sm100_release_staging()
        del hq, hk, hv, ho

    # ---- the optional O gather, timed on its own (not part of the step) ----------------------
    gather = None
    if args.gather and world > 1:
        from cuda_fused_attention_b200.sharded import SlabShard, time_gather
        gather = time_gather(o, SlabShard(full, rank, world), iters=max(1, min(args.steps, 5)),
                             warmup=max(1, min(args.warmup, 2)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The reference arm's first two steps: one dense and one causal whole slab per host thread.
        threads = host_threads()
        sample = cpu_sample(threads, 2, n, d)
        cpu = {"value": sample["tflops"], "unit": "TFLOP/s", "cores": threads, "kind": sample["kind"],
               "sample": f"the reference arm's first two steps: every host thread computes one whole ({n} x {d}) "
                         f"slab dense, then one causal; "
                         + ("the reference's own reference_attention from oracle/_ref"
                            if sample["kind"] == "reference" else "the oracle port of reference_attention")
                         + f"; {sample['seconds']:.1f} s wall",
               "per_mask": sample["per_mask"],
               "extrapolated": cpu_extrapolation(sample["tflops"]),
               "single_thread": cpu_single_thread_configs()}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: torch.randn N(0,1) rounded to bf16, seeds 11/22/33 per rank",
        "config": {"workload": ("BASELINE config 5: (16,32,8192,128), one dense + one causal forward per step"
                                if not args.shape and args.mask == "both" else
                                f"exploration shape {tuple(config.values())}, masks {args.mask} (not the headline)"),
                   **config, "global_batch": config["batch"],
                   "parallelism": f"slab-sharded x{world} (batch*heads split, no collective)",
                   "l2": "inputs larger than L2 (3 GiB of Q/K/V + 1 GiB O per forward)"},
        "soak": {"seconds": soak_s, "steps": soak_steps,
                 "gpu_busy": (min(1.0, soak_steps * (total_ms / args.steps) * 1e-3 / soak_s) if soak_s > 0 else None),
                 "note": "untimed steps after the warm-up, kept queued back to back, so that every N is "
                         "timed at the power-limited steady-state clock (rank 0's figures; gpu_busy = "
                         "soak steps x the timed step time / soak wall time)"},
        "pct_of_bf16_peak": 100.0 * value / world / peak,
        "dense_tflops": (flops_dense_local * world / (dense_ms_max * 1e-3) / 1e12) if 0 in masks else None,
        "causal_tflops": (flops_causal_local * world / (causal_ms_max * 1e-3) / 1e12) if 1 in masks else None,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     # The kernel runs the GPU into its 1000 W cap (clock and power samples in
                     # "clocks"); cuBLAS measured under the same cap:
                     "sustained_peak": sustained,
                     "frac_vs_sustained": None if sustained is None else achieved / sustained,
                     "kernel": "fa_sm100::fa_fwd_kernel<128, false, false>",
                     "traffic": None if traffic is None else traffic.get("bytes_per_launch"),
                     "traffic_note": None if traffic is None else traffic.get("note")},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": len(masks) * args.steps * world,
        "clocks": {**my_clocks, "window": "last 1 s of the soak + the timed region", "per_rank": per_rank_clocks},
        "clock_normalised": clock_norm,
    }
    if gather is not None:
        line["gather"] = gather
    emit(line)
    return 0


# The result line goes to the process's original stdout; everything else that writes to
# file descriptor 1 while the bench runs (NCCL prints its version banner there, for one)
# is sent to stderr, so stdout carries exactly one JSON line.
_RESULT_OUT = None


def emit(line):
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def _keep_stdout_for_result():
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def main():
    args = parse_args()
    _keep_stdout_for_result()
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
