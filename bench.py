"""Benchmark of the zonos2 decode-step output path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (every rank): the constrained large-batch sampling configuration --
4096 decode streams x 9 codebooks x 1024 vocab, softcapped f32 logits
~N(0, 4^2) with 1% of entries +8, delay-pattern masks, a 70% allow bitmask,
top-k 100, top-p 0.9, min-p 0.02, T 0.7, repetition penalty 1.1 over a
1024-entry history per row.  A step samples one batch of logits for every
stream; the delay step cycles through a 128-step rollout.  Streams are
batch-sharded: each of N ranks owns 4096 streams (weak scaling) and the int32
codes are all-gathered over NCCL every 32 steps (every step in e2e).  Logits and
history (151 MB each per rank) exceed the 126 MB L2, so no flush is needed
between steps.

The line printed by rank 0 carries: ``value`` (device-resident inputs,
CUDA-event timed, max over ranks), ``e2e`` (host logits -> codes on the host
through the library's public host API, copies inside the timed region),
``roofline`` of the sampler kernel against the measured HBM copy bandwidth,
``cpu_baseline`` (the reference's own sample_token, compiled unmodified,
timed on this host), ``clocks`` sampled through NVML during the timed
regions, and ``gpu_launches``.

``--impl reference`` times the reference's CPU implementation of the same
workload (oracle/_ref: the unmodified reference sources plus the build-defined
penalty / mask prologue) on all host cores; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "zonos2.cpp_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "sampled codes/sec (streams×9 codebooks) at B=4096; % HBM roofline; 1/2/4/8 GPU"
STREAMS, NCB, VOCAB, HIST = 4096, 9, 1024, 1024
TOPK, TOPP, MINP, TEMP, RHO, PAD = 100, 0.9, 0.02, 0.7, 1.1, 1023
ROLLOUT = 128
GATHER_EVERY = 32  # device-resident loop: steps of codes per all-gather
WORKLOAD = ("constrained sampling, 4096 streams x 9 codebooks x 1024 vocab per GPU: f32 "
            "logits ~N(0,4^2), 1% +8 spikes, softcap 15; delay masks over a 128-step rollout; "
            "70% allow bitmask; top-k 100, top-p 0.9, min-p 0.02, T 0.7; penalty 1.1 over "
            "1024-entry history")
# Algorithmic bytes of one (stream, codebook) row, the scope table's figure:
# logits read + history read + token write and history append + allow bits
# (one 128-byte mask per stream, shared by its 9 rows).
ROW_BYTES = 4 * VOCAB + 4 * HIST + 8 + 128 / NCB
# What the decode context actually has to move per row: logits, the 128-byte
# presence bitmap of the history instead of the ring, ring read + write,
# two u16 counts read and written, code and flag, allow bits, generator state.
DESIGN_ROW_BYTES = 4 * VOCAB + 128 + 8 + 8 + 8 + 128 / NCB + 64 / NCB
# DRAM bytes (read + write) of one sample_rows_kernel launch on this workload,
# from an ncu capture of `bench.py --steps 12 --warmup 3 --no-cpu-baseline
# --no-head`, launch 11 (dram__bytes_read.sum 167.17 MB +
# dram__bytes_write.sum 7.11 MB).
SAMPLER_TRAFFIC_BYTES = 174.28e6
# Kernels of ours per decode step: the persistent sampler (the decode context
# draws each step's uniforms during the step before).
LAUNCHES_PER_STEP = 1


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
class ClockSampler:
    """NVML samples of SM clock and throttle reasons while `active` is set."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons = [], set()
        self.active = threading.Event()
        self.stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        while not self.stop.is_set():
            if self.nv is not None and self.active.is_set():
                try:
                    mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                    rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.samples.append(mhz)
                    for bit, name in self.REASONS.items():
                        if rs & bit and name != "gpu_idle":
                            self.reasons.add(name)
                except Exception:
                    pass
            time.sleep(0.002)

    def result(self):
        self.stop.set()
        self.t.join(timeout=1)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
def cpu_reference_run(steps: int, warmup: int, streams: int, seed: int = 1234):
    """The reference's own sample_token (oracle/_ref) over `streams` streams of
    the workload per step, all host threads; returns (codes/s, threads, secs/step)."""
    import workloads as W
    from oracle import Reference, make_params
    R = Reference()
    cfg = W.CONFIGS[4]
    prm = make_params(TEMP, TOPK, TOPP, MINP, RHO, PAD)
    rs = np.random.default_rng(seed)
    batches = []
    for b in range(2):
        x = rs.normal(0.0, 4.0, size=(streams, NCB, VOCAB))
        x[rs.random(x.shape) < 0.01] = 8.0
        batches.append((15.0 * np.tanh(x / 15.0)).astype(np.float32))
    hist = W.initial_history(cfg, streams)
    allow = W.allow_bits(cfg, streams)
    from oracle import Oracle
    rng = Oracle().rng_seed_streams(seed, streams)
    for t in range(warmup):
        R.step(batches[t % 2], prm, rng, hist, hist_pos=t % HIST, allow=allow,
               delay_step=t % ROLLOUT)
    t0 = time.perf_counter()
    for i in range(steps):
        t = warmup + i
        R.step(batches[t % 2], prm, rng, hist, hist_pos=t % HIST, allow=allow,
               delay_step=t % ROLLOUT)
    dt = time.perf_counter() - t0
    return streams * NCB * steps / dt, R.num_threads(), dt / max(steps, 1)


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    try:
        value, threads, per_step = cpu_reference_run(args.steps, args.warmup, STREAMS)
    except Exception as e:  # the reference build is missing
        print(json.dumps({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"}))
        return
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "codes/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "streams": STREAMS, "threads": threads,
                   "implementation": "reference sample_token (unmodified sources) + "
                                     "build-defined prologue, OpenMP over streams"},
        "cpu_baseline": {"value": value, "unit": "codes/s", "cores": threads, "kind": "reference",
                         "sample": f"full steps of {STREAMS} streams x {NCB} rows"},
        "e2e": {"value": value, "unit": "codes/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def make_device_inputs(torch, dev, rank: int, n_batches: int = 2):
    """Config-4 inputs for this rank's 4096 streams, generated on the device."""
    import workloads as W
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + 7919 * rank)
    batches = []
    for _ in range(n_batches):
        x = torch.randn((STREAMS, NCB, VOCAB), generator=g, device=dev, dtype=torch.float32) * 4.0
        spike = torch.rand((STREAMS, NCB, VOCAB), generator=g, device=dev) < 0.01
        x = torch.where(spike, torch.full_like(x, 8.0), x)
        batches.append((15.0 * torch.tanh(x / 15.0)).contiguous())
        del x, spike
    cfg = W.CONFIGS[4]
    hist = W.initial_history(cfg, STREAMS, first=rank * STREAMS)
    allow = W.allow_bits(cfg, STREAMS, first=rank * STREAMS)
    return batches, hist, allow


def _bf16_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f).get("bf16_tflops", 1590.0))
    except Exception:
        return 1590.0


def time_head_gemm(torch, Z, dev, stream, Wt, B, g, reps: int = 20, warm: int = 3):
    """CUDA-event time of the bf16 head GEMM + softcap at batch B (ms/launch)."""
    h = torch.randn((B, 2048), generator=g, device=dev).to(torch.bfloat16)
    lg = torch.empty((B, NCB, VOCAB), dtype=torch.float32, device=dev)
    for _ in range(warm):
        Z.head_softcap(Wt, Z.BF16, VOCAB, NCB, VOCAB, h, lg, stream=stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        Z.head_softcap(Wt, Z.BF16, VOCAB, NCB, VOCAB, h, lg, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(reps, 1)
    tflops = 2.0 * B * 2048 * NCB * VOCAB / (ms / 1e3) / 1e12
    return {"ms": ms, "tflops": tflops, "frac_of_bf16_peak": tflops / _bf16_peak()}


def head_weights_dev(torch, dev, g):
    return (torch.randn((NCB * VOCAB, 2048), generator=g, device=dev) * 0.02).to(torch.bfloat16)


def measure_head(torch, Z, dev, stream, reps: int = 20):
    """The tcgen05 head GEMM (bf16, f32 accumulate, softcap epilogue) at the
    fused configurations' batch sizes, and the fused decode step at 4096
    streams (head + sampler, penalty 1.2 over 1024, top-k 50, top-p 0.95)."""
    import workloads as W
    out = {}
    g = torch.Generator(device=dev)
    g.manual_seed(2024)
    Wt = head_weights_dev(torch, dev, g)
    for B in (256, 4096):
        out[f"gemm_b{B}"] = time_head_gemm(torch, Z, dev, stream, Wt, B, g, reps)
    # the fused decode step, 4096 streams
    S = 4096
    cfg = W.CONFIGS[5]
    ctx = Z.Context(dev.index, S, NCB, VOCAB, 2048, HIST, seed=cfg.seed)
    ctx.set_head(W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=VOCAB)), Z.BF16, VOCAB)
    ctx.set_history(W.initial_history(cfg, S), 0)
    p = Z.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, PAD)
    h = torch.randn((S, 2048), generator=g, device=dev).to(torch.bfloat16)
    codes = torch.zeros((S, NCB), dtype=torch.int32, device=dev)
    for _ in range(3):
        ctx.step(h, Z.BF16, p, codes, stream=stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        ctx.step(h, Z.BF16, p, codes, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    out["fused_step_b4096"] = {"ms": ms, "codes_per_s": S * NCB / (ms / 1e3)}
    ctx.close()
    return out


def run_head_only(args):
    """Only the head GEMM at batch --head-only (warm-up, then --steps launches):
    the small case the head kernel is profiled on."""
    import torch
    import zonos2cu as Z
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(2024)
    Wt = head_weights_dev(torch, dev, g)
    r = time_head_gemm(torch, Z, dev, torch.cuda.current_stream(), Wt, args.head_only, g,
                       reps=args.steps, warm=args.warmup)
    err = Z.device_error()
    print(json.dumps({"head_only": args.head_only, **r, "device_error": err}), flush=True)
    if err:
        sys.exit(1)


def run_ours(args):
    import torch
    import torch.distributed as dist
    import sharding
    import zonos2cu as Z

    ws, rank, local = dist_env()
    first, _ = sharding.shard_range(ws * STREAMS, ws, rank)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    batches, hist, allow = make_device_inputs(torch, dev, rank)
    ctx = Z.Context(local, STREAMS, NCB, VOCAB, 0, HIST, seed=1234, first_stream=first)
    ctx.set_history(hist, 0)
    ctx.set_allow(allow)
    params = Z.SampleParams(TEMP, TOPK, TOPP, MINP, RHO, PAD)
    codes = torch.zeros((STREAMS, NCB), dtype=torch.int32, device=dev)
    flags = torch.zeros((STREAMS, NCB), dtype=torch.int32, device=dev)
    gathered = torch.zeros((ws * STREAMS, NCB), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def gather():
        sharding.gather_codes(codes, ws * STREAMS, ws, rank, out=gathered)

    # The device-resident loop keeps each step's codes in a ring of GATHER_EVERY
    # steps and all-gathers the ring to every rank once it is full (and at the
    # end): rank 0 collects output, which needs no per-step round trip.
    ring = torch.zeros((GATHER_EVERY, STREAMS, NCB), dtype=torch.int32, device=dev)
    ring_all = torch.zeros((ws, GATHER_EVERY, STREAMS, NCB), dtype=torch.int32, device=dev)

    def ring_step(t, i, n):
        ctx.sample(batches[t % len(batches)], params, ring[i % GATHER_EVERY], flags,
                   delay_step=t % ROLLOUT, stream=stream)

    def ring_flush(i, n):
        if ws > 1 and ((i + 1) % GATHER_EVERY == 0 or i == n - 1):
            dist.all_gather_into_tensor(ring_all, ring)

    clocks = ClockSampler(local) if rank == 0 else None

    # ---- device-resident timing -------------------------------------------
    for t in range(args.warmup):
        ring_step(t, t, args.warmup)
        ring_flush(t, args.warmup)
    barrier()
    if clocks:
        clocks.active.set()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ring_step(args.warmup + i, i, args.steps)
        ring_flush(i, args.steps)
    t_end.record(stream)
    barrier()
    # The sampler's own launch time (the roofline's denominator), from events
    # around each step's two launches, in a second pass of the same steps so the
    # events do not sit inside the throughput measurement.
    n_ev = args.steps
    k_start = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    k_end = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    for i in range(n_ev):
        k_start[i].record(stream)
        ring_step(args.warmup + args.steps + i, i, n_ev)
        k_end[i].record(stream)
        ring_flush(i, n_ev)
    barrier()
    if clocks:
        clocks.active.clear()
    total_ms = t_start.elapsed_time(t_end)
    kern_ms = sum(a.elapsed_time(b) for a, b in zip(k_start, k_end)) / max(n_ev, 1)
    if ws > 1:
        tt = torch.tensor([total_ms, kern_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, kern_ms = float(tt[0]), float(tt[1])
    rows = STREAMS * NCB
    value = rows * ws * args.steps / (total_ms / 1e3)

    # ---- end to end: host logits -> host codes ------------------------------
    host_batches = [b.cpu().pin_memory() for b in batches]
    host_codes = torch.zeros((ws, STREAMS, NCB), dtype=torch.int32).pin_memory()
    host_flags = torch.zeros((STREAMS, NCB), dtype=torch.int32).pin_memory()
    dev_in = torch.empty_like(batches[0])

    def e2e_step(t):
        hb = host_batches[t % len(host_batches)]
        if ws == 1:
            ctx.sample_host(hb.numpy(), params, host_codes[0].numpy(), host_flags.numpy(),
                            delay_step=t % ROLLOUT)
        else:
            dev_in.copy_(hb, non_blocking=True)
            ctx.sample(dev_in, params, codes, flags, delay_step=t % ROLLOUT, stream=stream)
            gather()
            if rank == 0:
                host_codes.view(ws * STREAMS, NCB).copy_(gathered, non_blocking=True)
            stream.synchronize()

    e2e_steps = max(1, min(args.steps, 64))
    for t in range(2):
        e2e_step(t)
    barrier()
    if clocks:
        clocks.active.set()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    w0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(args.warmup + i)
    e1.record(stream)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - w0) * 1e3
    if clocks:
        clocks.active.clear()
    e2e_ms = max(e0.elapsed_time(e1), wall_ms)
    if ws > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt[0])
    e2e_value = rows * ws * e2e_steps / (e2e_ms / 1e3)
    h2d = int(batches[0].numel() * 4)
    d2h = int(rows * 4 * (2 if ws == 1 else ws)) if rank == 0 else 0

    ctx.close()
    head = measure_head(torch, Z, dev, stream) if (rank == 0 and not args.no_head) else None
    if rank != 0:
        if ws > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    peaks = {}
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    launch_bytes = ROW_BYTES * rows
    achieved = launch_bytes / (kern_ms / 1e3) / 1e9

    cpu = None
    if ws == 1 and not args.no_cpu_baseline:
        try:
            cv, threads, _ = cpu_reference_run(steps=3, warmup=1, streams=args.cpu_streams)
            cpu = {"value": cv, "unit": "codes/s", "cores": threads, "kind": "reference",
                   "sample": f"{args.cpu_streams} streams x {NCB} rows x 3 steps of the same "
                             f"workload (unmodified reference sample_token, OpenMP)"}
        except Exception as e:
            cpu = {"value": None, "unit": "codes/s", "cores": 0, "kind": "reference",
                   "sample": f"unavailable: {type(e).__name__}: {e}"}

    line = {
        "metric": METRIC, "value": value, "unit": "codes/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "streams_per_gpu": STREAMS, "codebooks": NCB,
                   "vocab": VOCAB,
                   "parallelism": f"batch-sharded x{ws}, NCCL all-gather of the codes every "
                                  f"{GATHER_EVERY} steps (per step in e2e)",
                   "l2": "inputs larger than L2 (151 MB logits + 151 MB history per GPU per step)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": args.traffic,
                     "kernel": "sample_rows_kernel",
                     "kernel_ms": kern_ms,
                     "bytes_per_launch": launch_bytes, "peak_source": peak_src,
                     "design_bytes_per_launch": DESIGN_ROW_BYTES * rows,
                     "design_frac": DESIGN_ROW_BYTES * rows / (kern_ms / 1e3) / 1e9 / peak},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "codes/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "head": head,
        "clocks": clocks.result() if clocks else None,
    }
    print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-streams", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-head", action="store_true", help="skip the head GEMM / fused timing")
    ap.add_argument("--head-only", type=int, default=0, metavar="B",
                    help="time only the bf16 head GEMM at batch B (profiling case)")
    ap.add_argument("--traffic", type=float, default=SAMPLER_TRAFFIC_BYTES,
                    help="ncu dram bytes per sampler launch, when measured")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    elif args.head_only:
        run_head_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
