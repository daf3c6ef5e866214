"""Benchmark of the zonos2 decode-step output path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (every rank): the constrained large-batch sampling configuration --
4096 decode streams x 9 codebooks x 1024 vocab, softcapped f32 logits
~N(0, 4^2) with 1% of entries +8, delay-pattern masks, a 70% allow bitmask,
top-k 100, top-p 0.9, min-p 0.02, T 0.7, repetition penalty 1.1 over a
1024-entry history per row.  A step samples one batch of logits for every
stream; the delay step cycles through a 128-step rollout.  Streams are
batch-sharded: each of N ranks owns 4096 streams (weak scaling) and the int32
codes are collected on rank 0: in the device-resident loops every 32 steps (and
after the last) a ring half is pushed into rank 0's buffer by the copy engines
while the other half fills (zonos2cu_ipc_alloc / _ipc_open / _push_codes), in the
end-to-end loop and the check through the library's NCCL gather
(zonos2cu_gather_codes).
Logits and history (151 MB each per rank) exceed the 126 MB L2, so no flush is
needed between steps.

The line printed by rank 0 carries: ``value`` (device-resident inputs,
CUDA-event timed over the whole timed region, max over ranks), ``e2e`` (host
logits -> codes on the host through the library's public host API, copies
inside the timed region), ``roofline`` of the sampler kernel against the
measured HBM copy bandwidth, ``cpu_baseline`` (the reference's own
sample_token, compiled unmodified, timed on this host), ``fused`` (the
batch-sharded fused configuration: bf16 head GEMM + softcap + sampler over 4096
streams per rank, at every N), ``multi_gpu_check`` (N > 1: rank 0's gathered
and pushed codes against a one-GPU context over the whole global batch), ``clocks``
sampled through NVML during the timed regions, and ``gpu_launches``.

``--impl reference`` times the reference's CPU implementation of the same
workload (oracle/_ref: the unmodified reference sources plus the build-defined
penalty / mask prologue) on all host cores; rank 0 only.
"""
from __future__ import annotations

import argparse
import hashlib
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
STREAMS, NCB, VOCAB, HIST, DIM = 4096, 9, 1024, 1024, 2048
TOPK, TOPP, MINP, TEMP, RHO, PAD = 100, 0.9, 0.02, 0.7, 1.1, 1023
ROLLOUT = 128
GATHER_EVERY = 32  # device-resident loops: steps of codes per push to rank 0
VERIFY_STEPS = 3   # N > 1: steps compared against a one-GPU run of the global batch
WORKLOAD = ("constrained sampling, 4096 streams x 9 codebooks x 1024 vocab per GPU: f32 "
            "logits ~N(0,4^2), 1% +8 spikes, softcap 15; delay masks over a 128-step rollout; "
            "70% allow bitmask; top-k 100, top-p 0.9, min-p 0.02, T 0.7; penalty 1.1 over "
            "1024-entry history")
FUSED_WORKLOAD = ("batch-sharded fused step, 4096 streams per GPU (32768 at 8 GPUs): hidden "
                  "bf16 [4096, 2048] ~N(0,1) redrawn each step, heads bf16 [9*1024, 2048] "
                  "~N(0,0.02^2), f32 accumulate, softcap 15; penalty 1.2 over 1024-entry "
                  "history, top-k 50, top-p 0.95, min-p 0.02, T 0.7, seed 2024")
# Algorithmic bytes of one (stream, codebook) row, the scope table's figure:
# logits read + history read + token write and history append + allow bits
# (one 128-byte mask per stream, shared by its 9 rows).
ROW_BYTES = 4 * VOCAB + 4 * HIST + 8 + 128 / NCB
FUSED_ROW_BYTES = 4 * VOCAB + 4 * HIST + 8        # no allow bits in the fused configuration
# What the decode context actually has to move per row: logits, the 128-byte
# presence bitmap of the history instead of the ring, ring read + write,
# two u16 counts read and written, code and flag, allow bits, generator state.
DESIGN_ROW_BYTES = 4 * VOCAB + 128 + 8 + 8 + 8 + 128 / NCB + 64 / NCB
# DRAM bytes (read + write) of one sample_rows_kernel launch on this workload,
# from an ncu capture of `bench.py --steps 12 --warmup 3 --no-cpu-baseline
# --no-head --no-fused`, launch 11 (dram__bytes_read.sum 167.11 MB +
# dram__bytes_write.sum 5.60 MB).
SAMPLER_TRAFFIC_BYTES = 172.70e6
# Kernels of ours per decode step: the persistent sampler (the decode context
# draws each step's uniforms during the step before).
LAUNCHES_PER_STEP = 1
# Spin ahead of each timed region, so the host has queued the region's launches
# before its start event fires (the first launch does not wait on the host).
LEAD_CYCLES = 1_000_000


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


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
    the workload per step, on every host core (the thread count is passed
    explicitly: under torchrun OMP_NUM_THREADS is 1); returns (codes/s,
    threads, secs/step)."""
    import workloads as W
    from oracle import Oracle, Reference, make_params
    R = Reference()
    threads = host_cores()
    cfg = W.CONFIGS[4]
    prm = make_params(TEMP, TOPK, TOPP, MINP, RHO, PAD)
    rs = np.random.default_rng(seed)
    batches = []
    for b in range(2):
        x = rs.normal(0.0, 4.0, size=(streams, NCB, VOCAB))
        x[rs.random(x.shape) < 0.01] = 8.0
        batches.append((15.0 * np.tanh(x / 15.0)).astype(np.float32))
        del x
    hist = W.initial_history(cfg, streams)
    allow = W.allow_bits(cfg, streams)
    rng = Oracle().rng_seed_streams(seed, streams)
    for t in range(warmup):
        R.step(batches[t % 2], prm, rng, hist, hist_pos=t % HIST, allow=allow,
               delay_step=t % ROLLOUT, nthreads=threads)
    t0 = time.perf_counter()
    for i in range(steps):
        t = warmup + i
        R.step(batches[t % 2], prm, rng, hist, hist_pos=t % HIST, allow=allow,
               delay_step=t % ROLLOUT, nthreads=threads)
    dt = time.perf_counter() - t0
    return streams * NCB * steps / dt, threads, dt / max(steps, 1)


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
    """Config-4 inputs of rank `rank`'s 4096 streams, the logits generated on
    `dev` (a rank's inputs are the same whichever device makes them)."""
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


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def time_head_gemm(torch, Z, dev, stream, Wt, B, g, reps: int = 20, warm: int = 3):
    """CUDA-event time of the bf16 head GEMM + softcap at batch B (ms/launch)."""
    h = torch.randn((B, DIM), generator=g, device=dev).to(torch.bfloat16)
    lg = torch.empty((B, NCB, VOCAB), dtype=torch.float32, device=dev)
    for _ in range(warm):
        Z.head_softcap(Wt, Z.BF16, VOCAB, NCB, VOCAB, h, lg, stream=stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(LEAD_CYCLES)
    e0.record(stream)
    for _ in range(reps):
        Z.head_softcap(Wt, Z.BF16, VOCAB, NCB, VOCAB, h, lg, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(reps, 1)
    tflops = 2.0 * B * DIM * NCB * VOCAB / (ms / 1e3) / 1e12
    peak = float(_peaks()[0].get("bf16_tflops", 1590.0))
    return {"ms": ms, "tflops": tflops, "frac_of_bf16_peak": tflops / peak}


def head_weights_dev(torch, dev, g):
    return (torch.randn((NCB * VOCAB, DIM), generator=g, device=dev) * 0.02).to(torch.bfloat16)


def measure_head(torch, Z, dev, stream, reps: int = 20):
    """The tcgen05 head GEMM (bf16, f32 accumulate, softcap epilogue) at the
    fused configurations' batch sizes."""
    out = {}
    g = torch.Generator(device=dev)
    g.manual_seed(2024)
    Wt = head_weights_dev(torch, dev, g)
    for B in (256, 4096):
        out[f"gemm_b{B}"] = time_head_gemm(torch, Z, dev, stream, Wt, B, g, reps)
    return out


def measure_drop_in(Z, frames: int = 20):
    """Host-side latency of the sample_token drop-in (one row per call, 9 calls
    per frame as the reference's loop makes them)."""
    rs = np.random.default_rng(3)
    rows = (15 * np.tanh(rs.normal(0, 3, (frames + 2, NCB, 1026)) / 15)).astype(np.float32)
    rng = Z.Xoshiro256(42)
    for cb in range(NCB):
        Z.sample_token(rng, rows[0, cb], 1024, 0.7, 50, 0.9, 0.02)
    t0 = time.perf_counter()
    for f in range(frames):
        for cb in range(NCB):
            Z.sample_token(rng, rows[2 + f, cb], 1024, 0.7, 50, 0.9, 0.02)
    dt = time.perf_counter() - t0
    # the same frames as one call each through a one-stream context (9 codebooks,
    # the same generator, the reference's [9][1026] layout)
    ctx = Z.Context(0, 1, NCB, VOCAB, 0, 0, seed=42)
    params = Z.SampleParams(0.7, 50, 0.9, 0.02, 1.0, PAD)
    codes = np.zeros((1, NCB), np.int32)
    ctx.sample_host(rows[0:1], params, codes, row_stride=1026)
    t1 = time.perf_counter()
    for f in range(frames):
        ctx.sample_host(rows[2 + f:3 + f], params, codes, row_stride=1026)
    dt_ctx = time.perf_counter() - t1
    ctx.close()
    return {"us_per_call": dt / (frames * NCB) * 1e6, "us_per_frame": dt / frames * 1e6,
            "frames": frames, "context_us_per_frame": dt_ctx / frames * 1e6,
            "what": "zonos2cu_sample_token, 9 calls per frame; and one zonos2cu_ctx_sample_host "
                    "call per frame on a one-stream context"}


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


# ---------------------------------------------------------------------------
class Job:
    """One rank's view of the batch-sharded job: torch.distributed for the
    host-side plumbing (barriers, the timing max), the library's own NCCL
    communicator for the codes gather to rank 0, and rank 0's push buffer for
    the copy-engine collection (zonos2cu_ipc_alloc / _ipc_open / _push_codes)."""

    def __init__(self, torch, Z):
        import torch.distributed as dist
        self.torch, self.Z, self.dist = torch, Z, dist
        self.ws, self.rank, self.local = dist_env()
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.stream = torch.cuda.current_stream()
        self.comm = None
        if self.ws > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=self.dev)
            box = [Z.comm_unique_id() if self.rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            self.comm = Z.Comm(self.local, self.ws, self.rank, box[0])
            # rank 0's push buffer, [GATHER_EVERY][global streams][NCB] int32, mapped
            # into every other rank; each rank's block of a step is contiguous
            self.first, self.count = Z.shard_range(self.ws * STREAMS, self.ws, self.rank)
            self.push_buf = None
            box = [None]
            if self.rank == 0:
                self.push_buf, box[0] = Z.ipc_alloc(self.local,
                                                    4 * GATHER_EVERY * self.ws * STREAMS * NCB)
            dist.broadcast_object_list(box, src=0)
            self.push_dst = self.push_buf if self.rank == 0 else Z.ipc_open(self.local, box[0])
            self.copy_stream = torch.cuda.Stream(device=self.dev)
            # the loops' rings have two halves of GATHER_EVERY steps: one is pushed
            # while the other fills
            self.ready = [torch.cuda.Event() for _ in range(2)]
            self.done = [torch.cuda.Event() for _ in range(2)]
            self.pushed = [False, False]

    def barrier(self):
        if self.ws > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def aligned_start(self, ev):
        """Records `ev` on every rank once all have reached it on the device:
        a spin, then a one-element all-reduce, ahead of the start event."""
        self.torch.cuda._sleep(LEAD_CYCLES)
        if self.ws > 1:
            t = self.torch.ones(1, device=self.dev)
            self.dist.all_reduce(t)
        ev.record(self.stream)

    def max_over_ranks(self, *vals):
        if self.ws == 1:
            return vals
        t = self.torch.tensor(vals, device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return tuple(float(x) for x in t.tolist())

    def half_free(self, half):
        """The step stream waits for the ring half's previous push before the half
        is written again (once per GATHER_EVERY steps: a wait between two launches
        cuts their programmatic overlap)."""
        if self.ws > 1 and self.pushed[half]:
            self.stream.wait_event(self.done[half])

    def push_block(self, block, n_steps, half):
        """This rank's codes of n_steps steps ([n_steps][count][NCB], ring half
        `half`) to their place in rank 0's push buffer: one strided copy-engine
        copy on the copy stream, ordered after those steps."""
        if self.ws == 1:
            return
        self.ready[half].record(self.stream)
        self.copy_stream.wait_event(self.ready[half])
        self.Z.push_codes(block, n_steps, self.count * NCB, self.push_dst + 4 * self.first * NCB,
                          self.ws * STREAMS * NCB, stream=self.copy_stream)
        self.done[half].record(self.copy_stream)
        self.pushed[half] = True

    def pushes_done(self):
        """The step stream waits for every push issued so far (inside a timed
        region: the codes are on rank 0 when its end event fires)."""
        if self.ws > 1:
            ev = self.torch.cuda.Event()
            ev.record(self.copy_stream)
            self.stream.wait_event(ev)

    def gather(self, ring, n_steps, out):
        """n_steps of this rank's codes [n_steps][STREAMS][NCB] to rank 0."""
        if self.ws > 1 and n_steps > 0:
            self.comm.gather_codes(0, ring, n_steps, self.ws * STREAMS, NCB,
                                   out if self.rank == 0 else None, stream=self.stream)

    def close(self):
        if self.comm is not None:
            self.torch.cuda.synchronize()
            self.comm.close()
        if self.ws > 1:
            if self.rank != 0:
                self.Z.ipc_close(self.push_dst)
            self.dist.barrier()   # every mapping closed before rank 0 frees the buffer
            if self.rank == 0:
                self.Z.ipc_free(self.push_buf)
            self.dist.barrier()
            self.dist.destroy_process_group()


def codes_digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, np.int32).tobytes()).hexdigest()[:16]


def multi_gpu_check(job, params):
    """Rank 0's gathered codes of VERIFY_STEPS steps of the sharded run against
    one context over the whole global batch on rank 0's GPU (same inputs, same
    generators): every code must match."""
    torch, Z, ws, rank = job.torch, job.Z, job.ws, job.rank
    import workloads as W
    first, count = Z.shard_range(ws * STREAMS, ws, rank)
    batches, hist, allow = make_device_inputs(torch, job.dev, rank)
    ctx = Z.Context(job.local, count, NCB, VOCAB, 0, HIST, seed=1234, first_stream=first)
    ctx.set_history(hist, 0)
    ctx.set_allow(allow)
    ring = torch.zeros((VERIFY_STEPS, count, NCB), dtype=torch.int32, device=job.dev)
    for t in range(VERIFY_STEPS):
        ctx.sample(batches[t % 2], params, ring[t], delay_step=t, stream=job.stream)
    out = None
    if rank == 0:
        out = torch.zeros((ws * VERIFY_STEPS * STREAMS * NCB,), dtype=torch.int32, device=job.dev)
    job.gather(ring, VERIFY_STEPS, out)
    job.half_free(0)   # and the same steps pushed by the copy engines
    job.push_block(ring, VERIFY_STEPS, 0)
    job.pushes_done()
    job.barrier()   # every rank's pushes complete before rank 0 reads its buffer
    ctx.close()
    del batches
    result = None
    if rank == 0:
        got = out.view(ws, VERIFY_STEPS, STREAMS, NCB).permute(1, 0, 2, 3).reshape(
            VERIFY_STEPS, ws * STREAMS, NCB).cpu().numpy()
        N = ws * STREAMS
        pushed = torch.empty((VERIFY_STEPS * N * NCB,), dtype=torch.int32, device=job.dev)
        Z.push_codes(job.push_dst, 1, VERIFY_STEPS * N * NCB, pushed.data_ptr(),
                     VERIFY_STEPS * N * NCB, stream=job.stream)
        torch.cuda.synchronize()
        got_push = pushed.view(VERIFY_STEPS, N, NCB).cpu().numpy()
        del pushed
        whole = Z.Context(job.local, N, NCB, VOCAB, 0, HIST, seed=1234, first_stream=0)
        parts = [make_device_inputs(torch, job.dev, r) for r in range(ws)]
        whole.set_history(np.concatenate([p[1] for p in parts]), 0)
        whole.set_allow(np.concatenate([p[2] for p in parts]))
        glog = [torch.cat([p[0][b] for p in parts]) for b in range(2)]
        del parts
        codes = torch.zeros((N, NCB), dtype=torch.int32, device=job.dev)
        want = np.zeros((VERIFY_STEPS, N, NCB), np.int32)
        for t in range(VERIFY_STEPS):
            whole.sample(glog[t % 2], params, codes, delay_step=t, stream=job.stream)
            torch.cuda.synchronize()
            want[t] = codes.cpu().numpy()
        whole.close()
        del glog
        mism = int((got != want).sum())
        result = {"steps": VERIFY_STEPS, "global_streams": N, "rows": int(want.size),
                  "mismatches": mism, "mismatches_pushed": int((got_push != want).sum()),
                  "sha256_16_gathered": codes_digest(got),
                  "sha256_16_pushed": codes_digest(got_push),
                  "sha256_16_one_gpu": codes_digest(want),
                  "what": "rank 0's codes of the sharded run, gathered over NCCL and pushed by "
                          "the copy engines, vs one context over the whole global batch on "
                          "rank 0's GPU"}
        torch.cuda.empty_cache()
    job.barrier()
    return result


def time_sampler(job, params, steps, warmup, clocks):
    """The config-4 sampler loop: (total_ms, per-launch event ms, launches)."""
    torch = job.torch
    batches, hist, allow = make_device_inputs(torch, job.dev, job.rank)
    first, count = job.Z.shard_range(job.ws * STREAMS, job.ws, job.rank)
    ctx = job.Z.Context(job.local, count, NCB, VOCAB, 0, HIST, seed=1234, first_stream=first)
    ctx.set_history(hist, 0)
    ctx.set_allow(allow)
    flags = torch.zeros((STREAMS, NCB), dtype=torch.int32, device=job.dev)
    ring = torch.zeros((2, GATHER_EVERY, STREAMS, NCB), dtype=torch.int32, device=job.dev)

    def run(t0, n):
        # every GATHER_EVERY steps (and after the last) the filled ring half is
        # pushed to rank 0 by the copy engines while the other half fills (N > 1)
        for i in range(n):
            t = t0 + i
            blk, j = divmod(i, GATHER_EVERY)
            if j == 0:
                job.half_free(blk % 2)
            ctx.sample(batches[t % 2], params, ring[blk % 2, j], flags,
                       delay_step=t % ROLLOUT, stream=job.stream)
            if j == GATHER_EVERY - 1 or i == n - 1:
                job.push_block(ring[blk % 2], j + 1, blk % 2)
        job.pushes_done()

    run(0, warmup)
    job.barrier()
    if clocks:
        clocks.active.set()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    job.aligned_start(t_start)
    run(warmup, steps)
    t_end.record(job.stream)
    job.barrier()
    # Events around each launch, in a second pass (they break the programmatic
    # overlap of back-to-back launches, so they stay out of the timed region).
    ks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ke = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        ks[i].record(job.stream)
        ctx.sample(batches[i % 2], params, ring[0, i % GATHER_EVERY], flags,
                   delay_step=(warmup + steps + i) % ROLLOUT, stream=job.stream)
        ke[i].record(job.stream)
    job.barrier()
    if clocks:
        clocks.active.clear()
    total_ms = t_start.elapsed_time(t_end)
    ev_ms = sum(a.elapsed_time(b) for a, b in zip(ks, ke)) / max(steps, 1)
    ctx.close()
    return (batches, hist, allow), total_ms, ev_ms


def time_e2e(job, params, inputs, steps, clocks):
    """Host logits -> host codes: pinned host logits copied in, the sampler,
    codes collected on rank 0 and copied out, every step."""
    torch = job.torch
    batches, hist, allow = inputs
    first, count = job.Z.shard_range(job.ws * STREAMS, job.ws, job.rank)
    ctx = job.Z.Context(job.local, count, NCB, VOCAB, 0, HIST, seed=1234, first_stream=first)
    ctx.set_history(hist, 0)
    ctx.set_allow(allow)
    host_batches = [b.cpu().pin_memory() for b in batches]
    host_codes = torch.zeros((job.ws * STREAMS, NCB), dtype=torch.int32).pin_memory()
    host_flags = torch.zeros((STREAMS, NCB), dtype=torch.int32).pin_memory()
    dev_in = torch.empty_like(batches[0])
    codes = torch.zeros((STREAMS, NCB), dtype=torch.int32, device=job.dev)
    flags = torch.zeros((STREAMS, NCB), dtype=torch.int32, device=job.dev)
    gathered = torch.zeros((job.ws * STREAMS, NCB), dtype=torch.int32, device=job.dev)

    def step(t):
        hb = host_batches[t % 2]
        if job.ws == 1:
            ctx.sample_host(hb.numpy(), params, host_codes.numpy(), host_flags.numpy(),
                            delay_step=t % ROLLOUT)
        else:
            dev_in.copy_(hb, non_blocking=True)
            ctx.sample(dev_in, params, codes, flags, delay_step=t % ROLLOUT, stream=job.stream)
            job.gather(codes, 1, gathered)
            if job.rank == 0:
                host_codes.copy_(gathered, non_blocking=True)
            job.stream.synchronize()

    for t in range(2):
        step(t)
    job.barrier()
    if clocks:
        clocks.active.set()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(job.stream)
    w0 = time.perf_counter()
    for i in range(steps):
        step(2 + i)
    e1.record(job.stream)
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - w0) * 1e3
    if clocks:
        clocks.active.clear()
    ms = max(e0.elapsed_time(e1), wall_ms)
    ctx.close()
    return ms


def time_fused(job, steps, warmup, clocks):
    """The batch-sharded fused configuration: per rank 4096 streams, bf16
    head GEMM + softcap + sampler per step (zonos2cu_ctx_step), each step's
    codes pushed to rank 0 by the copy engines.  Returns the timed region's ms
    and the head / sampler kernel times from a second pass with events between
    the two kernels."""
    torch, Z = job.torch, job.Z
    import workloads as W
    cfg = W.CONFIGS[5]
    first, count = Z.shard_range(job.ws * STREAMS, job.ws, job.rank)
    ctx = Z.Context(job.local, count, NCB, VOCAB, DIM, HIST, seed=cfg.seed, first_stream=first)
    ctx.set_head(W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=VOCAB)), Z.BF16, VOCAB)
    ctx.set_history(W.initial_history(cfg, count, first=first), 0)
    p = Z.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, PAD)
    g = torch.Generator(device=job.dev)
    g.manual_seed(cfg.seed + 7919 * job.rank)
    hidden = [torch.randn((count, DIM), generator=g, device=job.dev).to(torch.bfloat16)
              for _ in range(2)]
    ring = torch.zeros((2, GATHER_EVERY, count, NCB), dtype=torch.int32, device=job.dev)

    def run(t0, n):
        for i in range(n):
            blk, j = divmod(i, GATHER_EVERY)
            if j == 0:
                job.half_free(blk % 2)
            ctx.step(hidden[(t0 + i) % 2], Z.BF16, p, ring[blk % 2, j], stream=job.stream)
            if j == GATHER_EVERY - 1 or i == n - 1:
                job.push_block(ring[blk % 2], j + 1, blk % 2)
        job.pushes_done()

    run(0, warmup)
    job.barrier()
    if clocks:
        clocks.active.set()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    job.aligned_start(t0)
    run(warmup, steps)
    t1.record(job.stream)
    job.barrier()
    if clocks:
        clocks.active.clear()
    total_ms = t0.elapsed_time(t1)
    # the two kernels apart, with events around each: the head GEMM on the same
    # bf16 weights into a logits buffer, then the context's sampler on it
    Wt = torch.from_numpy(W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=VOCAB)).view(
        np.int16)).to(job.dev).view(torch.bfloat16)
    lg = torch.empty((count, NCB, VOCAB), dtype=torch.float32, device=job.dev)
    n_ev = min(steps, 10)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_ev)]
    for i in range(n_ev):
        ev[i][0].record(job.stream)
        Z.head_softcap(Wt, Z.BF16, VOCAB, NCB, VOCAB, hidden[i % 2], lg, stream=job.stream)
        ev[i][1].record(job.stream)
        ctx.sample(lg, p, ring[0, i % GATHER_EVERY], stream=job.stream)
        ev[i][2].record(job.stream)
    job.barrier()
    head_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / n_ev
    sampler_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / n_ev
    ctx.close()
    return total_ms, head_ms, sampler_ms


def run_ours(args):
    import torch
    import zonos2cu as Z

    job = Job(torch, Z)
    ws, rank = job.ws, job.rank
    params = Z.SampleParams(TEMP, TOPK, TOPP, MINP, RHO, PAD)
    clocks = ClockSampler(job.local) if rank == 0 else None

    check = multi_gpu_check(job, params) if ws > 1 and not args.no_check else None

    inputs, total_ms, ev_ms = time_sampler(job, params, args.steps, args.warmup, clocks)
    total_ms, ev_ms = job.max_over_ranks(total_ms, ev_ms)
    rows = STREAMS * NCB
    value = rows * ws * args.steps / (total_ms / 1e3)

    e2e_steps = max(1, min(args.steps, 64))
    e2e_ms = job.max_over_ranks(time_e2e(job, params, inputs, e2e_steps, clocks))[0]
    e2e_value = rows * ws * e2e_steps / (e2e_ms / 1e3)
    h2d = int(inputs[0][0].numel() * 4)
    d2h = int(rows * 4 * (2 if ws == 1 else ws)) if rank == 0 else 0
    del inputs
    torch.cuda.empty_cache()

    fused = None
    if not args.no_fused:
        f_total, head_ms, f_samp = time_fused(job, args.steps, args.warmup, clocks)
        f_total, head_ms, f_samp = job.max_over_ranks(f_total, head_ms, f_samp)
        peaks, src = _peaks()
        flops = 2.0 * STREAMS * DIM * NCB * VOCAB
        fused = {
            "workload": FUSED_WORKLOAD, "streams_per_gpu": STREAMS, "n_gpus": ws,
            "steps": args.steps, "ms_per_step": f_total / args.steps,
            "codes_per_s": rows * ws * args.steps / (f_total / 1e3),
            "gather": f"codes pushed to rank 0 by the copy engines every {GATHER_EVERY} steps "
                      f"and after the last",
            "sampler_ms_events": f_samp,
            "head_ms_events": head_ms,
            "head_tflops": flops / (head_ms / 1e3) / 1e12,
            "head_frac_of_bf16_peak": flops / (head_ms / 1e3) / 1e12 /
                                      float(peaks.get("bf16_tflops", 1590.0)),
            "sampler_gbs": FUSED_ROW_BYTES * rows / (f_samp / 1e3) / 1e9,
            "sampler_frac_of_hbm": FUSED_ROW_BYTES * rows / (f_samp / 1e3) / 1e9 /
                                   float(peaks.get("hbm_gbs", 6650.0)),
            "peak_source": src,
            "kernels": "head_ms / sampler_ms from events around each kernel in a second pass "
                       "(the head on the same weights into a logits buffer, then the sampler)",
        }

    head = drop_in = None
    if rank == 0 and ws == 1 and not args.no_head:
        head = measure_head(torch, Z, job.dev, job.stream)
        drop_in = measure_drop_in(Z)

    if rank != 0:
        job.close()
        return

    peaks, peak_src = _peaks()
    peak = float(peaks.get("hbm_gbs", 6650.0))
    launch_bytes = ROW_BYTES * rows
    # The sampler's mean launch time: over the whole timed region at one GPU (it
    # holds nothing but the sampler's launches), from the per-launch events where
    # the region also waits for the pushes to rank 0.
    kern_ms = total_ms / args.steps if ws == 1 else ev_ms
    achieved = launch_bytes / (kern_ms / 1e3) / 1e9

    cpu = None
    if ws == 1 and not args.no_cpu_baseline:
        try:
            cv, threads, _ = cpu_reference_run(steps=args.cpu_steps, warmup=2, streams=STREAMS)
            cpu = {"value": cv, "unit": "codes/s", "cores": threads, "kind": "reference",
                   "sample": f"{args.cpu_steps} full steps of {STREAMS} streams x {NCB} rows of "
                             f"the same workload (unmodified reference sample_token, OpenMP "
                             f"on {threads} threads)"}
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
                   "parallelism": f"batch-sharded x{ws}, codes pushed to rank 0 by the copy "
                                  f"engines every {GATHER_EVERY} steps and after the last "
                                  f"(zonos2cu_push_codes into its zonos2cu_ipc_alloc buffer); "
                                  f"end to end: gathered over NCCL (zonos2cu_gather_codes) "
                                  f"every step",
                   "l2": "inputs larger than L2 (151 MB logits + 151 MB history per GPU per step)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": args.traffic,
                     "kernel": "sample_rows_kernel",
                     "kernel_ms": kern_ms,
                     "kernel_ms_source": "timed region / launches" if ws == 1
                                         else "events around each launch",
                     "kernel_ms_events": ev_ms,
                     "bytes_per_launch": launch_bytes, "peak_source": peak_src,
                     "design_bytes_per_launch": DESIGN_ROW_BYTES * rows,
                     "design_frac": DESIGN_ROW_BYTES * rows / (kern_ms / 1e3) / 1e9 / peak},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "codes/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "fused": fused,
        "multi_gpu_check": check,
        "head": head,
        "drop_in": drop_in,
        "clocks": clocks.result() if clocks else None,
    }
    print(json.dumps(line), flush=True)
    job.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-head", action="store_true", help="skip the head GEMM timings")
    ap.add_argument("--no-fused", action="store_true", help="skip the fused configuration")
    ap.add_argument("--no-check", action="store_true", help="skip the N > 1 codes check")
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
