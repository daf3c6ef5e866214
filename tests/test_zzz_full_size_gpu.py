"""Full-size runs on the GPU: the benchmark's whole per-GPU workload against the
oracle, and a short `bench.py` run against the JSON contract.  They take tens of
seconds (the inputs are made on the host) and are collected after every other
test.
"""
import subprocess
import sys

import numpy as np
import pytest

from oracle import make_params
from test_bench_contract import REPO, check_ours, last_json_line

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_context_full_size_bench_workload(z2, oracle, cuda):
    """The benchmark's per-GPU workload at full size -- 4096 streams x 9 x 1024,
    config-4 knobs, a 1024-entry history and 70% allow bits -- through the
    context as `bench.py` drives it (the first step primes the uniforms, the next
    ones use those drawn ahead by the sampler's own CTAs).  Every code, flag,
    generator state and history entry must equal the oracle's, step by step."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[4]
    S, Cb = 4096, 9
    ctx = z2.Context(0, S, Cb, 1024, 0, cfg.hist_len, seed=cfg.seed)
    hist = W.initial_history(cfg, S)
    ctx.set_history(hist, 0)
    allow = W.allow_bits(cfg, S)
    ctx.set_allow(allow)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    for i, delay in enumerate((7, 8, 9)):   # codebook 8 forced to PAD at delay step 7
        lg = W.step_logits(cfg, delay, S)
        oc, of, _ = oracle.step(lg, prm, rng, hist, hist_pos=i, allow=allow, delay_step=delay,
                                exp_mode=1)
        ctx.sample(_t(lg, cuda), p, codes, flags, delay_step=delay)
        torch.cuda.synchronize()
        gc = codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"step {i}: {len(bad)} token mismatches, first {bad[:5].tolist()}"
        assert (flags.cpu().numpy() == of).all(), i
        assert (ctx.get_rng() == rng).all(), i
    h, pos = ctx.get_history()
    assert pos == 3 and (h == hist).all()
    ctx.close()


def test_cuda_arm_line():
    """Five timed steps of the CUDA arm (no CPU baseline, no head timings)."""
    p = subprocess.run([sys.executable, "bench.py", "--steps", "5", "--warmup", "3",
                        "--no-cpu-baseline", "--no-head"], cwd=REPO, capture_output=True,
                       text=True, timeout=900)
    assert p.returncode == 0, p.stderr[-2000:]
    d = last_json_line(p.stdout)
    check_ours(d)
    assert d["n_gpus"] == 1 and d["steps"] == 5 and d["cpu_baseline"] is None
