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


def test_config5_shard_fused_step_full_size(z2, oracle, cuda):
    """One GPU's shard of the batch-sharded fused configuration at full size:
    4096 streams (rank 3 of 8 over 32768, so first_stream = 12288), bf16 head
    [9*1024, 2048] ~N(0, 0.02^2) with the softcap in its epilogue, penalty 1.2
    over a 1024-entry history, top-k 50, top-p 0.95, T 0.7, min-p 0.02, seed
    2024, hidden ~N(0,1) redrawn every step, four steps through zonos2cu_ctx_step.
      - logits: within the stated bf16 tolerance 2e-2 of the oracle's head on
        the same bf16 operands (sampled rows);
      - codes, flags, generators, history: bit-exact against the oracle's
        sampler on the GPU's logits, every row of every step;
      - against the oracle's own logits (and the reference's libm expf), on 256
        of the streams: a code may differ only where a decision's margin lies
        within the logits' measured difference (or at an equal-probability
        tie); such rows are counted."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[5]
    n_ranks, rank, S, Cb = 8, 3, 4096, 9
    first, count = z2.shard_range(cfg.streams, n_ranks, rank)
    assert count == S
    Wb = W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=1024))
    Wr = W.from_bf16_bits(Wb)
    ctx = z2.Context(0, S, Cb, 1024, 2048, cfg.hist_len, seed=cfg.seed, first_stream=first)
    ctx.set_head(Wb, z2.BF16, 1024)
    hist = W.initial_history(cfg, S, first=first)
    ctx.set_history(hist, 0)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed + first, S)
    assert (ctx.get_rng() == rng).all()
    sub = np.arange(0, S, 16)                 # streams checked against the oracle's own logits
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, Cb, 1024), dtype=torch.float32, device=cuda)
    margin_cases, max_err = 0, 0.0
    for step in range(4):
        hb = W.to_bf16_bits(W.hidden(cfg, step, S, first))
        rng_sub, hist_sub = rng[sub].copy(), hist[sub].copy()
        ctx.step(_t(hb, cuda), z2.BF16, p, codes, flags, logits_out=logits)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        ref = oracle.head_softcap(Wr, 1024, Cb, 1024, W.from_bf16_bits(hb)[sub])
        err = float(np.abs(g[sub] - ref).max())
        assert err <= 2e-2, err                # stated bf16 tolerance
        max_err = max(max_err, err)
        oc, of, _ = oracle.step(g, prm, rng, hist, hist_pos=step, exp_mode=1)
        gc = codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"step {step}: {len(bad)} token mismatches, first {bad[:5].tolist()}"
        assert (flags.cpu().numpy() == of).all(), step
        assert (ctx.get_rng() == rng).all(), step
        # the oracle end to end (its own logits, libm expf) on the sampled streams
        rc, _, dg = oracle.step(ref, prm, rng_sub, hist_sub, hist_pos=step, exp_mode=0,
                                diags=True)
        tol = 4.0 * max(err, 1e-6) / cfg.temperature + 1e-5
        for s_, c_ in np.argwhere(rc != gc[sub]):
            d = dg[s_ * Cb + c_]
            assert d.margin < tol or d.tie, (step, s_, c_, d.margin, tol)
            margin_cases += 1
    h, pos = ctx.get_history()
    assert pos == 4 and (h == hist).all()
    assert z2.device_error() == 0
    print(f"config-5 shard: max |logit err| {max_err:.2e}; end-to-end margin cases "
          f"{margin_cases} of {4 * len(sub) * Cb} rows")
    assert margin_cases <= 0.01 * 4 * len(sub) * Cb
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
