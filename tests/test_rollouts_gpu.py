"""Whole rollouts of the sampler-only and the fused configurations through the
decode context, every step checked against the oracle.

The state these carry from step to step is the generate loop's
(src/zonos2_generate.cpp:232-279): the generators, which advance by one draw per
codebook, and the repetition-history ring with its token index, which wraps
several times.  Every code, flag and generator state is compared bit for bit
with the oracle (correctly rounded exp, as the GPU computes it) at every step;
the oracle with the reference's libm expf may differ only where a decision's
margin lies within the f32 logit tolerance (counted), checked on the same
pre-step state so the two runs never diverge.
"""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu

MARGIN_TOL = 1e-5


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_config2_sampler_rollout_all_512_steps(z2, oracle, cuda):
    """64 streams x 9 x 1024, logits ~N(0, 3^2) softcapped, penalty 1.2 over a
    256-entry history (the ring wraps twice), T 0.8, top-k 50, top-p 0.95,
    min-p 0.02, seed 1234: all 512 steps."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[2]
    S, Cb = cfg.streams, 9
    ctx = z2.Context(0, S, Cb, 1024, 0, cfg.hist_len, seed=cfg.seed)
    hist = W.initial_history(cfg)
    ctx.set_history(hist, 0)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    margin_cases = 0
    for step in range(cfg.steps):
        lg = W.step_logits(cfg, step)
        pos = step % cfg.hist_len
        rng_l, hist_l = rng.copy(), hist.copy()
        oc, of, _ = oracle.step(lg, prm, rng, hist, hist_pos=pos, exp_mode=1)
        ctx.sample(_t(lg, cuda), p, codes, flags)
        torch.cuda.synchronize()
        gc = codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"step {step}: {len(bad)} mismatches, first {bad[:5].tolist()}"
        assert (flags.cpu().numpy() == of).all(), step
        rc, _, dg = oracle.step(lg, prm, rng_l, hist_l, hist_pos=pos, exp_mode=0, diags=True)
        for s_, c_ in np.argwhere(rc != gc):
            d = dg[s_ * Cb + c_]
            assert d.margin < MARGIN_TOL or d.tie, (step, s_, c_, d.margin)
            margin_cases += 1
        if step % 64 == 63:
            assert (ctx.get_rng() == rng).all(), step
    h, hp = ctx.get_history()
    assert hp == cfg.steps % cfg.hist_len and (h == hist).all()
    assert (ctx.get_rng() == rng).all()
    assert z2.device_error() == 0
    print(f"config 2: libm-expf margin cases {margin_cases} of {cfg.steps * S * Cb} rows")
    assert margin_cases <= 1e-3 * cfg.steps * S * Cb
    ctx.close()


def test_config3_fused_rollout_all_256_steps(z2, oracle, cuda):
    """256 streams, bf16 hidden ~N(0,1) redrawn each step and bf16 heads
    [9*1024, 2048] ~N(0, 0.02^2), T 1.0, top-k 50, top-p 0.9, min-p 0.05,
    penalty 1.2 over a 512-entry history, seed 7: all 256 steps of the fused
    step (head + softcap + sampler).  Logits within the stated bf16 tolerance
    2e-2 of the oracle's head on sampled rows; codes bit-exact against the
    oracle's sampler on the GPU's logits."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[3]
    S, Cb = cfg.streams, 9
    Wb = W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=1024))
    Wr = W.from_bf16_bits(Wb)
    ctx = z2.Context(0, S, Cb, 1024, 2048, cfg.hist_len, seed=cfg.seed)
    ctx.set_head(Wb, z2.BF16, 1024)
    hist = W.initial_history(cfg)
    ctx.set_history(hist, 0)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, Cb, 1024), dtype=torch.float32, device=cuda)
    max_err = 0.0
    for step in range(cfg.steps):
        hb = W.to_bf16_bits(W.hidden(cfg, step))
        ctx.step(_t(hb, cuda), z2.BF16, p, codes, flags, logits_out=logits)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        rows = np.arange(step % 31, S, 31)
        ref = oracle.head_softcap(Wr, 1024, Cb, 1024, W.from_bf16_bits(hb)[rows])
        err = float(np.abs(g[rows] - ref).max())
        assert err <= 2e-2, (step, err)        # stated bf16 tolerance
        max_err = max(max_err, err)
        oc, of, _ = oracle.step(g, prm, rng, hist, hist_pos=step % cfg.hist_len, exp_mode=1)
        gc = codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"step {step}: {len(bad)} mismatches, first {bad[:5].tolist()}"
        assert (flags.cpu().numpy() == of).all(), step
    h, hp = ctx.get_history()
    assert hp == cfg.steps % cfg.hist_len and (h == hist).all()
    assert (ctx.get_rng() == rng).all()
    assert z2.device_error() == 0
    print(f"config 3: 256 steps, max |logit err| {max_err:.2e}")
    ctx.close()
