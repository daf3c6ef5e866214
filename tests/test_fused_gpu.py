"""The fused decode step through the context: hidden -> head + softcap ->
sampler, against the oracle.

Tokens are compared bit for bit with the oracle run on the GPU's own logits
(the sampler is exact); the logits against the oracle's head within the
stated tolerances; and tokens against the oracle on the oracle's logits may
differ only where a draw or cut lies within that tolerance of a boundary
(counted).
"""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu


def _dev(x, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def test_fused_config1_f32_batch1(z2, oracle, cuda):
    """B=1, f32 heads [9*1026, 2048] ~N(0, 0.02^2), seed 42, default knobs."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[1]
    Wt = W.head_weights(cfg)                       # [9*1026, 2048] f32
    ctx = z2.Context(0, 1, 9, 1024, 2048, 0, seed=cfg.seed)
    ctx.set_head(Wt, z2.F32, W.ROWS_PER_CB)
    p = z2.default_params()
    prm = make_params(p.temperature, p.top_k, p.top_p, p.min_p, 1.0, 1023)
    rng = oracle.rng_seed_streams(cfg.seed, 1)
    codes = torch.zeros((1, 9), dtype=torch.int32, device=cuda)
    logits = torch.zeros((1, 9, 1024), dtype=torch.float32, device=cuda)
    margin_cases = 0
    for step in range(4):
        h = W.hidden(cfg, step)
        ctx.step(_dev(h, cuda), z2.F32, p, codes, logits_out=logits)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        ref = oracle.head_softcap(Wt, W.ROWS_PER_CB, 9, 1024, h)
        assert (np.abs(g - ref) / np.maximum(1.0, np.abs(ref))).max() <= 1e-5
        st = rng.copy()
        oc, _, _ = oracle.step(g, prm, rng, exp_mode=1)             # on the GPU's logits
        assert (codes.cpu().numpy() == oc).all()
        rc, _, dg = oracle.step(ref, prm, st, exp_mode=0, diags=True)   # reference path
        for c in np.argwhere(rc[0] != oc[0]).ravel():
            assert dg[c].margin < 1e-5 or dg[c].tie
            margin_cases += 1
    assert margin_cases <= 1
    # the host entry point gives the same codes
    ctx.set_rng(oracle.rng_seed_streams(cfg.seed, 1))
    h = W.hidden(cfg, 0)
    hc = np.zeros((1, 9), np.int32)
    ctx.step_host(h, z2.F32, p, hc)
    ctx.set_rng(oracle.rng_seed_streams(cfg.seed, 1))
    ctx.step(_dev(h, cuda), z2.F32, p, codes)
    torch.cuda.synchronize()
    assert (hc == codes.cpu().numpy()).all()
    ctx.close()


def test_fused_config3_bf16_rollout(z2, oracle, cuda):
    """B=256 bf16 hidden and heads, T 1.0, top-p 0.9, min-p 0.05, penalty 1.2
    over a 512-entry history, hidden redrawn every step."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[3]
    S = cfg.streams
    Wf = W.head_weights(cfg, rows_per_cb=1024)
    Wb = W.to_bf16_bits(Wf)
    Wr = W.from_bf16_bits(Wb)
    ctx = z2.Context(0, S, 9, 1024, 2048, cfg.hist_len, seed=cfg.seed)
    ctx.set_head(Wb, z2.BF16, 1024)
    hist = W.initial_history(cfg)
    ctx.set_history(hist, 0)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, 1023)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, 1023)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    codes = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    flags = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, 9, 1024), dtype=torch.float32, device=cuda)
    for step in range(3):
        hb = W.to_bf16_bits(W.hidden(cfg, step))
        ctx.step(_dev(hb, cuda), z2.BF16, p, codes, flags, logits_out=logits)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        rows = np.arange(0, S, 37)
        ref = oracle.head_softcap(Wr, 1024, 9, 1024, W.from_bf16_bits(hb)[rows])
        assert np.abs(g[rows] - ref).max() <= 1e-3      # stated bf16 tolerance: 2e-2
        oc, of, _ = oracle.step(g, prm, rng, hist, hist_pos=step, exp_mode=1)
        assert (codes.cpu().numpy() == oc).all(), step
        assert (flags.cpu().numpy() == of).all()
    h, pos = ctx.get_history()
    assert pos == 3 and (h == hist).all()
    assert z2.device_error() == 0
    ctx.close()


def test_fused_step_without_logits_out(z2, oracle, cuda):
    """The context's own logits buffer carries the step when no output is asked for."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[3]
    S = 40
    Wb = W.to_bf16_bits(W.head_weights(cfg, rows_per_cb=1024))
    a = z2.Context(0, S, 9, 1024, 2048, 0, seed=5)
    b = z2.Context(0, S, 9, 1024, 2048, 0, seed=5)
    a.set_head(Wb, z2.BF16, 1024)
    b.set_head(Wb, z2.BF16, 1024)
    p = z2.SampleParams(1.0, 50, 0.9, 0.05, 1.0, 1023)
    ca = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    cb = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    lg = torch.zeros((S, 9, 1024), dtype=torch.float32, device=cuda)
    for step in range(2):
        hb = _dev(W.to_bf16_bits(W.hidden(cfg, step, S)), cuda)
        a.step(hb, z2.BF16, p, ca)
        b.step(hb, z2.BF16, p, cb, logits_out=lg)
        torch.cuda.synchronize()
        assert (ca.cpu().numpy() == cb.cpu().numpy()).all()
    a.close()
    b.close()
