"""CUDA sampler parity against the oracle, through the C ABI.

The GPU computes the correctly rounded exp, so against the oracle in the same
exp mode every token, flag, generator state and history entry must be
bit-identical.  Against the oracle with the reference's own libm expf, a token
may differ only where the CDF margin at the draw (or at a top-p / min-p
cut) is below the f32 logit tolerance 1e-5; those rows are counted and logged.
"""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu

MARGIN_TOL = 1e-5   # f32 logit tolerance, applied to CDF / threshold margins


def _t(x, dev, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev)


def _u64(dev, a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).to(dev)


def _np_u64(t):
    return t.cpu().numpy().view(np.uint64)


def run_step(z2, oracle, dev, logits, prm, rng, hist=None, hist_pos=0, allow=None, delay=-1,
             row_stride=None):
    """One GPU step and the oracle on the same pre-step state; returns both."""
    import torch
    S, Cb = logits.shape[0], logits.shape[1]
    V = logits.shape[-1] if row_stride is None else logits.shape[-1]
    d_logits = _t(logits, dev)
    d_rng = _u64(dev, rng)
    d_hist = None if hist is None else _t(hist, dev)
    d_allow = None if allow is None else _t(allow.view(np.int32), dev)
    d_codes = torch.full((S, Cb), -7, dtype=torch.int32, device=dev)
    d_flags = torch.full((S, Cb), -7, dtype=torch.int32, device=dev)
    p = z2.SampleParams(prm.temperature, prm.top_k, prm.top_p, prm.min_p, prm.repetition_penalty,
                        prm.pad_id)
    z2.sample_rows(d_logits, p, d_rng, d_codes, flags=d_flags, hist=d_hist, hist_pos=hist_pos,
                   allow=d_allow, delay_step=delay, vocab=V)
    torch.cuda.synchronize()
    o_rng = rng.copy()
    o_hist = None if hist is None else hist.copy()
    oc, of, dg = oracle.step(logits, prm, o_rng, o_hist, hist_pos=hist_pos, allow=allow,
                             delay_step=delay, exp_mode=1, diags=True)
    g = dict(codes=d_codes.cpu().numpy(), flags=d_flags.cpu().numpy(), rng=_np_u64(d_rng),
             hist=None if d_hist is None else d_hist.cpu().numpy())
    o = dict(codes=oc, flags=of, rng=o_rng, hist=o_hist, diags=dg)
    return g, o


def assert_exact(g, o, what=""):
    bad = np.argwhere(g["codes"] != o["codes"])
    assert len(bad) == 0, f"{what}: {len(bad)} token mismatches, first {bad[:5].tolist()}"
    assert (g["flags"] == o["flags"]).all(), what
    assert (g["rng"] == o["rng"]).all(), what
    if o["hist"] is not None:
        assert (g["hist"] == o["hist"]).all(), what


def softcapped(rs, shape, sigma, spikes=0.0):
    x = rs.normal(0, sigma, size=shape)
    if spikes:
        x[rs.random(shape) < spikes] = 8.0
    return (15 * np.tanh(x / 15)).astype(np.float32)


def test_sampler_config2_teacher_forced(z2, oracle, cuda):
    """Config 2 shapes (64 x 9 x 1024, penalty 1.2 over 256, T .8, k 50, p .95)."""
    import workloads as W
    cfg = W.CONFIGS[2]
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, cfg.streams)
    hist = W.initial_history(cfg)
    for step in range(12):
        g, o = run_step(z2, oracle, cuda, W.step_logits(cfg, step), prm, rng, hist,
                        hist_pos=step % cfg.hist_len)
        assert_exact(g, o, f"step {step}")
        rng, hist = g["rng"], g["hist"]


def test_sampler_config4_constrained(z2, oracle, cuda):
    """Config 4 regime (spikes, delay masks, 70% allow bits, k 100, penalty 1.1/1024)
    on 96 streams, steps 0..9 so the delay pattern is exercised."""
    import workloads as W
    cfg = W.CONFIGS[4]
    S = 96
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    hist = W.initial_history(cfg, S)
    allow = W.allow_bits(cfg, S)
    for step in range(10):
        g, o = run_step(z2, oracle, cuda, W.step_logits(cfg, step, S), prm, rng, hist,
                        hist_pos=step, allow=allow, delay=step)
        assert_exact(g, o, f"step {step}")
        if step < 8:   # codebooks above the step are forced to PAD
            assert (g["codes"][:, step + 1:] == W.PAD).all()
        rng, hist = g["rng"], g["hist"]


KNOBS = [
    # temperature, top_k, top_p, min_p
    (0.7, 50, 0.9, 0.02),
    (0.7, 0, 0.9, 0.02),        # top-k off (full sort path)
    (0.7, 1024, 1.0, 0.0),      # every filter off
    (1.0, 1, 0.9, 0.02),        # greedy by top-k
    (0.7, 1023, 0.95, 0.0),
    (0.05, 50, 0.9, 0.02),      # near-greedy temperature
    (2.5, 300, 0.99, 0.001),    # > 256 candidates (shared-memory sort)
    (0.7, 50, 0.0, 0.0),        # top-p 0 keeps one
    (0.7, 50, 1.0, 1.0),        # min-p 1 keeps the maximum's ties
    (1e-30, 50, 0.9, 0.02),     # probabilities underflow: zero tail
]


@pytest.mark.parametrize("knobs", KNOBS)
def test_sampler_knob_regimes(z2, oracle, cuda, knobs):
    T, k, p, mp = knobs
    rs = np.random.default_rng(hash(knobs) % 2**32)
    S = 24
    lg = np.concatenate([
        softcapped(rs, (S // 4, 9, 1024), 3.0),
        softcapped(rs, (S // 4, 9, 1024), 4.0, spikes=0.02),
        np.round(rs.normal(0, 2, (S // 4, 9, 1024))).astype(np.float32),   # heavy ties
        rs.normal(0, 0.9, (S // 4, 9, 1024)).astype(np.float32),
    ])
    prm = make_params(T, k, p, mp, 1.0, 1023)
    rng = oracle.rng_seed_streams(3, S)
    g, o = run_step(z2, oracle, cuda, lg, prm, rng)
    assert_exact(g, o, str(knobs))


def test_sampler_masks_and_nonfinite(z2, oracle, cuda):
    rs = np.random.default_rng(5)
    S, Cb, V, H = 6, 9, 1024, 37           # odd history: scalar history path
    lg = softcapped(rs, (S, Cb, V), 3.0)
    lg[0, 0, 5] = np.nan
    lg[0, 1, 9] = np.inf
    lg[1, :, :] = -np.inf                   # stream 1: every logit masked
    lg[2, 3, :] = -2e9                      # finite but below the -1e9 running max start
    lg[3, 4, :] = 0.0                       # all equal: one giant tie
    allow = np.full((S, V // 32), 0xFFFFFFFF, np.uint32)
    allow[4, :] = 0x0000FFFF                # half the tokens of stream 4
    allow[5, :] = 0
    allow[5, 31] = 0x80000000               # only token 1023 for stream 5
    hist = rs.integers(-3, V + 3, (S, Cb, H), dtype=np.int32)   # out-of-range entries ignored
    prm = make_params(0.7, 50, 0.9, 0.02, 1.3, 1023)
    rng = oracle.rng_seed_streams(8, S)
    g, o = run_step(z2, oracle, cuda, lg, prm, rng, hist, hist_pos=H - 1, allow=allow, delay=2)
    assert_exact(g, o, "masks")
    assert g["flags"][0, 0] & z2.FLAG_NONFINITE and g["flags"][0, 1] & z2.FLAG_NONFINITE
    assert (g["flags"][1] & z2.FLAG_ALL_MASKED).all() and (g["codes"][1] == 1023).all()
    assert g["flags"][2, 3] & z2.FLAG_ALL_MASKED
    assert (g["codes"][5] == 1023).all()


@pytest.mark.parametrize("V,stride", [(1024, 1026), (1000, 1000), (7, 9), (1, 1), (513, 600)])
def test_sampler_vocab_and_stride(z2, oracle, cuda, V, stride):
    """Odd vocab sizes and the reference's [n_tok, 9, 1026] row stride (unaligned rows)."""
    import torch
    rs = np.random.default_rng(V)
    S, Cb = 5, 9
    buf = softcapped(rs, (S, Cb, stride), 3.0)
    prm = make_params(0.8, 40, 0.92, 0.03, 1.0, V - 1)
    rng = oracle.rng_seed_streams(77, S)
    d_buf = _t(buf, cuda)
    d_rng = _u64(cuda, rng)
    codes = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
    p = z2.SampleParams(0.8, 40, 0.92, 0.03, 1.0, V - 1)
    z2.sample_rows(d_buf, p, d_rng, codes, n_streams=S, n_cb=Cb, vocab=V, row_stride=stride)
    torch.cuda.synchronize()
    oc, _, _ = oracle.step(np.ascontiguousarray(buf[:, :, :V]), prm, rng, exp_mode=1)
    assert (codes.cpu().numpy() == oc).all()
    assert (_np_u64(d_rng) == rng).all()


def test_sampler_against_reference_expf_with_margins(z2, oracle, cuda):
    """GPU vs the oracle in the reference's libm-expf mode: mismatches only at margins."""
    import workloads as W
    cfg = W.CONFIGS[4]
    S = 256
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng0 = oracle.rng_seed_streams(cfg.seed, S)
    hist0 = W.initial_history(cfg, S)
    allow = W.allow_bits(cfg, S)
    logits = W.step_logits(cfg, 20, S)
    g, _ = run_step(z2, oracle, cuda, logits, prm, rng0, hist0, hist_pos=3, allow=allow, delay=20)
    o_rng, o_hist = rng0.copy(), hist0.copy()
    oc, _, dg = oracle.step(logits, prm, o_rng, o_hist, hist_pos=3, allow=allow, delay_step=20,
                            exp_mode=0, diags=True)
    margin_cases = 0
    for s, c in np.argwhere(g["codes"] != oc):
        d = dg[s * 9 + c]
        assert d.margin < MARGIN_TOL or d.tie, (s, c, d.margin)
        margin_cases += 1
    print(f"libm-expf margin cases: {margin_cases} of {S * 9} rows")
    assert margin_cases <= 3


def test_sample_token_drop_in_golden(z2, oracle, cuda):
    """The drop-in on the reference's golden rows: the reference's token unless tied."""
    import os
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "sample_kat.npz"))
    for i in range(len(g["token"])):
        T, k, p, mp = (float(x) for x in g["params"][i])
        rng = z2.Xoshiro256(0)
        rng.s[:] = g["rng"][i]
        tok = z2.sample_token(rng, g["logits"][i], 1024, T, int(k), p, mp)
        st = g["rng"][i].copy()
        otok, d = oracle.sample_token(st, g["logits"][i], T, int(k), p, mp, exp_mode=1)
        assert tok == otok, i
        assert (rng.s == st).all()
        if tok != g["token"][i]:
            _, d0 = oracle.sample_token(g["rng"][i].copy(), g["logits"][i], T, int(k), p, mp,
                                        exp_mode=0)
            assert d0.tie or d0.margin < MARGIN_TOL, i


def test_sample_token_drop_in_loop_matches_reference_loop(z2, oracle, cuda):
    """The reference's per-step loop (one generator, codebooks 0..8 in order,
    src/zonos2_generate.cpp:259-267) driven through the drop-in."""
    rs = np.random.default_rng(9)
    rng = z2.Xoshiro256(42)
    st = oracle.rng_seed(42)
    for step in range(4):
        frame = softcapped(rs, (9, 1026), 3.0)
        for cb in range(9):
            t1 = z2.sample_token(rng, frame[cb], 1024, 0.7, 50, 0.9, 0.02)
            t2, _ = oracle.sample_token(st, frame[cb, :1024], 0.7, 50, 0.9, 0.02, exp_mode=1)
            assert t1 == t2
    assert (rng.s == st).all()


def test_context_rollout_and_host_path(z2, oracle, cuda):
    """Context state (generators, history ring, allow bits) across steps, device and host calls."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[4]
    S = 32
    ctx = z2.Context(0, S, 9, 1024, 0, cfg.hist_len, seed=cfg.seed)
    hist = W.initial_history(cfg, S)
    ctx.set_history(hist, 0)
    allow = W.allow_bits(cfg, S)
    ctx.set_allow(allow)
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    rng = oracle.rng_seed_streams(cfg.seed, S)
    assert (ctx.get_rng() == rng).all()
    codes_d = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    for step in range(6):
        lg = W.step_logits(cfg, step, S)
        oc, _, _ = oracle.step(lg, prm, rng, hist, hist_pos=step, allow=allow, delay_step=step,
                               exp_mode=1)
        if step % 2 == 0:
            ctx.sample(_t(lg, cuda), p, codes_d, delay_step=step)
            torch.cuda.synchronize()
            gc = codes_d.cpu().numpy()
        else:
            gc = np.zeros((S, 9), np.int32)
            ctx.sample_host(lg, p, gc, delay_step=step)
        assert (gc == oc).all(), step
    h, pos = ctx.get_history()
    assert pos == 6 and (h == hist).all()
    assert (ctx.get_rng() == rng).all()
    ctx.close()


@pytest.mark.parametrize("H", [1, 6, 37, 1024])
def test_context_incremental_history_rollout(z2, oracle, cuda, H):
    """The context keeps token counts + a presence bitmap instead of scanning the
    ring; over a long rollout with heavy eviction and repeats the codes must
    equal the oracle's full-ring scan every step (low temperature: repeats)."""
    import torch
    S, Cb, V = 12, 9, 1024
    rs = np.random.default_rng(H)
    ctx = z2.Context(0, S, Cb, V, 0, H, seed=31)
    hist = rs.integers(-2, 40, (S, Cb, H), dtype=np.int32)   # few distinct tokens, empties
    ctx.set_history(hist, H - 1)
    prm = make_params(0.3, 20, 0.95, 0.0, 1.7, 1023)
    p = z2.SampleParams(0.3, 20, 0.95, 0.0, 1.7, 1023)
    rng = oracle.rng_seed_streams(31, S)
    pos = H - 1
    codes = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
    for step in range(40):
        lg = softcapped(rs, (S, Cb, V), 1.0)
        lg[:, :, :48] += 3.0                     # keep sampling the same few tokens
        oc, _, _ = oracle.step(lg, prm, rng, hist, hist_pos=pos, exp_mode=1)
        ctx.sample(_t(lg, cuda), p, codes)
        torch.cuda.synchronize()
        assert (codes.cpu().numpy() == oc).all(), step
        pos = (pos + 1) % H
    h, hp = ctx.get_history()
    assert hp == pos and (h == hist).all()
    # re-indexing from a new ring mid-rollout
    hist2 = rs.integers(0, V, (S, Cb, H), dtype=np.int32)
    ctx.set_history(hist2, 0)
    lg = softcapped(rs, (S, Cb, V), 2.0)
    oc, _, _ = oracle.step(lg, prm, rng, hist2, hist_pos=0, exp_mode=1)
    ctx.sample(_t(lg, cuda), p, codes)
    torch.cuda.synchronize()
    assert (codes.cpu().numpy() == oc).all()
    ctx.close()


def _state_with_first_uniform(oracle, u, seed):
    """A generator state whose first draw gives the f32 uniform `u` (a multiple
    of 2^-24): the output rotl(s1 * 5, 7) * 9 is inverted for s1 (5 and 9 are
    odd, so invertible mod 2^64); s0, s2, s3 come from a seeded state."""
    M64 = (1 << 64) - 1
    out = (int(round(u * 2 ** 53)) << 11) & M64
    x = (out * pow(9, -1, 1 << 64)) & M64
    x = ((x >> 7) | (x << 57)) & M64          # rotr 7
    s1 = (x * pow(5, -1, 1 << 64)) & M64
    st = oracle.rng_seed(seed).copy()
    st[1] = np.uint64(s1)
    assert oracle.randf(st.copy()) == np.float32(u)
    return st


def test_sampler_exact_fallbacks(z2, oracle, cuda):
    """Rows built to leave the fast paths: (a) a penalty < 1 (the prologue logit
    by logit), (b) pairs of logits one ulp apart with their tokens in reverse
    order (the quantized sort keys tie, the exact order check re-sorts), (c) a
    uniform exactly on a partial sum of the CDF (the walk term by term)."""
    rs = np.random.default_rng(21)
    S, Cb, V, H = 8, 9, 1024, 64
    lg = softcapped(rs, (S, Cb, V), 3.0)
    # (b) streams 0-3: 24 one-ulp pairs near each row's top, larger logit on the larger token
    for s in range(4):
        for c in range(Cb):
            row = lg[s, c]
            top = float(row.max())
            toks = rs.choice(V, size=48, replace=False)
            for a_, b_ in zip(sorted(toks[:24]), sorted(toks[24:])):
                lo_t, hi_t = min(a_, b_), max(a_, b_)
                v = np.float32(top - rs.uniform(0.05, 1.5))
                row[hi_t] = v
                row[lo_t] = np.nextafter(v, np.float32(-np.inf))
    # (c) streams 4-7, codebook 0: four equal maxima, top-k 4 -> CDF 1/4, 1/2, 3/4, 1;
    # the stream's first uniform is exactly 1/2
    for s in range(4, 8):
        lg[s, 0, :] = -20.0
        lg[s, 0, [3, 100, 517, 1000]] = 5.0
    hist = rs.integers(0, V, (S, Cb, H), dtype=np.int32)
    for s in range(4, 8):   # keep the four maxima unpenalised, hence equal
        h0 = hist[s, 0]
        h0[np.isin(h0, [3, 100, 517, 1000])] = 0
    rng = oracle.rng_seed_streams(11, S)
    for s in range(4, 8):
        rng[s] = _state_with_first_uniform(oracle, 0.5, 100 + s)
    for rho in (1.15, 0.85):   # (a): 0.85 < 1
        prm = make_params(0.7, 4, 0.9, 0.0, rho, 1023)
        g, o = run_step(z2, oracle, cuda, lg, prm, rng.copy(), hist.copy(), hist_pos=5)
        assert_exact(g, o, f"top-k 4, penalty {rho}")
        prm = make_params(0.7, 100, 0.9, 0.02, rho, 1023)
        g, o = run_step(z2, oracle, cuda, lg, prm, rng.copy(), hist.copy(), hist_pos=5)
        assert_exact(g, o, f"top-k 100, penalty {rho}")
