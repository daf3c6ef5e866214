"""Randomised sampler parity against the oracle, through the C ABI.

Seeded draws over the knob space and over logit shapes chosen to stress the
certified decisions of the fast path: near-greedy and very flat temperatures,
heavy ties and logits one ulp apart, spikes, probabilities that underflow,
deep and shallow top-p cuts, min-p near its ends, penalties on both sides of 1,
allow masks, delay-forced codebooks, odd vocab sizes and row strides.  Every
case must equal the oracle (correctly rounded exp mode) bit for bit: tokens,
flags, generator states and history.

The stateless batched call scans history rings and reads standard bitmaps; the
decode context keeps the history as counts + a presence map and the allow bits
lane-major, so the context cases run a few steps of a rollout through it.
Restates no reference code: the oracle (src/zonos2_generate.cpp:36-93 and the
build prologue) is the checker.
"""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu

CASES_PER_CHUNK = 40
CHUNKS = 12
CTX_CASES = 40
KINDS = ("normal", "softcap", "spiky", "ties", "near_ties", "flat", "huge", "extreme")


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _u64(dev, a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).to(dev)


def _logits(rs, shape, kind):
    """f32 logits of one of the shapes in KINDS."""
    if kind == "normal":
        x = rs.normal(0, 10 ** rs.uniform(-1.5, 1.5), shape)
    elif kind == "softcap":
        x = 15 * np.tanh(rs.normal(0, rs.uniform(1, 8), shape) / 15)
    elif kind == "spiky":
        x = rs.normal(0, 3, shape)
        x[rs.random(shape) < rs.uniform(0.002, 0.05)] += rs.uniform(4, 12)
    elif kind == "ties":        # few distinct values: long runs of equal probabilities
        x = np.round(rs.normal(0, rs.uniform(0.5, 4), shape) * rs.choice([1, 2, 8])) / 4
    elif kind == "near_ties":   # pairs one ulp apart, the larger logit on either token
        x = rs.normal(0, 2, shape).astype(np.float32)
        flat = x.reshape(-1, shape[-1])
        V = shape[-1]
        for row in flat:
            if V < 4:
                break
            k = int(rs.integers(1, max(2, V // 8)))
            a = rs.choice(V, size=k, replace=False)
            b = rs.choice(V, size=k, replace=False)
            row[b] = np.nextafter(row[a], np.float32(np.inf) if rs.random() < 0.5
                                  else np.float32(-np.inf))
        return x
    elif kind == "flat":        # nearly uniform: deep top-p cuts, long CDF walks
        x = rs.normal(rs.uniform(-5, 5), 10 ** rs.uniform(-4, -1), shape)
    elif kind == "huge":        # most probabilities underflow to zero
        x = rs.normal(0, 10 ** rs.uniform(2, 4), shape)
    else:                       # non-finite and out-of-range values mixed in
        x = rs.normal(0, 3, shape)
        u = rs.random(shape)
        x[u < 0.01] = np.nan
        x[(u >= 0.01) & (u < 0.02)] = np.inf
        x[(u >= 0.02) & (u < 0.06)] = -np.inf
        x[(u >= 0.06) & (u < 0.08)] = -3e9
    return np.asarray(x, np.float32)


def _knobs(rs, V):
    T = float(rs.choice([10 ** rs.uniform(-3, 1), 1.0, 0.7, 1e-20], p=[0.7, 0.1, 0.15, 0.05]))
    k = int(rs.choice([0, 1, 2, int(rs.integers(1, 200)), int(rs.integers(1, V + 5)), V - 1, V,
                       1024, 5000]))
    top_p = float(rs.choice([1.0, 0.0, rs.uniform(0.5, 0.999), rs.uniform(0, 1)],
                            p=[0.2, 0.05, 0.5, 0.25]))
    min_p = float(rs.choice([0.0, 10 ** rs.uniform(-4, -0.5), 1.0], p=[0.3, 0.65, 0.05]))
    rho = float(rs.choice([1.0, rs.uniform(1.01, 2.0), rs.uniform(0.5, 0.99)], p=[0.3, 0.5, 0.2]))
    pad = int(rs.choice([V - 1, int(rs.integers(0, V))]))
    return np.float32(T), k, np.float32(top_p), np.float32(min_p), np.float32(rho), pad


def _allow(rs, S, V):
    if rs.random() < 0.5:
        return None
    words = (V + 31) // 32
    dens = rs.choice([0.05, 0.5, 0.9, 1.0])
    bits = rs.random((S, words * 32)) < dens
    bits[:, V:] = False
    if rs.random() < 0.3:
        bits[0, :] = False                  # one stream with nothing allowed
    return np.packbits(bits.reshape(S, words, 4, 8)[..., ::-1], axis=-1).reshape(
        S, words, 4).view("<u4").reshape(S, words).astype(np.uint32)


@pytest.mark.parametrize("chunk", range(CHUNKS))
def test_sampler_fuzz_stateless(z2, oracle, cuda, chunk):
    import torch
    rs = np.random.default_rng(1000 + chunk)
    for case in range(CASES_PER_CHUNK):
        S = int(rs.integers(1, 12))
        Cb = int(rs.choice([1, 3, 9]))
        V = int(rs.choice([1024, 1024, 1024, int(rs.integers(1, 1025))]))
        stride = V + int(rs.choice([0, 0, 2, int(rs.integers(0, 9))]))
        kind = KINDS[int(rs.integers(0, len(KINDS)))]
        buf = _logits(rs, (S, Cb, stride), kind)
        T, k, tp, mp, rho, pad = _knobs(rs, V)
        H = int(rs.choice([0, 1, 17, 64, 256]))
        hist = None if H == 0 else rs.integers(-2, V + 2, (S, Cb, H), dtype=np.int32)
        pos = int(rs.integers(0, max(H, 1)))
        allow = _allow(rs, S, V)
        delay = int(rs.choice([-1, -1, int(rs.integers(0, 10))]))
        rng = oracle.rng_seed_streams(int(rs.integers(0, 2**31)), S)
        what = (f"chunk {chunk} case {case}: S={S} Cb={Cb} V={V} stride={stride} {kind} T={T} "
                f"k={k} p={tp} min_p={mp} rho={rho} pad={pad} H={H} allow={allow is not None} "
                f"delay={delay}")

        d_rng = _u64(cuda, rng)
        d_hist = None if hist is None else _t(hist, cuda)
        d_allow = None if allow is None else _t(allow.view(np.int32), cuda)
        d_codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
        d_flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
        p = z2.SampleParams(float(T), k, float(tp), float(mp), float(rho), pad)
        z2.sample_rows(_t(buf, cuda), p, d_rng, d_codes, flags=d_flags, hist=d_hist, hist_pos=pos,
                       allow=d_allow, delay_step=delay, n_streams=S, n_cb=Cb, vocab=V,
                       row_stride=stride)
        torch.cuda.synchronize()
        prm = make_params(float(T), k, float(tp), float(mp), float(rho), pad)
        o_rng = rng.copy()
        o_hist = None if hist is None else hist.copy()
        oc, of, _ = oracle.step(np.ascontiguousarray(buf[:, :, :V]), prm, o_rng, o_hist,
                                hist_pos=pos, allow=allow, delay_step=delay, exp_mode=1)
        gc = d_codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"{what}: {len(bad)} token mismatches, first {bad[:4].tolist()}"
        assert (d_flags.cpu().numpy() == of).all(), what
        assert (d_rng.cpu().numpy().view(np.uint64) == o_rng).all(), what
        if hist is not None:
            assert (d_hist.cpu().numpy() == o_hist).all(), what
    assert z2.device_error() == 0


def test_sampler_fuzz_context_rollouts(z2, oracle, cuda):
    """Decode contexts (history index, lane-major allow bits, uniforms drawn a
    step ahead): a few steps per random case, every code against the oracle's
    full-ring scan, then the generator states and the ring."""
    import torch
    rs = np.random.default_rng(77)
    for case in range(CTX_CASES):
        S = int(rs.integers(1, 40))
        Cb = int(rs.choice([1, 9]))
        V = 1024
        H = int(rs.choice([1, 5, 64, 1024]))
        seed = int(rs.integers(0, 2**31))
        kind = KINDS[int(rs.integers(0, len(KINDS)))]
        T, k, tp, mp, rho, pad = _knobs(rs, V)
        prm = make_params(float(T), k, float(tp), float(mp), float(rho), pad)
        p = z2.SampleParams(float(T), k, float(tp), float(mp), float(rho), pad)
        hist = rs.integers(-1, V, (S, Cb, H), dtype=np.int32)
        pos = int(rs.integers(0, H))
        allow = _allow(rs, S, V)
        ctx = z2.Context(0, S, Cb, V, 0, H, seed=seed)
        ctx.set_history(hist, pos)
        if allow is not None:
            ctx.set_allow(allow)
        rng = oracle.rng_seed_streams(seed, S)
        codes = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
        flags = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
        for step in range(4):
            lg = _logits(rs, (S, Cb, V), kind)
            delay = int(rs.choice([-1, step]))
            oc, of, _ = oracle.step(lg, prm, rng, hist, hist_pos=pos, allow=allow,
                                    delay_step=delay, exp_mode=1)
            ctx.sample(_t(lg, cuda), p, codes, flags=flags, delay_step=delay)
            torch.cuda.synchronize()
            what = (f"context case {case} step {step}: S={S} Cb={Cb} H={H} {kind} T={T} k={k} "
                    f"p={tp} min_p={mp} rho={rho} allow={allow is not None} delay={delay}")
            assert (codes.cpu().numpy() == oc).all(), what
            assert (flags.cpu().numpy() == of).all(), what
            pos = (pos + 1) % H
        h, hp = ctx.get_history()
        assert hp == pos and (h == hist).all(), f"context case {case}: history"
        assert (ctx.get_rng() == rng).all(), f"context case {case}: generators"
        ctx.close()
    assert z2.device_error() == 0
