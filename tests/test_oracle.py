"""The oracle (C restatement) against the reference's golden vectors.

tests/golden/*.npz were produced by the reference's own unmodified sources
(tests/golden/make_golden.py).  These tests pin the restatement before it is
trusted as the checker of the CUDA path.  CPU only.
"""
import os

import numpy as np
import pytest

from oracle import FLAG_ALL_MASKED, Oracle, Reference, make_params

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_rng_kat(oracle):
    g = load("rng_kat.npz")
    for i, seed in enumerate(g["seeds"]):
        st = oracle.rng_seed(int(seed))
        assert (st == g["seeded_state"][i]).all()
        st2 = st.copy()
        nxt = [oracle.rng_next(st) for _ in range(64)]
        assert nxt == [int(x) for x in g["next"][i]]
        uni = np.array([oracle.randf(st2) for _ in range(64)], np.float32)
        assert (uni.view(np.uint32) == g["randf"][i].view(np.uint32)).all()


def test_streams_seed_plus_index(oracle):
    st = oracle.rng_seed_streams(1234, 5)
    for s in range(5):
        assert (st[s] == oracle.rng_seed(1234 + s)).all()


def test_sample_kat(oracle):
    """Libm-exp restatement == reference token, except equal-probability ties."""
    g = load("sample_kat.npz")
    ties = 0
    for i in range(len(g["token"])):
        T, k, p, mp = (float(x) for x in g["params"][i])
        st = g["rng"][i].copy()
        tok, d = oracle.sample_token(st, g["logits"][i], T, int(k), p, mp, exp_mode=0)
        if tok != g["token"][i]:
            assert d.tie, f"row {i}: {tok} != {g['token'][i]} without a tie"
            ties += 1
    assert ties <= 4


def test_step_kat(oracle):
    """Two batched steps with penalty, allow mask, delay mask, all-masked stream."""
    g = load("step_kat.npz")
    T, k, p, mp, rho, pad = g["params"]
    prm = make_params(float(T), int(k), float(p), float(mp), float(rho), int(pad))
    rng = g["rng0"].copy()
    hist = g["hist0"].copy()
    for step in range(2):
        codes, flags, dg = oracle.step(g["logits"][step], prm, rng, hist, hist_pos=step,
                                       allow=g["allow"], delay_step=step, exp_mode=0, diags=True)
        diff = np.argwhere(codes != g["codes"][step])
        for s, c in diff:
            assert dg[s * codes.shape[1] + c].tie, (step, s, c)
        assert (flags == g["flags"][step]).all()
        assert (flags[1] == FLAG_ALL_MASKED).all()      # stream 1 has an empty allow mask
    assert (rng == g["rng_out"]).all()
    assert len(np.argwhere(hist != g["hist_out"])) <= 2


def test_head_kat(oracle):
    g = load("head_kat.npz")
    out = oracle.head_softcap(g["W"], int(g["rows_per_cb"]), 2, int(g["vocab"]), g["h"])
    assert (out.view(np.uint32) == g["out"].view(np.uint32)).all()


def test_exp_modes_differ_only_by_one_ulp(oracle):
    xs = -np.linspace(0, 100, 200001).astype(np.float32)
    a = np.array([oracle.L.orc_exp(float(x), 0) for x in xs[::97]], np.float32)
    b = np.array([oracle.L.orc_exp(float(x), 1) for x in xs[::97]], np.float32)
    assert np.abs(a.view(np.int32) - b.view(np.int32)).max() <= 1


ref_available = os.path.exists(os.path.join(os.path.dirname(GOLD), "..", "oracle", "_ref",
                                            "libzonos2_ref.so"))


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
def test_restatement_matches_reference_on_random_rows(oracle):
    """Random rows, all knob regimes: any mismatch is a tie with equal probability."""
    R = Reference()
    rs = np.random.default_rng(7)
    for trial in range(3000):
        kind = trial % 4
        if kind == 0:
            l = 15 * np.tanh(rs.normal(0, 3, 1024) / 15)
        elif kind == 1:
            x = rs.normal(0, 4, 1024)
            x[rs.random(1024) < 0.01] = 8
            l = 15 * np.tanh(x / 15)
        elif kind == 2:
            l = np.round(rs.normal(0, 2, 1024))
        else:
            l = rs.normal(0, 0.9, 1024)
        l = l.astype(np.float32)
        T = [0.7, 0.8, 1.0, 0.05][trial % 4]
        k = [50, 100, 0, 1024, 7][trial % 5]
        p = [0.9, 0.95, 1.0, 0.5][trial % 4]
        mp = [0.02, 0.05, 0.0][trial % 3]
        st = oracle.rng_seed(trial)
        st2 = st.copy()
        t1, d = oracle.sample_token(st, l, T, k, p, mp, exp_mode=0)
        t2 = R.sample_token(st2, l, T, k, p, mp)
        assert (st == st2).all()
        if t1 != t2:
            assert d.tie
            mx = max(np.float32(-1e9), l.max())
            e1 = oracle.L.orc_exp(float(np.float32((l[t1] - mx) / np.float32(T))), 0)
            e2 = oracle.L.orc_exp(float(np.float32((l[t2] - mx) / np.float32(T))), 0)
            assert e1 == e2


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
def test_restatement_step_matches_reference_harness(oracle):
    R = Reference()
    rs = np.random.default_rng(11)
    S, Cb, V, H = 8, 9, 1024, 96
    prm = make_params(0.7, 100, 0.9, 0.02, 1.1, 1023)
    rng = oracle.rng_seed_streams(5, S)
    hist = rs.integers(0, V, (S, Cb, H), dtype=np.int32)
    rng2, hist2 = rng.copy(), hist.copy()
    for step in range(4):
        x = rs.normal(0, 4, (S, Cb, V))
        lg = (15 * np.tanh(x / 15)).astype(np.float32)
        c1, f1, dg = oracle.step(lg, prm, rng, hist, hist_pos=step, delay_step=step, exp_mode=0,
                                 diags=True)
        c2, f2 = R.step(lg, prm, rng2, hist2, hist_pos=step, delay_step=step)
        for s, c in np.argwhere(c1 != c2):
            assert dg[s * Cb + c].tie
        assert (f1 == f2).all()
        hist2[:] = hist          # continue both from the same state
    assert (rng == rng2).all()


@pytest.mark.skipif(not ref_available, reason="oracle/_ref not built")
@pytest.mark.parametrize("dim,rows", [(2048, 9), (37, 5)])
def test_out_norm_pinned_to_reference(oracle, dim, rows):
    """The restated output RMSNorm equals the reference's own rms_norm_per_token
    (compiled unmodified), bit for bit, with and without a scale weight."""
    R = Reference()
    rs = np.random.default_rng(dim + rows)
    x = rs.normal(0, 3, (rows, dim)).astype(np.float32)
    w = rs.normal(1, 0.2, dim).astype(np.float32)
    for weight in (w, None):
        a = oracle.out_norm(x, 1e-5, weight)
        b = R.out_norm(x, 1e-5, weight)
        assert (a.view(np.uint32) == b.view(np.uint32)).all()


def test_cfg_blend_formula(oracle):
    rs = np.random.default_rng(3)
    c = rs.normal(0, 4, 1000).astype(np.float32)
    u = rs.normal(0, 4, 1000).astype(np.float32)
    s = np.float32(1.7)
    want = (u + s * (c - u)).astype(np.float32)   # float32 numpy: one rounding per op
    assert (oracle.cfg_blend(c, u, s) == want).all()
