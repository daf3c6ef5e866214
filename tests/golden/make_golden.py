"""Generate the golden vectors in this folder from the reference itself.

Runs the reference's own, unmodified sources, compiled by oracle/Makefile into
oracle/_ref/libzonos2_ref.so, on seeded synthetic inputs and stores inputs and
outputs as small .npz fixtures:

  rng_kat.npz     Xoshiro256** seeding + first outputs / uniforms
                  (src/zonos2_generate.cpp:11-33)
  sample_kat.npz  sample_token on single rows (src/zonos2_generate.cpp:36-93)
  step_kat.npz    one batched decode step through the unmodified sample_token
                  inside the build-defined prologue (penalty, masks, per-stream
                  generators), two steps in a row
  head_kat.npz    linear_forward + the softcap expression
                  (src/zonos2_model.cpp:200-216, :692-703)

Only this container has the reference tree; the fixtures travel with the repo.
Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from oracle import Reference, build, make_params  # noqa: E402


def softcap(x, cap=15.0):
    return (cap * np.tanh(x / cap)).astype(np.float32)


def row_logits(rs, kind, V):
    if kind == 0:   # softcapped N(0, 3^2)
        return softcap(rs.normal(0, 3, V))
    if kind == 1:   # softcapped N(0, 4^2) with 1% spikes at +8
        x = rs.normal(0, 4, V)
        x[rs.random(V) < 0.01] = 8.0
        return softcap(x)
    if kind == 2:   # head-like N(0, 0.9^2), no softcap saturation
        return rs.normal(0, 0.9, V).astype(np.float32)
    return softcap(rs.normal(0, 6, V))   # saturating


def main():
    build()
    R = Reference()

    # -- generator KATs ------------------------------------------------------
    seeds = np.array([0, 1, 7, 42, 99, 1234, 2024, 2**32 + 3, 2**64 - 1], dtype=np.uint64)
    nexts = np.zeros((len(seeds), 64), np.uint64)
    unis = np.zeros((len(seeds), 64), np.float32)
    states = np.zeros((len(seeds), 4), np.uint64)
    for i, s in enumerate(seeds):
        st = R.rng_seed(int(s))
        states[i] = st
        st2 = st.copy()
        for j in range(64):
            nexts[i, j] = R.rng_next(st)
        for j in range(64):
            unis[i, j] = R.randf(st2)
    np.savez_compressed(os.path.join(HERE, "rng_kat.npz"), seeds=seeds, seeded_state=states,
                        next=nexts, randf=unis)

    # -- single-row sampler KATs ---------------------------------------------
    rs = np.random.default_rng(20261201)
    rows, params, rng_in, toks = [], [], [], []
    psets = [  # temperature, top_k, top_p, min_p
        (0.7, 50, 0.9, 0.02),     # Zonos2GenParams defaults (src/zonos2.h:245-252)
        (0.8, 50, 0.95, 0.02),
        (1.0, 50, 0.9, 0.05),
        (0.7, 100, 0.9, 0.02),
        (0.7, 0, 0.9, 0.02),      # top-k off
        (0.7, 1024, 1.0, 0.0),    # every filter off
        (1.3, 7, 0.5, 0.0),
        (0.05, 50, 0.9, 0.02),    # near-greedy
    ]
    V = 1024
    for i in range(48):
        l = row_logits(rs, i % 4, V)
        T, k, p, mp = psets[i % len(psets)]
        st = R.rng_seed(1000 + i)
        st_in = st.copy()
        tok = R.sample_token(st, l, T, k, p, mp)
        rows.append(l)
        params.append((T, float(k), p, mp))
        rng_in.append(st_in)
        toks.append(tok)
    np.savez_compressed(os.path.join(HERE, "sample_kat.npz"), logits=np.stack(rows),
                        params=np.array(params, np.float32), rng=np.stack(rng_in),
                        token=np.array(toks, np.int32))

    # -- batched decode step KATs (two steps) --------------------------------
    S, Cb, V, H = 4, 9, 1024, 64
    prm = make_params(temperature=0.7, top_k=100, top_p=0.9, min_p=0.02,
                      repetition_penalty=1.1, pad_id=1023)
    logits = np.stack([row_logits(rs, 1, V) for _ in range(S * Cb * 2)]).reshape(2, S, Cb, V)
    hist0 = rs.integers(0, V, size=(S, Cb, H), dtype=np.int32)
    allow = np.zeros((S, V // 32), np.uint32)
    bits = rs.random((S, V)) < 0.7
    for s in range(S):
        for w in range(V // 32):
            allow[s, w] = int(sum(int(b) << j for j, b in enumerate(bits[s, w * 32:(w + 1) * 32])))
    allow[1, :] = 0   # an all-masked stream
    rng0 = np.stack([R.rng_seed(99 + s) for s in range(S)])
    rng, hist = rng0.copy(), hist0.copy()
    codes, flags = [], []
    for step in range(2):
        c, f = R.step(logits[step], prm, rng, hist, hist_pos=step, allow=allow, delay_step=step)
        codes.append(c)
        flags.append(f)
    np.savez_compressed(os.path.join(HERE, "step_kat.npz"), logits=logits, hist0=hist0,
                        allow=allow, rng0=rng0, codes=np.stack(codes), flags=np.stack(flags),
                        rng_out=rng, hist_out=hist,
                        params=np.array([prm.temperature, prm.top_k, prm.top_p, prm.min_p,
                                         prm.repetition_penalty, prm.pad_id], np.float32))

    # -- head + softcap KATs -------------------------------------------------
    D, Cb, rows_per_cb, Vh, B = 2048, 2, 10, 8, 3
    W = rs.normal(0, 0.02, size=(Cb * rows_per_cb, D)).astype(np.float32)
    h = rs.normal(0, 1, size=(B, D)).astype(np.float32)
    h[2] *= 40.0   # drives the softcap into saturation
    out = R.head_softcap(W, rows_per_cb, Cb, Vh, h, 15.0)
    np.savez_compressed(os.path.join(HERE, "head_kat.npz"), W=W, h=h, out=out,
                        rows_per_cb=rows_per_cb, vocab=Vh)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
