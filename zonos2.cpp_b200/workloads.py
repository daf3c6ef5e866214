"""Seeded synthetic inputs with the shapes and value distributions of the five
decode-step configurations this path is measured on (there is no checkpoint
or dataset here: logits, hidden states and head weights are synthetic).

  1. one step, batch 1: hidden f32 ~N(0,1) [2048], heads f32 ~N(0, 0.02^2),
     seed 42, default knobs, empty history
  2. sampler rollout: 64 streams x 9 x 1024, 512 steps, logits ~N(0, 3^2)
     softcapped, penalty 1.2 over a 256-entry history, T 0.8, top-k 50,
     top-p 0.95, seed 1234
  3. fused head + sampler: 256 streams, hidden bf16 ~N(0,1), heads bf16
     ~N(0, 0.02^2), T 1.0, top-p 0.9, min-p 0.05, history 512, seed 7
  4. constrained sampling: 4096 x 9 x 1024, logits ~N(0, 4^2) with 1% of
     entries +8 before the softcap, delay-pattern masks, 70% allow bitmask
     (Bernoulli, seed 99), top-k 100, top-p 0.9, penalty 1.1 over 1024,
     128 steps
  5. batch-sharded scaling: 32768 streams split across GPUs, bf16 head +
     sampler, penalty 1.2 / history 1024, top-k 50, top-p 0.95, seed 2024
Unspecified knobs take the reference's Zonos2GenParams defaults
(src/zonos2.h:245-252): T 0.7, top-k 50, top-p 0.9, min-p 0.02.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

N_CB, VOCAB, DIM, ROWS_PER_CB, SOFTCAP, PAD = 9, 1024, 2048, 1026, 15.0, 1023


@dataclass(frozen=True)
class Config:
    name: str
    streams: int
    steps: int
    seed: int
    temperature: float = 0.7
    top_k: int = 50
    top_p: float = 0.9
    min_p: float = 0.02
    penalty: float = 1.0
    hist_len: int = 0
    logit_sigma: float = 0.0      # sampler-only configs: logits ~N(0, sigma^2)
    spikes: float = 0.0           # fraction of entries set to +8 before the softcap
    delay: bool = False
    allow_frac: float = 0.0       # 0: no allow bitmask
    fused: bool = False           # hidden -> head GEMM -> sampler
    dtype: str = "f32"


CONFIGS = {
    1: Config("single-step-b1-f32", 1, 1, 42, fused=True, dtype="f32"),
    2: Config("sampler-rollout-b64", 64, 512, 1234, temperature=0.8, top_k=50, top_p=0.95,
              penalty=1.2, hist_len=256, logit_sigma=3.0),
    3: Config("fused-head-b256-bf16", 256, 256, 7, temperature=1.0, top_p=0.9, min_p=0.05,
              penalty=1.2, hist_len=512, fused=True, dtype="bf16"),
    4: Config("constrained-b4096", 4096, 128, 1234, top_k=100, top_p=0.9, penalty=1.1,
              hist_len=1024, logit_sigma=4.0, spikes=0.01, delay=True, allow_frac=0.7),
    5: Config("sharded-b32768-bf16", 32768, 1000, 2024, top_k=50, top_p=0.95, penalty=1.2,
              hist_len=1024, fused=True, dtype="bf16"),
}


def softcap(x, cap=SOFTCAP):
    return (cap * np.tanh(x / cap)).astype(np.float32)


def step_logits(cfg: Config, step: int, streams: int | None = None, first: int = 0) -> np.ndarray:
    """[streams, 9, 1024] f32 softcapped logits of one step (sampler configs)."""
    S = cfg.streams if streams is None else streams
    rs = np.random.default_rng([cfg.seed, step, first])
    x = rs.normal(0.0, cfg.logit_sigma, size=(S, N_CB, VOCAB))
    if cfg.spikes:
        x[rs.random(x.shape) < cfg.spikes] = 8.0
    return softcap(x)


def initial_history(cfg: Config, streams: int | None = None, first: int = 0) -> np.ndarray:
    S = cfg.streams if streams is None else streams
    rs = np.random.default_rng([cfg.seed, 10**6, first])
    return rs.integers(0, VOCAB, size=(S, N_CB, cfg.hist_len), dtype=np.int32)


def allow_bits(cfg: Config, streams: int | None = None, first: int = 0) -> np.ndarray | None:
    """[streams, 32] u32: bit t of stream s set with probability allow_frac (seed 99)."""
    if not cfg.allow_frac:
        return None
    S = cfg.streams if streams is None else streams
    rs = np.random.default_rng([99, first])
    bits = rs.random((S, VOCAB)) < cfg.allow_frac
    return pack_bits(bits)


def pack_bits(bits: np.ndarray) -> np.ndarray:
    S, V = bits.shape
    w = bits.reshape(S, V // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return w.sum(axis=-1).astype(np.uint32)


def head_weights(cfg: Config, rows_per_cb: int = ROWS_PER_CB) -> np.ndarray:
    """[9*rows_per_cb, 2048] f32 ~N(0, 0.02^2) (bf16 configs round it)."""
    rs = np.random.default_rng([cfg.seed, 7777])
    return rs.normal(0.0, 0.02, size=(N_CB * rows_per_cb, DIM)).astype(np.float32)


def hidden(cfg: Config, step: int, streams: int | None = None, first: int = 0) -> np.ndarray:
    S = cfg.streams if streams is None else streams
    rs = np.random.default_rng([cfg.seed, step, first, 55])
    return rs.normal(0.0, 1.0, size=(S, DIM)).astype(np.float32)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 (round to nearest even) as uint16 bits."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)
