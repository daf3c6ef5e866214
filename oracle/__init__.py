"""TEST INFRASTRUCTURE ONLY -- ctypes bindings for the CPU checkers.

``Oracle`` wraps ``liboracle.so``, the C restatement of zonos2.cpp's
per-decode-step output path (``zonos2_oracle.c``).  ``Reference`` wraps
``_ref/libzonos2_ref.so``, the reference's own unmodified sources compiled by
``oracle/Makefile``.  Only tests, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline / reference legs import this package; the CUDA library never
does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libzonos2_ref.so")

FLAG_ALL_MASKED = 1
FLAG_NONFINITE = 2


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (the reference part only when its sources exist)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


class Params(C.Structure):
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_int),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("repetition_penalty", C.c_float),
        ("pad_id", C.c_int),
    ]


class Diag(C.Structure):
    _fields_ = [
        ("token", C.c_int),
        ("n_topk", C.c_int),
        ("n_final", C.c_int),
        ("pos", C.c_int),
        ("r", C.c_float),
        ("margin", C.c_float),
        ("tie", C.c_int),
    ]


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _u64(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint64))


def make_params(temperature=0.7, top_k=50, top_p=0.9, min_p=0.02, repetition_penalty=1.0,
                pad_id=1023) -> Params:
    return Params(temperature, top_k, top_p, min_p, repetition_penalty, pad_id)


class Oracle:
    """The C restatement (checker)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.orc_rng_seed.argtypes = [C.c_uint64, C.POINTER(C.c_uint64)]
        L.orc_rng_next.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_rng_next.restype = C.c_uint64
        L.orc_randf.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_randf.restype = C.c_float
        L.orc_rng_seed_streams.argtypes = [C.c_uint64, C.c_int, C.POINTER(C.c_uint64)]
        L.orc_exp.argtypes = [C.c_float, C.c_int]
        L.orc_exp.restype = C.c_float
        L.orc_sample_token_r.argtypes = [C.c_float, C.c_void_p, C.c_int, C.c_float, C.c_int,
                                         C.c_float, C.c_float, C.c_int, C.POINTER(Diag)]
        L.orc_sample_token_r.restype = C.c_int
        L.orc_sample_token.argtypes = [C.POINTER(C.c_uint64), C.c_void_p, C.c_int, C.c_float,
                                       C.c_int, C.c_float, C.c_float, C.c_int, C.POINTER(Diag)]
        L.orc_sample_token.restype = C.c_int
        L.orc_sample_row.argtypes = [C.c_float, C.c_void_p, C.c_int, C.POINTER(Params),
                                     C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                     C.POINTER(Diag), C.POINTER(C.c_int)]
        L.orc_sample_row.restype = C.c_int
        L.orc_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_long, C.POINTER(Params),
                               C.POINTER(C.c_uint64), C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                               C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                               C.c_int]
        L.orc_step.restype = C.c_int
        L.orc_head_softcap.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                       C.c_int, C.c_float, C.c_void_p, C.c_int]
        L.orc_out_norm.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p]
        L.orc_cfg_blend.argtypes = [C.c_void_p, C.c_void_p, C.c_long, C.c_float, C.c_void_p]
        L.orc_embed_frames.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.c_int, C.c_void_p]
        L.orc_shear_up.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int32, C.c_void_p]

    # generator -------------------------------------------------------------
    def rng_seed(self, seed: int) -> np.ndarray:
        st = np.zeros(4, np.uint64)
        self.L.orc_rng_seed(seed, _u64(st))
        return st

    def rng_seed_streams(self, seed: int, n: int) -> np.ndarray:
        st = np.zeros((n, 4), np.uint64)
        self.L.orc_rng_seed_streams(seed, n, _u64(st))
        return st

    def rng_next(self, st: np.ndarray) -> int:
        return int(self.L.orc_rng_next(_u64(st)))

    def randf(self, st: np.ndarray) -> float:
        return float(self.L.orc_randf(_u64(st)))

    # sampler ---------------------------------------------------------------
    def sample_token_r(self, r, logits, temp, top_k, top_p, min_p, exp_mode=0):
        logits = np.ascontiguousarray(logits, np.float32)
        d = Diag()
        tok = self.L.orc_sample_token_r(r, _p(logits), logits.size, temp, top_k, top_p, min_p,
                                        exp_mode, C.byref(d))
        return tok, d

    def sample_token(self, st, logits, temp, top_k, top_p, min_p, exp_mode=0):
        logits = np.ascontiguousarray(logits, np.float32)
        d = Diag()
        tok = self.L.orc_sample_token(_u64(st), _p(logits), logits.size, temp, top_k, top_p,
                                      min_p, exp_mode, C.byref(d))
        return tok, d

    def step(self, logits, params: Params, rng, hist=None, hist_pos=0, allow=None, delay_step=-1,
             exp_mode=1, diags=False, nthreads=0, row_stride=None):
        """One decode step; logits [S, C, V] (or [S*C, row_stride]); rng/hist updated in place."""
        S, Cb, V = logits.shape[0], logits.shape[1], logits.shape[-1]
        logits = np.ascontiguousarray(logits, np.float32)
        stride = V if row_stride is None else row_stride
        H = 0 if hist is None else hist.shape[-1]
        codes = np.zeros((S, Cb), np.int32)
        flags = np.zeros((S, Cb), np.int32)
        dg = (Diag * (S * Cb))() if diags else None
        aw = 0 if allow is None else allow.shape[-1]
        rc = self.L.orc_step(_p(logits), S, Cb, V, stride, C.byref(params), _u64(rng), _p(hist), H,
                             hist_pos, _p(allow), aw, delay_step, _p(codes), _p(flags), exp_mode,
                             dg, nthreads)
        if rc != 0:
            raise ValueError("orc_step rejected its arguments")
        return codes, flags, dg

    # head ------------------------------------------------------------------
    def head_softcap(self, W, rows_per_cb, n_cb, vocab, h, softcap=15.0, nthreads=0):
        W = np.ascontiguousarray(W, np.float32)
        h = np.ascontiguousarray(h, np.float32)
        B, D = h.shape
        out = np.zeros((B, n_cb, vocab), np.float32)
        self.L.orc_head_softcap(_p(W), rows_per_cb, n_cb, vocab, D, _p(h), B, softcap, _p(out),
                                nthreads)
        return out

    def out_norm(self, x, eps=1e-5, weight=None):
        """rms_norm_per_token over the rows of x ([n, dim] f32); returns a copy."""
        x = np.array(x, np.float32, copy=True, order="C")
        w = None if weight is None else np.ascontiguousarray(weight, np.float32)
        self.L.orc_out_norm(_p(x), x.shape[-1], x.size // x.shape[-1], eps, _p(w))
        return x

    def embed_frames(self, cb_tables, text_table, ids):
        """embedding_sum of frames ids [n][n_cb+1]; tables f32 row-major."""
        cb_tables = np.ascontiguousarray(cb_tables, np.float32)
        text_table = np.ascontiguousarray(text_table, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        n_cb, audio_vocab, dim = cb_tables.shape
        out = np.zeros((ids.shape[0], dim), np.float32)
        self.L.orc_embed_frames(_p(cb_tables), _p(text_table), n_cb, audio_vocab,
                                text_table.shape[0] - 1, dim, _p(ids), ids.shape[0], _p(out))
        return out

    def shear_up(self, codes, pad=1025):
        codes = np.ascontiguousarray(codes, np.int32)
        out = np.empty_like(codes)
        self.L.orc_shear_up(_p(codes), codes.shape[0], codes.shape[1], pad, _p(out))
        return out

    def cfg_blend(self, cond, uncond, scale):
        cond = np.ascontiguousarray(cond, np.float32)
        uncond = np.ascontiguousarray(uncond, np.float32)
        out = np.empty_like(cond)
        self.L.orc_cfg_blend(_p(cond), _p(uncond), cond.size, scale, _p(out))
        return out


class Reference:
    """The reference's own sources, compiled unmodified (oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            build()
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        self.L = L
        L.ref_rng_seed.argtypes = [C.c_uint64, C.POINTER(C.c_uint64)]
        L.ref_rng_next.argtypes = [C.POINTER(C.c_uint64)]
        L.ref_rng_next.restype = C.c_uint64
        L.ref_randf.argtypes = [C.POINTER(C.c_uint64)]
        L.ref_randf.restype = C.c_float
        L.ref_sample_token.argtypes = [C.POINTER(C.c_uint64), C.c_void_p, C.c_int, C.c_float,
                                       C.c_int, C.c_float, C.c_float]
        L.ref_sample_token.restype = C.c_int
        L.ref_linear_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                         C.c_void_p]
        L.ref_head_softcap.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                       C.c_int, C.c_float, C.c_void_p, C.c_int]
        L.ref_out_norm.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p]
        L.ref_write_codes.argtypes = [C.c_char_p, C.c_void_p, C.c_int, C.c_int]
        L.ref_write_codes.restype = C.c_int
        L.ref_embed_frames.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.c_int, C.c_void_p]
        L.ref_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_long, C.c_float, C.c_int,
                               C.c_float, C.c_float, C.c_float, C.c_int, C.POINTER(C.c_uint64),
                               C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int,
                               C.c_void_p, C.c_void_p, C.c_int]
        L.ref_step.restype = C.c_int
        L.ref_num_threads.restype = C.c_int

    def rng_seed(self, seed: int) -> np.ndarray:
        st = np.zeros(4, np.uint64)
        self.L.ref_rng_seed(seed, _u64(st))
        return st

    def rng_next(self, st) -> int:
        return int(self.L.ref_rng_next(_u64(st)))

    def randf(self, st) -> float:
        return float(self.L.ref_randf(_u64(st)))

    def sample_token(self, st, logits, temp, top_k, top_p, min_p) -> int:
        logits = np.ascontiguousarray(logits, np.float32)
        return int(self.L.ref_sample_token(_u64(st), _p(logits), logits.size, temp, top_k, top_p,
                                           min_p))

    def head_softcap(self, W, rows_per_cb, n_cb, vocab, h, softcap=15.0, nthreads=0):
        W = np.ascontiguousarray(W, np.float32)
        h = np.ascontiguousarray(h, np.float32)
        B, D = h.shape
        out = np.zeros((B, n_cb, vocab), np.float32)
        self.L.ref_head_softcap(_p(W), rows_per_cb, n_cb, vocab, D, _p(h), B, softcap, _p(out),
                                nthreads)
        return out

    def write_codes(self, stem, frames):
        """The reference writes `stem`.codes.bin (and prints a line)."""
        fr = np.ascontiguousarray(frames, np.int32)
        return self.L.ref_write_codes(stem.encode(), _p(fr), fr.shape[0], fr.shape[1])

    def embed_frames(self, cb_tables, text_table, ids):
        cb_tables = np.ascontiguousarray(cb_tables, np.float32)
        text_table = np.ascontiguousarray(text_table, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        n_cb, audio_vocab, dim = cb_tables.shape
        out = np.zeros((ids.shape[0], dim), np.float32)
        self.L.ref_embed_frames(_p(cb_tables), _p(text_table), n_cb, audio_vocab,
                                text_table.shape[0] - 1, dim, _p(ids), ids.shape[0], _p(out))
        return out

    def out_norm(self, x, eps=1e-5, weight=None):
        x = np.array(x, np.float32, copy=True, order="C")
        w = None if weight is None else np.ascontiguousarray(weight, np.float32)
        self.L.ref_out_norm(_p(x), x.shape[-1], x.size // x.shape[-1], eps, _p(w))
        return x

    def step(self, logits, params: Params, rng, hist=None, hist_pos=0, allow=None, delay_step=-1,
             nthreads=0, row_stride=None):
        S, Cb, V = logits.shape[0], logits.shape[1], logits.shape[-1]
        logits = np.ascontiguousarray(logits, np.float32)
        stride = V if row_stride is None else row_stride
        H = 0 if hist is None else hist.shape[-1]
        codes = np.zeros((S, Cb), np.int32)
        flags = np.zeros((S, Cb), np.int32)
        aw = 0 if allow is None else allow.shape[-1]
        rc = self.L.ref_step(_p(logits), S, Cb, V, stride, params.temperature, params.top_k,
                             params.top_p, params.min_p, params.repetition_penalty, params.pad_id,
                             _u64(rng), _p(hist), H, hist_pos, _p(allow), aw, delay_step,
                             _p(codes), _p(flags), nthreads)
        if rc != 0:
            raise ValueError("ref_step rejected its arguments")
        return codes, flags

    def num_threads(self) -> int:
        return int(self.L.ref_num_threads())


def gen_append(codes, frames, n_frames, eos_at, max_frames, codebook_size=1024, eoa_id=1024):
    """One generation step for a batch, as the reference's loop does it for one
    stream (src/zonos2_generate.cpp:214-226, :259-276): each sampled code is
    clamped to codebook_size - 1, a stream that has ended (an EOA code in its
    previous frame, or max_frames frames) takes no more frames, and a frame
    holding eoa_id ends its stream after being kept.  codes [S][n_cb];
    frames [S][max_frames][n_cb], n_frames [S], eos_at [S] are updated in place."""
    S = codes.shape[0]
    for s in range(S):
        if eos_at[s] >= 0 or n_frames[s] >= max_frames:
            continue
        f = [min(int(t), codebook_size - 1) for t in codes[s]]
        frames[s, n_frames[s]] = f
        if any(t == eoa_id for t in f):
            eos_at[s] = n_frames[s]
        n_frames[s] += 1
