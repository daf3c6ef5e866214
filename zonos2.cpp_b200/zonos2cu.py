"""Python mirror of zonos2.cpp's decode-step output path over the CUDA library.

Thin ctypes bindings to ``libzonos2cu.so`` (the C ABI in
``include/zonos2_cuda.h``).  The names follow the reference:

* ``Xoshiro256`` -- the generator of src/zonos2_generate.cpp:11-33 (state
  words in host memory; seeding and stepping match bit for bit);
* ``sample_token(rng, logits, vocab_size, temp, top_k, top_p, min_p)`` -- the
  drop-in for src/zonos2_generate.cpp:36-93, sampled on the current GPU;
* ``sample_rows`` / ``head_softcap`` -- the batched device-pointer entry points;
* ``Context`` -- device-resident decode state for a shard of streams.

Device buffers are passed as torch CUDA tensors (PyTorch is only the memory
and stream plumbing here).  There is no CPU fallback: if the library is
missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzonos2cu.so")

OK, EINVAL, ECUDA, ENOMEM, ESTATE, EUNSUPPORTED, EDEVICE, ETOOBIG, ENCCL = (
    0, -1, -2, -3, -4, -5, -6, -7, -8)
NOALLOC_MAX_LOGITS = 64 * 9 * 1024
FLAG_ALL_MASKED, FLAG_NONFINITE = 1, 2
F32, BF16 = 0, 1

EXPORTS = (
    "zonos2cu_default_params", "zonos2cu_version", "zonos2cu_last_error", "zonos2cu_rng_seed",
    "zonos2cu_sample_token", "zonos2cu_sample_rows", "zonos2cu_head_softcap",
    "zonos2cu_ctx_create", "zonos2cu_ctx_destroy", "zonos2cu_set_head", "zonos2cu_set_history",
    "zonos2cu_get_history", "zonos2cu_set_rng", "zonos2cu_get_rng", "zonos2cu_set_allow",
    "zonos2cu_ctx_sample", "zonos2cu_ctx_sample_host", "zonos2cu_ctx_step",
    "zonos2cu_ctx_step_host", "zonos2cu_ctx_stream", "zonos2cu_device_error",
    "zonos2cu_step_noalloc", "zonos2cu_set_out_norm", "zonos2cu_set_cfg",
    "zonos2cu_gen_begin", "zonos2cu_gen_end", "zonos2cu_gen_read", "zonos2cu_gen_next_input",
    "zonos2cu_gen_shear_up", "zonos2cu_set_embeddings", "zonos2cu_gen_embed_next",
    "zonos2cu_embed_frames", "zonos2cu_write_codes_bin", "zonos2cu_shard_range",
    "zonos2cu_comm_unique_id", "zonos2cu_comm_create", "zonos2cu_comm_destroy",
    "zonos2cu_gather_codes", "zonos2cu_comm_create_timeout", "zonos2cu_comm_abort",
    "zonos2cu_ipc_alloc", "zonos2cu_ipc_free", "zonos2cu_ipc_open", "zonos2cu_ipc_close",
    "zonos2cu_push_codes",
)


class Zonos2cuError(RuntimeError):
    def __init__(self, code: int, what: str):
        names = {EINVAL: "EINVAL", ECUDA: "ECUDA", ENOMEM: "ENOMEM", ESTATE: "ESTATE",
                 EUNSUPPORTED: "EUNSUPPORTED", EDEVICE: "EDEVICE", ETOOBIG: "ETOOBIG",
                 ENCCL: "ENCCL"}
        msg = f"{what} failed: {names.get(code, code)}"
        detail = last_error() if _lib is not None else ""
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)
        self.code = code


class SampleParams(C.Structure):
    """zonos2cu_sample_params; defaults follow Zonos2GenParams (src/zonos2.h:244-254)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("min_p", C.c_float), ("repetition_penalty", C.c_float), ("pad_id", C.c_int)]

    def __init__(self, temperature=0.7, top_k=50, top_p=0.9, min_p=0.02, repetition_penalty=1.0,
                 pad_id=1023):
        super().__init__(temperature, top_k, top_p, min_p, repetition_penalty, pad_id)


class Dims(C.Structure):
    _fields_ = [("n_streams", C.c_int), ("n_cb", C.c_int), ("vocab", C.c_int), ("dim", C.c_int),
                ("hist_len", C.c_int), ("seed", C.c_uint64), ("first_stream", C.c_uint64)]


_lib = None


def lib() -> C.CDLL:
    """Load libzonos2cu.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() or make -C "
                          f"{HERE}")
    L = C.CDLL(LIB_PATH)
    vp, i, f, ll, u64p = C.c_void_p, C.c_int, C.c_float, C.c_longlong, C.POINTER(C.c_uint64)
    sig = {
        "zonos2cu_default_params": (None, [C.POINTER(SampleParams)]),
        "zonos2cu_version": (C.c_char_p, []),
        "zonos2cu_last_error": (C.c_char_p, []),
        "zonos2cu_rng_seed": (None, [C.c_uint64, u64p]),
        "zonos2cu_sample_token": (i, [u64p, vp, i, f, i, f, f]),
        "zonos2cu_sample_rows": (i, [vp, i, i, i, ll, C.POINTER(SampleParams), vp, vp, i, i, vp,
                                     i, vp, vp, vp]),
        "zonos2cu_head_softcap": (i, [vp, i, i, i, i, i, vp, i, f, vp, vp]),
        "zonos2cu_ctx_create": (i, [i, C.POINTER(Dims), C.POINTER(vp)]),
        "zonos2cu_ctx_destroy": (i, [vp]),
        "zonos2cu_set_head": (i, [vp, vp, i, i]),
        "zonos2cu_set_history": (i, [vp, vp, i]),
        "zonos2cu_get_history": (i, [vp, vp, C.POINTER(i)]),
        "zonos2cu_set_rng": (i, [vp, vp]),
        "zonos2cu_set_out_norm": (i, [vp, i, vp, f]),
        "zonos2cu_set_cfg": (i, [vp, i, f]),
        "zonos2cu_gen_begin": (i, [vp, i, i, i, i]),
        "zonos2cu_gen_end": (i, [vp]),
        "zonos2cu_gen_read": (i, [vp, vp, vp, vp]),
        "zonos2cu_gen_next_input": (vp, [vp]),
        "zonos2cu_gen_shear_up": (i, [vp, vp, vp]),
        "zonos2cu_set_embeddings": (i, [vp, vp, vp, i, i]),
        "zonos2cu_gen_embed_next": (i, [vp, vp, vp]),
        "zonos2cu_embed_frames": (i, [vp, vp, i, i, i, i, vp, i, vp, vp]),
        "zonos2cu_write_codes_bin": (i, [C.c_char_p, vp, i, i]),
        "zonos2cu_get_rng": (i, [vp, vp]),
        "zonos2cu_set_allow": (i, [vp, vp]),
        "zonos2cu_ctx_sample": (i, [vp, vp, ll, C.POINTER(SampleParams), i, vp, vp, vp]),
        "zonos2cu_ctx_sample_host": (i, [vp, vp, ll, C.POINTER(SampleParams), i, vp, vp]),
        "zonos2cu_ctx_step": (i, [vp, vp, i, C.POINTER(SampleParams), i, vp, vp, vp, vp]),
        "zonos2cu_ctx_step_host": (i, [vp, vp, i, C.POINTER(SampleParams), i, vp, vp]),
        "zonos2cu_ctx_stream": (vp, [vp]),
        "zonos2cu_device_error": (i, []),
        "zonos2cu_step_noalloc": (i, [vp, i, i, i, i, i, vp, i, f, C.POINTER(SampleParams), vp,
                                      vp, i, i, vp, i, vp, vp, vp]),
        "zonos2cu_shard_range": (i, [ll, i, i, C.POINTER(ll), C.POINTER(ll)]),
        "zonos2cu_comm_unique_id": (i, [C.c_char_p]),
        "zonos2cu_comm_create": (i, [i, i, i, C.c_char_p, C.POINTER(vp)]),
        "zonos2cu_comm_destroy": (i, [vp]),
        "zonos2cu_comm_create_timeout": (i, [i, i, i, C.c_char_p, i, C.POINTER(vp)]),
        "zonos2cu_comm_abort": (i, [vp]),
        "zonos2cu_gather_codes": (i, [vp, i, vp, i, ll, i, vp, vp]),
        "zonos2cu_ipc_alloc": (i, [i, ll, C.POINTER(vp), C.c_char_p]),
        "zonos2cu_ipc_free": (i, [vp]),
        "zonos2cu_ipc_open": (i, [i, C.c_char_p, C.POINTER(vp)]),
        "zonos2cu_ipc_close": (i, [vp]),
        "zonos2cu_push_codes": (i, [vp, i, ll, vp, ll, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    s = lib().zonos2cu_last_error()
    return s.decode() if s else ""


def _check(rc: int, what: str) -> int:
    if rc < 0:
        raise Zonos2cuError(rc, what)
    return rc


def _ptr(t) -> int | None:
    """Device (or host) address of a torch tensor / numpy array, None for None."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def default_params() -> SampleParams:
    p = SampleParams()
    lib().zonos2cu_default_params(C.byref(p))
    return p


class Xoshiro256:
    """The reference's generator (src/zonos2_generate.cpp:11-33); ``s`` are its
    four state words, seeded by the library as the reference seeds them."""

    def __init__(self, seed: int = 42):
        self.s = np.zeros(4, np.uint64)
        lib().zonos2cu_rng_seed(C.c_uint64(seed), self.s.ctypes.data_as(C.POINTER(C.c_uint64)))


def sample_token(rng: Xoshiro256, logits, vocab_size: int, temp: float, top_k: int,
                 top_p: float, min_p: float) -> int:
    """Drop-in for sample_token (src/zonos2_generate.cpp:36-37): one row of host
    logits sampled on the current GPU; ``rng`` advances by one draw."""
    row = np.ascontiguousarray(np.asarray(logits, np.float32)[:vocab_size])
    rc = lib().zonos2cu_sample_token(rng.s.ctypes.data_as(C.POINTER(C.c_uint64)),
                                     row.ctypes.data, vocab_size, temp, top_k, top_p, min_p)
    return _check(rc, "zonos2cu_sample_token")


def sample_rows(logits, params: SampleParams, rng, codes, *, flags=None, hist=None, hist_pos=0,
                allow=None, delay_step=-1, n_streams=None, n_cb=None, vocab=None,
                row_stride=None, stream=None) -> None:
    """One batched step.  logits: CUDA f32 [S, C, V] (or give the sizes and a
    row stride); rng: CUDA int64/uint64 [S, 4]; codes/flags: CUDA int32 [S, C];
    hist: CUDA int32 [S, C, H] or None; allow: CUDA int32/uint32 [S, ceil(V/32)]."""
    S = logits.shape[0] if n_streams is None else n_streams
    Cb = logits.shape[1] if n_cb is None else n_cb
    V = logits.shape[-1] if vocab is None else vocab
    stride = logits.shape[-1] if row_stride is None else row_stride
    H = 0 if hist is None else hist.shape[-1]
    rc = lib().zonos2cu_sample_rows(_ptr(logits), S, Cb, V, stride, C.byref(params), _ptr(rng),
                                    _ptr(hist), H, hist_pos, _ptr(allow), delay_step, _ptr(codes),
                                    _ptr(flags), _stream(stream))
    _check(rc, "zonos2cu_sample_rows")


def head_softcap(W, dtype: int, rows_per_cb: int, n_cb: int, vocab: int, hidden, out,
                 softcap: float = 15.0, stream=None) -> None:
    """logits[b, c, v] = softcap * tanh(W[c*rows_per_cb + v] . hidden[b] / softcap)."""
    B, D = hidden.shape
    rc = lib().zonos2cu_head_softcap(_ptr(W), dtype, rows_per_cb, n_cb, vocab, D, _ptr(hidden), B,
                                     softcap, _ptr(out), _stream(stream))
    _check(rc, "zonos2cu_head_softcap")


def step_noalloc(W, dtype: int, rows_per_cb: int, n_cb: int, vocab: int, hidden, params,
                 rng, codes, *, flags=None, hist=None, hist_pos=0, allow=None, delay_step=-1,
                 softcap: float = 15.0, stream=None) -> None:
    """Head + softcap + sampler with the logits in the library's fixed array
    (no device allocation; at most NOALLOC_MAX_LOGITS logits per call)."""
    S, D = hidden.shape
    H = 0 if hist is None else hist.shape[-1]
    rc = lib().zonos2cu_step_noalloc(_ptr(W), dtype, rows_per_cb, n_cb, vocab, D, _ptr(hidden), S,
                                     softcap, C.byref(params), _ptr(rng), _ptr(hist), H, hist_pos,
                                     _ptr(allow), delay_step, _ptr(codes), _ptr(flags),
                                     _stream(stream))
    _check(rc, "zonos2cu_step_noalloc")


def shard_range(n_streams: int, n_ranks: int, rank: int) -> tuple[int, int]:
    """(first global stream, number of streams) of `rank`'s slice."""
    first, count = C.c_longlong(), C.c_longlong()
    _check(lib().zonos2cu_shard_range(n_streams, n_ranks, rank, C.byref(first), C.byref(count)),
           "zonos2cu_shard_range")
    return first.value, count.value


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes), made on the job's first rank."""
    buf = C.create_string_buffer(128)
    _check(lib().zonos2cu_comm_unique_id(buf), "zonos2cu_comm_unique_id")
    return buf.raw


class Comm:
    """An NCCL communicator made by the library (zonos2cu_comm_create); every
    rank creates it collectively with the id rank 0 made."""

    def __init__(self, device: int, n_ranks: int, rank: int, uid: bytes,
                 timeout_ms: int | None = None):
        """timeout_ms: set up without blocking and abort if not every rank joins
        in time (zonos2cu_comm_create_timeout); None: NCCL's blocking set-up."""
        if len(uid) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        h = C.c_void_p()
        if timeout_ms is None:
            _check(lib().zonos2cu_comm_create(device, n_ranks, rank, uid, C.byref(h)),
                   "zonos2cu_comm_create")
        else:
            _check(lib().zonos2cu_comm_create_timeout(device, n_ranks, rank, uid, timeout_ms,
                                                      C.byref(h)), "zonos2cu_comm_create_timeout")
        self.h, self.n_ranks, self.rank = h, n_ranks, rank

    def gather_codes(self, root: int, codes, n_steps: int, n_streams: int, n_cb: int, out=None,
                     stream=None) -> None:
        """Rank `root` receives every rank's [n_steps][count][n_cb] block in rank order."""
        _check(lib().zonos2cu_gather_codes(self.h, root, _ptr(codes), n_steps, n_streams, n_cb,
                                           _ptr(out), _stream(stream)), "zonos2cu_gather_codes")

    def close(self) -> None:
        if self.h:
            h, self.h = self.h, C.c_void_p()
            _check(lib().zonos2cu_comm_destroy(h), "zonos2cu_comm_destroy")

    def abort(self) -> None:
        if self.h:
            h, self.h = self.h, C.c_void_p()
            _check(lib().zonos2cu_comm_abort(h), "zonos2cu_comm_abort")


def ipc_alloc(device: int, nbytes: int):
    """(device address, 64-byte handle) of a buffer other processes can map."""
    p = C.c_void_p()
    buf = C.create_string_buffer(64)
    _check(lib().zonos2cu_ipc_alloc(device, nbytes, C.byref(p), buf), "zonos2cu_ipc_alloc")
    return p.value, buf.raw


def ipc_free(ptr: int) -> None:
    _check(lib().zonos2cu_ipc_free(ptr), "zonos2cu_ipc_free")


def ipc_open(device: int, handle: bytes) -> int:
    """This process's address of another process's ipc_alloc buffer."""
    if len(handle) != 64:
        raise ValueError("a CUDA IPC handle is 64 bytes")
    p = C.c_void_p()
    _check(lib().zonos2cu_ipc_open(device, handle, C.byref(p)), "zonos2cu_ipc_open")
    return p.value


def ipc_close(ptr: int) -> None:
    _check(lib().zonos2cu_ipc_close(ptr), "zonos2cu_ipc_close")


def push_codes(codes, n_steps: int, elems_per_step: int, dst: int, dst_stride: int,
               stream=None) -> None:
    """n_steps contiguous blocks of elems_per_step int32 codes to dst + k * dst_stride
    (elements; dst e.g. an ipc_open address) on `stream`."""
    _check(lib().zonos2cu_push_codes(_ptr(codes), n_steps, elems_per_step, dst, dst_stride,
                                     _stream(stream)), "zonos2cu_push_codes")


def device_error() -> int:
    return _check(lib().zonos2cu_device_error(), "zonos2cu_device_error")


@dataclass
class _Shape:
    n_streams: int
    n_cb: int
    vocab: int
    dim: int
    hist_len: int


class Context:
    """Device-resident decode state for one shard of streams (zonos2cu_ctx)."""

    def __init__(self, device: int, n_streams: int, n_cb: int = 9, vocab: int = 1024,
                 dim: int = 0, hist_len: int = 0, seed: int = 42, first_stream: int = 0):
        d = Dims(n_streams, n_cb, vocab, dim, hist_len, seed, first_stream)
        h = C.c_void_p()
        _check(lib().zonos2cu_ctx_create(device, C.byref(d), C.byref(h)), "zonos2cu_ctx_create")
        self.h = h
        self.shape = _Shape(n_streams, n_cb, vocab, dim, hist_len)

    def close(self) -> None:
        if self.h:
            lib().zonos2cu_ctx_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().zonos2cu_ctx_stream(self.h)

    def set_head(self, W: np.ndarray, dtype: int, rows_per_cb: int) -> None:
        W = np.ascontiguousarray(W)
        _check(lib().zonos2cu_set_head(self.h, W.ctypes.data, dtype, rows_per_cb), "set_head")

    def set_history(self, hist: np.ndarray, hist_pos: int) -> None:
        hist = np.ascontiguousarray(hist, np.int32)
        _check(lib().zonos2cu_set_history(self.h, hist.ctypes.data, hist_pos), "set_history")

    def get_history(self):
        s = self.shape
        hist = np.zeros((s.n_streams, s.n_cb, s.hist_len), np.int32)
        pos = C.c_int()
        _check(lib().zonos2cu_get_history(self.h, hist.ctypes.data, C.byref(pos)), "get_history")
        return hist, pos.value

    def set_rng(self, st: np.ndarray) -> None:
        st = np.ascontiguousarray(st, np.uint64)
        _check(lib().zonos2cu_set_rng(self.h, st.ctypes.data), "set_rng")

    def get_rng(self) -> np.ndarray:
        st = np.zeros((self.shape.n_streams, 4), np.uint64)
        _check(lib().zonos2cu_get_rng(self.h, st.ctypes.data), "get_rng")
        return st

    def set_allow(self, bits) -> None:
        if bits is None:
            _check(lib().zonos2cu_set_allow(self.h, None), "set_allow")
            return
        bits = np.ascontiguousarray(bits, np.uint32)
        _check(lib().zonos2cu_set_allow(self.h, bits.ctypes.data), "set_allow")

    def set_out_norm(self, weight=None, eps: float = 1e-5, enable: bool = True) -> None:
        """The output RMSNorm ahead of the head (weight [dim] f32 or None)."""
        w = None if weight is None else np.ascontiguousarray(weight, np.float32)
        _check(lib().zonos2cu_set_out_norm(self.h, int(enable),
                                           None if w is None else w.ctypes.data,
                                           C.c_float(eps)), "set_out_norm")

    def set_cfg(self, scale: float, enable: bool = True) -> None:
        """Guidance blend; steps then take 2 * n_streams hidden rows (2s cond, 2s+1 uncond)."""
        _check(lib().zonos2cu_set_cfg(self.h, int(enable), C.c_float(scale)), "set_cfg")

    # ---- generation loop
    def gen_begin(self, max_frames: int, eoa_id: int = 1024, audio_pad_id: int = 1025,
                  text_pad_id: int = 519) -> None:
        _check(lib().zonos2cu_gen_begin(self.h, max_frames, eoa_id, audio_pad_id, text_pad_id),
               "gen_begin")
        self._max_frames = max_frames

    def gen_end(self) -> None:
        _check(lib().zonos2cu_gen_end(self.h), "gen_end")

    def gen_read(self):
        """(frames [S][max_frames][n_cb], n_frames [S], eos_at [S]) as numpy arrays."""
        s = self.shape
        frames = np.zeros((s.n_streams, self._max_frames, s.n_cb), np.int32)
        nf = np.zeros(s.n_streams, np.int32)
        eos = np.zeros(s.n_streams, np.int32)
        _check(lib().zonos2cu_gen_read(self.h, frames.ctypes.data, nf.ctypes.data,
                                       eos.ctypes.data), "gen_read")
        return frames, nf, eos

    def gen_next_input_ptr(self) -> int:
        return lib().zonos2cu_gen_next_input(self.h) or 0

    def gen_shear_up(self, out, stream=None) -> None:
        _check(lib().zonos2cu_gen_shear_up(self.h, _ptr(out), _stream(stream)), "gen_shear_up")

    def set_embeddings(self, codebook_tables, text_table) -> None:
        cb = np.ascontiguousarray(codebook_tables, np.float32)
        tx = np.ascontiguousarray(text_table, np.float32)
        _check(lib().zonos2cu_set_embeddings(self.h, cb.ctypes.data, tx.ctypes.data, cb.shape[1],
                                             tx.shape[0] - 1), "set_embeddings")

    def gen_embed_next(self, out, stream=None) -> None:
        _check(lib().zonos2cu_gen_embed_next(self.h, _ptr(out), _stream(stream)),
               "gen_embed_next")

    def sample(self, logits, params: SampleParams, codes, flags=None, delay_step=-1,
               row_stride=None, stream=None) -> None:
        """Device step on ``stream`` (default: torch's current stream)."""
        stride = logits.shape[-1] if row_stride is None else row_stride
        rc = lib().zonos2cu_ctx_sample(self.h, _ptr(logits), stride, C.byref(params), delay_step,
                                       _ptr(codes), _ptr(flags), _stream(stream))
        _check(rc, "zonos2cu_ctx_sample")

    def sample_host(self, logits: np.ndarray, params: SampleParams, codes: np.ndarray,
                    flags: np.ndarray | None = None, delay_step=-1, row_stride=None) -> None:
        stride = logits.shape[-1] if row_stride is None else row_stride
        rc = lib().zonos2cu_ctx_sample_host(self.h, _ptr(logits), stride, C.byref(params),
                                            delay_step, _ptr(codes), _ptr(flags))
        _check(rc, "zonos2cu_ctx_sample_host")

    def step(self, hidden, dtype: int, params: SampleParams, codes, flags=None, delay_step=-1,
             logits_out=None, stream=None) -> None:
        rc = lib().zonos2cu_ctx_step(self.h, _ptr(hidden), dtype, C.byref(params), delay_step,
                                     _ptr(codes), _ptr(flags), _ptr(logits_out), _stream(stream))
        _check(rc, "zonos2cu_ctx_step")

    def step_host(self, hidden, dtype: int, params: SampleParams, codes, flags=None,
                  delay_step=-1) -> None:
        rc = lib().zonos2cu_ctx_step_host(self.h, _ptr(hidden), dtype, C.byref(params),
                                          delay_step, _ptr(codes), _ptr(flags))
        _check(rc, "zonos2cu_ctx_step_host")


def embed_frames(codebook_tables, text_table, ids, out, stream=None) -> None:
    """embedding_sum on device buffers: tables [n_cb][audio_vocab][dim] and
    [text_vocab+1][dim] f32, ids [n][n_cb+1] int32, out [n][dim] f32."""
    n_cb, audio_vocab, dim = codebook_tables.shape
    _check(lib().zonos2cu_embed_frames(_ptr(codebook_tables), _ptr(text_table), n_cb, audio_vocab,
                                       text_table.shape[0] - 1, dim, _ptr(ids), ids.shape[0],
                                       _ptr(out), _stream(stream)), "zonos2cu_embed_frames")


def write_codes_bin(path: str, frames) -> None:
    """frames [n_frames][n_cb] int32 -> the reference's codes.bin format."""
    fr = np.ascontiguousarray(frames, np.int32)
    _check(lib().zonos2cu_write_codes_bin(path.encode(), fr.ctypes.data if fr.size else None,
                                          fr.shape[0], fr.shape[1]), "zonos2cu_write_codes_bin")
