"""The C-ABI library loads and exports every entry point include/*.h declares;
host-side argument checks and helpers.  CPU only: nothing here launches a kernel."""
import ctypes as C
import glob
import os
import re

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(zonos2cu_\w+)\s*\(", src))
    return names


def test_header_declares_the_boundary():
    names = declared_symbols()
    for must in ("zonos2cu_sample_token", "zonos2cu_sample_rows", "zonos2cu_head_softcap",
                 "zonos2cu_ctx_create", "zonos2cu_ctx_step"):
        assert must in names


def test_library_exports_every_declared_symbol(z2):
    L = z2.lib()
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, missing
    assert set(z2.EXPORTS) == declared_symbols()


def test_version_and_defaults(z2):
    assert b"sm_100a" in z2.lib().zonos2cu_version()
    p = z2.default_params()
    # Zonos2GenParams defaults (src/zonos2.h:245-252); the penalty is off by default
    assert abs(p.temperature - 0.7) < 1e-7 and p.top_k == 50
    assert abs(p.top_p - 0.9) < 1e-7 and abs(p.min_p - 0.02) < 1e-9
    assert p.repetition_penalty == 1.0 and p.pad_id == 1023


def test_host_seeding_matches_oracle(z2, oracle):
    for seed in (0, 42, 1234, 2**64 - 1):
        assert (z2.Xoshiro256(seed).s == oracle.rng_seed(seed)).all()


def _rows(z2, **over):
    args = dict(logits=1 << 20, S=4, Cb=9, V=1024, stride=1024, rng=1 << 21, hist=0, H=0, pos=0,
                allow=0, delay=-1, codes=1 << 22, flags=0)
    args.update(over)
    p = over.pop("params", None) or z2.SampleParams()
    return z2.lib().zonos2cu_sample_rows(args["logits"], args["S"], args["Cb"], args["V"],
                                         args["stride"], C.byref(p), args["rng"],
                                         args["hist"] or None, args["H"], args["pos"],
                                         args["allow"] or None, args["delay"], args["codes"],
                                         args["flags"] or None, None)


def test_sample_rows_rejects_bad_arguments(z2):
    E, U = z2.EINVAL, z2.EUNSUPPORTED
    assert _rows(z2, Cb=0) == E
    assert _rows(z2, Cb=17) == E
    assert _rows(z2, V=0) == E
    assert _rows(z2, V=1025) == U
    assert _rows(z2, stride=1000) == E
    assert _rows(z2, S=-1) == E
    assert _rows(z2, H=8, hist=0) == E                 # history length without a buffer
    assert _rows(z2, H=8, hist=1 << 23, pos=8) == E    # write position outside the ring
    assert _rows(z2, logits=0) == E
    assert _rows(z2, codes=0) == E
    assert _rows(z2, rng=(1 << 21) + 8) == E           # generator states not 16-byte aligned
    for bad in (dict(temperature=0.0), dict(temperature=float("nan")),
                dict(temperature=float("inf")), dict(top_p=float("nan")), dict(min_p=1.5),
                dict(min_p=float("nan")), dict(repetition_penalty=0.0), dict(pad_id=1024),
                dict(pad_id=-1)):
        p = z2.SampleParams()
        for k, v in bad.items():
            setattr(p, k, v)
        assert _rows(z2, params=p) == E, bad


def test_drop_in_rejects_undefined_reference_cases(z2):
    st = z2.Xoshiro256(1)
    row = np.zeros(1024, np.float32)
    L = z2.lib()
    u64 = st.s.ctypes.data_as(C.POINTER(C.c_uint64))
    assert L.zonos2cu_sample_token(u64, row.ctypes.data, 1024, 0.0, 50, 0.9, 0.02) == z2.EINVAL
    assert L.zonos2cu_sample_token(u64, row.ctypes.data, 1024, 0.7, 50, 0.9, 2.0) == z2.EINVAL
    assert L.zonos2cu_sample_token(u64, None, 1024, 0.7, 50, 0.9, 0.02) == z2.EINVAL
    assert L.zonos2cu_sample_token(u64, row.ctypes.data, 0, 0.7, 50, 0.9, 0.02) == z2.EINVAL


def test_head_rejects_bad_arguments(z2):
    L = z2.lib()
    ok = dict(W=1 << 20, dt=z2.BF16, rpc=1026, C=9, V=1024, D=2048, h=1 << 21, B=4, cap=15.0,
              out=1 << 22)

    def call(**o):
        a = dict(ok)
        a.update(o)
        return L.zonos2cu_head_softcap(a["W"], a["dt"], a["rpc"], a["C"], a["V"], a["D"], a["h"],
                                       a["B"], a["cap"], a["out"], None)
    assert call(rpc=1000) == z2.EINVAL
    assert call(C=0) == z2.EINVAL
    assert call(D=0) == z2.EINVAL
    assert call(W=0) == z2.EINVAL
    assert call(dt=7) == z2.EINVAL
    assert call(cap=float("nan")) == z2.EINVAL


def test_context_rejects_bad_dims(z2):
    L = z2.lib()
    h = C.c_void_p()
    for d in (z2.Dims(-1, 9, 1024, 0, 0, 0, 0), z2.Dims(4, 0, 1024, 0, 0, 0, 0),
              z2.Dims(4, 9, 0, 0, 0, 0, 0), z2.Dims(4, 9, 1024, -1, 0, 0, 0),
              z2.Dims(4, 9, 1024, 0, -3, 0, 0)):
        assert L.zonos2cu_ctx_create(0, C.byref(d), C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_ctx_destroy(None) == 0


def test_shard_range_matches_the_python_shard_arithmetic(z2):
    import sharding
    for n in (0, 1, 7, 4096, 32768, 32769, 100003):
        for ws in (1, 2, 3, 4, 7, 8):
            for r in range(ws):
                assert z2.shard_range(n, ws, r) == sharding.shard_range(n, ws, r), (n, ws, r)
    L = z2.lib()
    f, c = C.c_longlong(), C.c_longlong()
    assert L.zonos2cu_shard_range(10, 0, 0, C.byref(f), C.byref(c)) == z2.EINVAL
    assert L.zonos2cu_shard_range(10, 2, 2, C.byref(f), C.byref(c)) == z2.EINVAL
    assert L.zonos2cu_shard_range(-1, 2, 0, C.byref(f), C.byref(c)) == z2.EINVAL


def test_gather_and_comm_reject_bad_arguments(z2):
    """Checked before NCCL is touched (no GPU or NCCL needed)."""
    L = z2.lib()
    assert L.zonos2cu_gather_codes(None, 0, 1 << 20, 1, 8, 9, 1 << 21, None) == z2.EINVAL
    assert L.zonos2cu_gather_codes(1 << 12, 0, 1 << 20, -1, 8, 9, 1 << 21, None) == z2.EINVAL
    assert L.zonos2cu_gather_codes(1 << 12, 0, 1 << 20, 1, 8, 0, 1 << 21, None) == z2.EINVAL
    h = C.c_void_p()
    uid = bytes(128)
    assert L.zonos2cu_comm_create(0, 0, 0, uid, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create(0, 2, 2, uid, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create(0, 1, 0, None, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_destroy(None) == 0
    # the bounded set-up: the same checks, and a timeout of at least 1 ms
    assert L.zonos2cu_comm_create_timeout(0, 0, 0, uid, 1000, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create_timeout(0, 2, 2, uid, 1000, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create_timeout(0, 1, 0, None, 1000, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create_timeout(0, 1, 0, uid, 0, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_create_timeout(0, 1, 0, uid, -5, C.byref(h)) == z2.EINVAL
    assert L.zonos2cu_comm_abort(None) == 0


def test_push_gather_rejects_bad_arguments(z2):
    """The copy-engine collection's checks come before CUDA is touched."""
    L = z2.lib()
    p = C.c_void_p()
    hbuf = C.create_string_buffer(64)
    assert L.zonos2cu_ipc_alloc(0, 1024, None, hbuf) == z2.EINVAL
    assert L.zonos2cu_ipc_alloc(0, 1024, C.byref(p), None) == z2.EINVAL
    assert L.zonos2cu_ipc_alloc(0, 0, C.byref(p), hbuf) == z2.EINVAL
    assert L.zonos2cu_ipc_open(0, None, C.byref(p)) == z2.EINVAL
    assert L.zonos2cu_ipc_open(0, bytes(64), None) == z2.EINVAL
    assert L.zonos2cu_push_codes(None, -1, 9, None, 9, None) == z2.EINVAL
    assert L.zonos2cu_push_codes(None, 1, -1, None, 9, None) == z2.EINVAL
    assert L.zonos2cu_push_codes(1 << 20, 2, 9, 1 << 21, 8, None) == z2.EINVAL   # stride < block
    assert L.zonos2cu_push_codes(None, 2, 9, 1 << 21, 9, None) == z2.EINVAL
    assert L.zonos2cu_push_codes(1 << 20, 2, 9, None, 9, None) == z2.EINVAL
    assert L.zonos2cu_push_codes(None, 0, 9, None, 9, None) == 0
    assert L.zonos2cu_push_codes(None, 3, 0, None, 0, None) == 0
    assert L.zonos2cu_ipc_free(None) == 0
    assert L.zonos2cu_ipc_close(None) == 0
