"""zonos2cu_step_noalloc: the decode step for callers that may not allocate
device memory (their memory belongs to another framework's pool, or they
decode under real-time constraints).  It keeps its intermediate logits in a
fixed array inside the library; here it must give exactly what the two entry
points it stands for give -- zonos2cu_head_softcap into a caller buffer, then
zonos2cu_sample_rows -- on two calls in a row (the array is reused).

Collected after the small-case parity tests on purpose; it needs nothing from
the other tests.
"""
import ctypes as C

import numpy as np
import pytest


def _dev(x, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def test_noalloc_rejects_requests_beyond_its_array(z2):
    L = z2.lib()
    p = z2.SampleParams()
    big = z2.NOALLOC_MAX_LOGITS // (9 * 1024) + 1          # one stream too many
    rc = L.zonos2cu_step_noalloc(1 << 20, z2.BF16, 1024, 9, 1024, 2048, 1 << 21, big, 15.0,
                                 C.byref(p), 1 << 22, None, 0, 0, None, -1, 1 << 23, None, None)
    assert rc == z2.ETOOBIG


def test_noalloc_checks_sampler_arguments_before_any_launch(z2):
    """Invalid sampler arguments are rejected as zonos2cu_sample_rows rejects
    them -- with no stream at all, and before the head would be launched (the
    pointers here are never dereferenced, so no GPU is needed)."""
    L = z2.lib()
    bad_t = z2.SampleParams(temperature=0.0)
    bad_minp = z2.SampleParams(min_p=1.5)
    good = z2.SampleParams()
    W, h, rng, codes = 1 << 20, 1 << 21, 1 << 22, 1 << 23
    for S in (0, 3):
        for p in (bad_t, bad_minp):
            rc = L.zonos2cu_step_noalloc(W, z2.BF16, 1024, 9, 1024, 2048, h, S, 15.0, C.byref(p),
                                         rng, None, 0, 0, None, -1, codes, None, None)
            assert rc == z2.EINVAL, (S, rc)
            assert L.zonos2cu_sample_rows(256, S, 9, 1024, 1024, C.byref(p), rng, None, 0, 0,
                                          None, -1, codes, None, None) == z2.EINVAL
        # misaligned generator states, a history position outside the ring, too many codebooks
        for args in ((rng + 8, None, 0, 0, 9), (rng, 1 << 24, 16, 16, 9), (rng, None, 0, 0, 17)):
            r, hist, H, pos, ncb = args
            rc = L.zonos2cu_step_noalloc(W, z2.BF16, 1024, ncb, 1024, 2048, h, S, 15.0,
                                         C.byref(good), r, hist, H, pos, None, -1, codes, None,
                                         None)
            assert rc == z2.EINVAL, (S, args, rc)
    # n_streams = 0 with valid arguments launches nothing and succeeds
    assert L.zonos2cu_step_noalloc(W, z2.BF16, 1024, 9, 1024, 2048, h, 0, 15.0, C.byref(good),
                                   rng, None, 0, 0, None, -1, codes, None, None) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,S,H", [("bf16", 64, 96), ("f32", 3, 0)])
def test_noalloc_step_matches_head_then_sample(z2, oracle, cuda, dtype, S, H):
    import torch
    import workloads as W
    L = z2.lib()
    rs = np.random.default_rng(2024 + S)
    rpc = 1026
    Wf = rs.normal(0, 0.02, size=(9 * rpc, 2048)).astype(np.float32)
    if dtype == "bf16":
        dt, Wd = z2.BF16, W.to_bf16_bits(Wf)
    else:
        dt, Wd = z2.F32, Wf
    W_dev = _dev(Wd, cuda)
    p = z2.SampleParams(0.8, 50, 0.95, 0.02, 1.2, 1023)
    rng0 = oracle.rng_seed_streams(77, S)
    hist0 = rs.integers(0, 1024, size=(S, 9, max(H, 1)), dtype=np.int32)
    allow = W.pack_bits(rs.random((S, 1024)) < 0.8)
    rng_a, rng_b = _dev(rng0.view(np.int64), cuda), _dev(rng0.view(np.int64), cuda)
    hist_a, hist_b = _dev(hist0, cuda), _dev(hist0, cuda)
    allow_d = _dev(allow.view(np.int32), cuda)
    codes_a = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    codes_b = torch.zeros_like(codes_a)
    flags_a, flags_b = torch.zeros_like(codes_a), torch.zeros_like(codes_a)
    logits = torch.empty((S, 9, 1024), dtype=torch.float32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):                                     # two calls in a row
        h = rs.normal(0, 1, size=(S, 2048)).astype(np.float32)
        hd = _dev(W.to_bf16_bits(h) if dtype == "bf16" else h, cuda)
        hist_arg_a = hist_a.data_ptr() if H else None
        hist_arg_b = hist_b.data_ptr() if H else None
        rc = L.zonos2cu_step_noalloc(W_dev.data_ptr(), dt, rpc, 9, 1024, 2048, hd.data_ptr(), S,
                                     15.0, C.byref(p), rng_a.data_ptr(), hist_arg_a, H,
                                     call % max(H, 1), allow_d.data_ptr(), call,
                                     codes_a.data_ptr(), flags_a.data_ptr(), stream)
        assert rc == 0, z2.last_error()
        z2.head_softcap(W_dev, dt, rpc, 9, 1024, hd, logits)
        z2.sample_rows(logits, p, rng_b, codes_b, flags=flags_b, hist=hist_b if H else None,
                       hist_pos=call % max(H, 1), allow=allow_d, delay_step=call)
        torch.cuda.synchronize()
        assert (codes_a == codes_b).all().item(), call
        assert (flags_a == flags_b).all().item()
        assert (rng_a == rng_b).all().item()
        assert (hist_a == hist_b).all().item()
    assert z2.device_error() == 0
