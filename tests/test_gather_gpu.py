"""The codes gather to one rank (zonos2cu_gather_codes) through the C ABI, on a
one-rank NCCL communicator made by the library: the root's output must be its
own block, step-major within the block, for whole and partial rings.  The
several-rank shard arithmetic is covered on CPU (test_capi, test_sharding)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gather_codes_one_rank_communicator(z2, cuda):
    import torch
    uid = z2.comm_unique_id()
    comm = z2.Comm(0, 1, 0, uid)
    try:
        S, Cb = 777, 9
        ring = torch.randint(0, 1024, (32, S, Cb), dtype=torch.int32, device=cuda)
        for n_steps in (1, 20, 32):
            out = torch.full((n_steps * S * Cb,), -5, dtype=torch.int32, device=cuda)
            comm.gather_codes(0, ring, n_steps, S, Cb, out)
            torch.cuda.synchronize()
            assert torch.equal(out.view(n_steps, S, Cb), ring[:n_steps])
        # in place: the root's own block already where it belongs
        comm.gather_codes(0, ring, 32, S, Cb, ring)
        torch.cuda.synchronize()
        with pytest.raises(z2.Zonos2cuError):
            comm.gather_codes(1, ring, 1, S, Cb, ring)      # root outside the communicator
    finally:
        comm.close()
    assert z2.device_error() == 0


def test_gather_codes_non_blocking_communicator(z2, cuda):
    """The bounded set-up (zonos2cu_comm_create_timeout): a one-rank
    communicator set up without blocking gathers like the blocking one, and its
    destroy flushes it (finalise, polled) before freeing it."""
    import torch
    comm = z2.Comm(0, 1, 0, z2.comm_unique_id(), timeout_ms=30000)
    try:
        S, Cb = 300, 9
        ring = torch.randint(0, 1024, (8, S, Cb), dtype=torch.int32, device=cuda)
        out = torch.full((8 * S * Cb,), -5, dtype=torch.int32, device=cuda)
        comm.gather_codes(0, ring, 8, S, Cb, out)
        torch.cuda.synchronize()
        assert torch.equal(out.view(8, S, Cb), ring)
    finally:
        comm.close()


_ABSENT_PEER = r'''
import sys, time
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import zonos2cu as z2
uid = z2.comm_unique_id()
t0 = time.monotonic()
try:
    z2.Comm(0, 2, 0, uid, timeout_ms=3000)    # rank 1 never starts
    print("created"); sys.exit(1)
except z2.Zonos2cuError as e:
    waited = time.monotonic() - t0
    print("refused", e.code, round(waited, 2), z2.last_error())
    assert e.code == z2.ENCCL and 2.9 <= waited < 60, (e.code, waited)
c = z2.Comm(0, 1, 0, z2.comm_unique_id(), timeout_ms=30000)   # the process carries on
c.close()
print("ok")
'''


def test_comm_set_up_times_out_when_a_rank_never_joins(z2, cuda, tmp_path):
    """A two-rank set-up whose second rank never starts (the failure made on the
    host: nothing runs on the GPU) ends with ZONOS2CU_ENCCL after the timeout,
    aborted, instead of waiting for good; the process then makes a working
    communicator.  Run in a child process with NVLS off."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", _ABSENT_PEER, repo,
                        os.path.join(repo, "zonos2.cpp_b200")],
                       env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout, r.stderr[-2000:])
