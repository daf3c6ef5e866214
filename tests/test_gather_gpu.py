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
