"""The copy-engine collection through the C ABI on one GPU.  The parent
allocates the root's buffer (zonos2cu_ipc_alloc); a child process, standing in
for another rank, maps it (zonos2cu_ipc_open), pushes its strided block of
steps into its columns (zonos2cu_push_codes) and unmaps it; the parent's
buffer must then hold those codes and nothing else.  (IPC needs two processes,
not two GPUs; the several-GPU path is bench.py's multi_gpu_check.)"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_STEPS, COUNT, FIRST, N = 5, 300, 200, 1000

_CHILD = r'''
import sys
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import torch
import zonos2cu as z2
n_steps, count, first, n = (int(x) for x in sys.argv[4:8])
dst = z2.ipc_open(0, bytes.fromhex(sys.argv[3]))
src = (torch.arange(n_steps * count * 9, dtype=torch.int32, device="cuda:0") + 7).view(
    n_steps, count, 9)
z2.push_codes(src, n_steps, count * 9, dst + 4 * first * 9, n * 9)
torch.cuda.synchronize()
z2.ipc_close(dst)
print("pushed")
'''


def test_push_codes_into_another_process_buffer(z2, cuda):
    import torch
    total = N_STEPS * N * 9
    ptr, handle = z2.ipc_alloc(0, 4 * total)
    try:
        minus = torch.full((total,), -1, dtype=torch.int32, device=cuda)
        z2.push_codes(minus, 1, total, ptr, total)   # a local copy: the buffer starts at -1
        torch.cuda.synchronize()
        here = os.path.dirname(os.path.abspath(__file__))
        repo = os.path.dirname(here)
        r = subprocess.run([sys.executable, "-c", _CHILD, repo, os.path.join(repo, "zonos2.cpp_b200"),
                            handle.hex(), str(N_STEPS), str(COUNT), str(FIRST), str(N)],
                           capture_output=True, text=True, timeout=180)
        assert r.returncode == 0 and "pushed" in r.stdout, (r.stdout, r.stderr[-2000:])
        out = torch.empty((total,), dtype=torch.int32, device=cuda)
        z2.push_codes(ptr, 1, total, out.data_ptr(), total)
        torch.cuda.synchronize()
        got = out.view(N_STEPS, N, 9).cpu().numpy()
        want = np.full((N_STEPS, N, 9), -1, np.int32)
        want[:, FIRST:FIRST + COUNT] = (np.arange(N_STEPS * COUNT * 9, dtype=np.int32) + 7).reshape(
            N_STEPS, COUNT, 9)
        assert (got == want).all()
    finally:
        z2.ipc_free(ptr)
    assert z2.device_error() == 0
