"""Seeded shapes of the output head through the C ABI (zonos2cu_head_softcap).

bf16 (tcgen05 kernels): codebooks 1-9, vocab a multiple of 64 up to 1024, rows
per codebook >= vocab (the EOA/PAD rows of output.bin skipped), dim a multiple of
64, batches across the one-SM and pair kernels, the softcap on or off; against a
torch f32 product of the same bf16 values (f32 summation order only: <= 1e-3).
f32 (the f64-accumulating GEMV): odd dims and vocabularies (the scalar path)
and aligned ones (the vector path); against the oracle's head within the
reference's own sequential-f32 error bound.  Shapes the bf16 kernels do not
implement must be refused with ZONOS2CU_EUNSUPPORTED, not computed.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _shape_bf16(rs):
    n_cb = int(rs.choice([1, 2, 9]))
    vocab = int(64 * rs.integers(1, 17))
    rpc = vocab + int(rs.choice([0, 0, 2, 64]))
    dim = int(64 * rs.choice([1, 2, 3, 8, 32]))
    B = int(rs.choice([1, 5, 64, 130, 256, 300, 513, int(rs.integers(1, 900))]))
    cap = float(rs.choice([15.0, 15.0, 0.0, 4.0]))
    return n_cb, vocab, rpc, dim, B, cap


@pytest.mark.parametrize("chunk", range(4))
def test_head_bf16_shapes(z2, cuda, chunk):
    import torch
    rs = np.random.default_rng(500 + chunk)
    g = torch.Generator(device=cuda)
    g.manual_seed(500 + chunk)
    for case in range(10):
        n_cb, vocab, rpc, dim, B, cap = _shape_bf16(rs)
        W = (torch.randn((n_cb * rpc, dim), generator=g, device=cuda) * 0.05).to(torch.bfloat16)
        h = torch.randn((B, dim), generator=g, device=cuda).to(torch.bfloat16)
        out = torch.full((B, n_cb, vocab), float("nan"), dtype=torch.float32, device=cuda)
        what = f"case {case}: n_cb={n_cb} vocab={vocab} rpc={rpc} dim={dim} B={B} cap={cap}"
        z2.head_softcap(W, z2.BF16, rpc, n_cb, vocab, h, out, softcap=cap)
        torch.cuda.synchronize()
        Wk = W.float().reshape(n_cb, rpc, dim)[:, :vocab].reshape(n_cb * vocab, dim)
        ref = h.float() @ Wk.t()
        if cap > 0:
            ref = cap * torch.tanh(ref / cap)
        got = out.reshape(B, -1)
        assert torch.isfinite(got).all().item(), what
        err = (got - ref).abs().max().item()
        assert err <= 1e-3 * max(1.0, float(ref.abs().max().item()) / 15), (what, err)
    assert z2.device_error() == 0


def test_head_bf16_refuses_unsupported_shapes(z2, cuda):
    import torch
    W = torch.zeros((2 * 96, 100), dtype=torch.bfloat16, device=cuda)
    h = torch.zeros((4, 100), dtype=torch.bfloat16, device=cuda)
    out = torch.zeros((4, 2, 96), dtype=torch.float32, device=cuda)
    with pytest.raises(z2.Zonos2cuError) as e:   # vocab 96, dim 100: not multiples of 64
        z2.head_softcap(W, z2.BF16, 96, 2, 96, h, out)
    assert e.value.code == z2.EUNSUPPORTED


@pytest.mark.parametrize("n_cb,vocab,rpc,dim,B", [(1, 7, 9, 33, 3), (3, 100, 101, 64, 2),
                                                   (9, 1024, 1026, 2048, 4), (2, 513, 513, 130, 5)])
def test_head_f32_shapes(z2, oracle, cuda, n_cb, vocab, rpc, dim, B):
    import torch
    rs = np.random.default_rng(dim + vocab)
    W = rs.normal(0, 0.05, (n_cb * rpc, dim)).astype(np.float32)
    h = rs.normal(0, 1, (B, dim)).astype(np.float32)
    out = torch.full((B, n_cb, vocab), float("nan"), dtype=torch.float32, device=cuda)
    z2.head_softcap(torch.from_numpy(W).to(cuda), z2.F32, rpc, n_cb, vocab,
                    torch.from_numpy(h).to(cuda), out)
    torch.cuda.synchronize()
    ref = oracle.head_softcap(W, rpc, n_cb, vocab, h)
    got = out.cpu().numpy()
    Wr = W.reshape(n_cb, rpc, dim)[:, :vocab]
    bound = dim * 2.0 ** -24 * np.einsum("cvd,bd->bcv", np.abs(Wr), np.abs(h))
    assert (np.abs(got - ref) <= 1e-5 * np.maximum(1.0, np.abs(ref)) + bound).all()
