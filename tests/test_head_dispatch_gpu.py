"""The bf16 tcgen05 head at every tile-dispatch boundary, through the C ABI.

The dispatch picks the one-SM kernel with 64-, 128- or 256-wide N tiles or the
two-SM pair kernel by batch; each kernel has a ragged last M tile unless the
batch is a multiple of its M.  Batches on both sides of every boundary, with
and without guidance (paired rows blended after the softcap), against a torch
f32 product of the same bf16 values: the observed error is f32 summation order
only (<= 1e-3, against the stated bf16 tolerance 2e-2).  The output buffer is
longer than the batch and its tail must stay untouched (the tensor stores are
clipped at the batch's last row).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BATCHES = [63, 64, 65, 127, 129, 255, 257, 383, 384, 385, 511, 513, 767, 769, 1537]


def _weights(cuda, seed):
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    W = (torch.randn((9 * 1024, 2048), generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    return W, g


@pytest.mark.parametrize("B", BATCHES)
def test_head_bf16_dispatch_boundaries(z2, cuda, B):
    import torch
    W, g = _weights(cuda, 100 + B)
    h = torch.randn((B, 2048), generator=g, device=cuda).to(torch.bfloat16)
    buf = torch.full((B + 3, 9, 1024), float("nan"), dtype=torch.float32, device=cuda)
    z2.head_softcap(W, z2.BF16, 1024, 9, 1024, h, buf[:B])
    torch.cuda.synchronize()
    assert z2.device_error() == 0
    ref = 15 * torch.tanh((h.float() @ W.float().t()) / 15)
    got = buf[:B].reshape(B, -1)
    assert torch.isfinite(got).all().item()
    assert (got - ref).abs().max().item() <= 1e-3
    assert torch.isnan(buf[B:]).all().item(), "rows past the batch were written"


@pytest.mark.parametrize("S", [65, 129, 193, 385])
def test_head_bf16_guidance_boundaries(z2, cuda, S):
    """Guidance through the decode context: 2S hidden rows (2s conditional,
    2s+1 unconditional), S output rows u + s * (c - u) of the softcapped pair."""
    import torch
    import numpy as np
    scale = 1.7
    W, g = _weights(cuda, 7 + S)
    h = torch.randn((2 * S, 2048), generator=g, device=cuda).to(torch.bfloat16)
    Wb = W.view(torch.int16).cpu().numpy().view(np.uint16)
    ctx = z2.Context(0, S, 9, 1024, 2048, 0, seed=1)
    ctx.set_head(Wb, z2.BF16, 1024)
    ctx.set_cfg(scale)
    p = z2.SampleParams(0.8, 50, 0.95, 0.02, 1.0, 1023)
    codes = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    logits = torch.full((S, 9, 1024), float("nan"), dtype=torch.float32, device=cuda)
    ctx.step(h, z2.BF16, p, codes, logits_out=logits)
    torch.cuda.synchronize()
    assert z2.device_error() == 0
    capped = 15 * torch.tanh((h.float() @ W.float().t()) / 15)
    c, u = capped[0::2], capped[1::2]
    ref = u + scale * (c - u)
    got = logits.reshape(S, -1)
    assert torch.isfinite(got).all().item()
    assert (got - ref).abs().max().item() <= 1e-3 * (1 + 2 * scale)
    ctx.close()
