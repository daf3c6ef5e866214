"""Decode-context steps through the bf16 head + sampler (zonos2cu_ctx_step) at
batches past one block of 256 streams, against the oracle, through the C ABI.

Ragged batches (the last 128-row tile partly filled), the output norm folded
into the head, allow masks, delay-forced codebooks, top-k off, a penalty below
1, and a rollout over several steps:
  - the step's logits equal the standalone bf16 head's on the same operands bit
    for bit, and lie within the stated bf16 tolerance of the oracle's head;
  - codes, flags, generators and history equal the oracle's sampler on those
    logits bit for bit.
"""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _t(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("S,norm,allow,knobs", [
    (520, False, False, (0.7, 50, 0.95, 0.02, 1.2)),
    (1000, True, True, (1.0, 100, 0.9, 0.05, 1.1)),
    (768, True, False, (0.3, 0, 0.8, 0.0, 0.9)),     # top-k off, penalty < 1
])
def test_fused_step_rollout(z2, oracle, cuda, S, norm, allow, knobs):
    import torch
    import workloads as W
    T, k, tp, mp, rho = knobs
    rs = np.random.default_rng(S)
    Cb, V, D, H = 9, 1024, 2048, 64
    Wf = rs.normal(0, 0.02, size=(Cb * V, D)).astype(np.float32)
    Wb = W.to_bf16_bits(Wf)
    ctx = z2.Context(0, S, Cb, V, D, H, seed=5, first_stream=3 * S)
    ctx.set_head(Wb, z2.BF16, V)
    nw = None
    if norm:
        nw = rs.uniform(0.5, 1.5, D).astype(np.float32)
        ctx.set_out_norm(nw, 1e-5)
    hist = rs.integers(-1, V, (S, Cb, H), dtype=np.int32)
    ctx.set_history(hist, 7)
    bits = None
    if allow:
        mask = rs.random((S, V)) < 0.6
        mask[:, 1023] = True
        bits = np.packbits(mask.reshape(S, 32, 4, 8)[..., ::-1], axis=-1).reshape(
            S, 32, 4).view("<u4").reshape(S, 32).astype(np.uint32)
        ctx.set_allow(bits)
    p = z2.SampleParams(T, k, tp, mp, rho, 1023)
    prm = make_params(T, k, tp, mp, rho, 1023)
    rng = oracle.rng_seed_streams(5 + 3 * S, S)
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    flags = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, Cb, V), dtype=torch.float32, device=cuda)
    solo = torch.zeros((S, Cb, V), dtype=torch.float32, device=cuda)
    Wd = _t(Wb.view(np.int16), cuda)
    pos = 7
    for step in range(3):
        h = rs.normal(0, 1, (S, D)).astype(np.float32)
        hb = W.to_bf16_bits(h)
        delay = 1 if step == 0 else -1
        ctx.step(_t(hb.view(np.int16), cuda), z2.BF16, p, codes, flags, delay_step=delay,
                 logits_out=logits)
        torch.cuda.synchronize()
        g = logits.cpu().numpy()
        sub = np.unique(np.array([0, 1, 255, 256, S // 2, S - 1]))
        hf = W.from_bf16_bits(hb)
        if norm:
            ref = oracle.head_softcap(W.from_bf16_bits(Wb), V, Cb, V,
                                      oracle.out_norm(hf[sub], 1e-5, nw))
        else:
            ref = oracle.head_softcap(W.from_bf16_bits(Wb), V, Cb, V, hf[sub])
        assert np.abs(g[sub] - ref).max() <= BF16_TOL
        if not norm:   # the standalone head on the same operands: the same bits
            z2.head_softcap(Wd, z2.BF16, V, Cb, V, _t(hb.view(np.int16), cuda), solo)
            torch.cuda.synchronize()
            assert np.array_equal(solo.cpu().numpy(), g), step
        oc, of, _ = oracle.step(g, prm, rng, hist, hist_pos=pos, allow=bits, delay_step=delay,
                                exp_mode=1)
        gc = codes.cpu().numpy()
        bad = np.argwhere(gc != oc)
        assert len(bad) == 0, f"step {step}: {len(bad)} token mismatches, first {bad[:5].tolist()}"
        assert (flags.cpu().numpy() == of).all(), step
        assert (ctx.get_rng() == rng).all(), step
        pos = (pos + 1) % H
    hh, hp = ctx.get_history()
    assert hp == pos and (hh == hist).all()
    assert z2.device_error() == 0
    ctx.close()


def test_context_checkpoint_and_resume(z2, oracle, cuda):
    """The decode state (generators, history ring and position) read from one
    context mid-rollout and written into a fresh one: both continue with the
    same codes (and the same state) as the uninterrupted rollout."""
    import torch
    import workloads as W
    cfg = W.CONFIGS[4]
    S, Cb = 64, 9
    p = z2.SampleParams(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    a = z2.Context(0, S, Cb, 1024, 0, cfg.hist_len, seed=cfg.seed)
    a.set_history(W.initial_history(cfg, S), 0)
    a.set_allow(W.allow_bits(cfg, S))
    codes_a = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
    codes_b = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
    for step in range(3):
        a.sample(_t(W.step_logits(cfg, step, S), cuda), p, codes_a, delay_step=step)
    torch.cuda.synchronize()
    rng, (hist, pos) = a.get_rng(), a.get_history()
    b = z2.Context(0, S, Cb, 1024, 0, cfg.hist_len, seed=12345)   # another seed: overwritten
    b.set_history(hist, pos)
    b.set_rng(rng)
    b.set_allow(W.allow_bits(cfg, S))
    for step in range(3, 9):
        lg = _t(W.step_logits(cfg, step, S), cuda)
        a.sample(lg, p, codes_a, delay_step=step)
        b.sample(lg, p, codes_b, delay_step=step)
        torch.cuda.synchronize()
        assert torch.equal(codes_a, codes_b), step
    assert (a.get_rng() == b.get_rng()).all()
    ha, pa = a.get_history()
    hb, pb = b.get_history()
    assert pa == pb and (ha == hb).all()
    a.close()
    b.close()


def test_failed_allocation_is_reported_and_leaves_the_device_usable(z2, oracle, cuda):
    """A context whose history ring cannot fit (2^20 streams x 16 codebooks x
    65535 entries: 4.4 TB) is refused with ZONOS2CU_ENOMEM after the buffers it
    did get are freed; the next context on the same thread samples normally
    (the refused allocation's error is not left for the next launch to find)."""
    import torch
    with pytest.raises(z2.Zonos2cuError) as e:
        z2.Context(0, 1 << 20, 16, 1024, 0, 65535, seed=1)
    assert e.value.code == z2.ENOMEM
    S, Cb = 8, 9
    ctx = z2.Context(0, S, Cb, 1024, 0, 0, seed=3)
    lg = np.random.default_rng(3).normal(0, 3, (S, Cb, 1024)).astype(np.float32)
    codes = torch.full((S, Cb), -7, dtype=torch.int32, device=cuda)
    p = z2.SampleParams(0.7, 50, 0.9, 0.02, 1.0, 1023)
    ctx.sample(_t(lg, cuda), p, codes)
    torch.cuda.synchronize()
    rng = oracle.rng_seed_streams(3, S)
    oc, _, _ = oracle.step(lg, make_params(0.7, 50, 0.9, 0.02, 1.0, 1023), rng, None, exp_mode=1)
    assert (codes.cpu().numpy() == oc).all()
    assert (ctx.get_rng() == rng).all()
    ctx.close()
