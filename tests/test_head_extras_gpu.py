"""Output RMSNorm ahead of the head and classifier-free guidance after the
softcap, through the decode context (zonos2cu_set_out_norm / zonos2cu_set_cfg):
logits against the oracle's restatement (rms_norm_per_token, the head, the
softcap, the blend), and the sampled codes against the oracle's sampler run on
the same logits."""
import numpy as np
import pytest

from oracle import make_params

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5


def _dev(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _bf16(x):
    import workloads as W
    b = W.to_bf16_bits(x)
    return b, W.from_bf16_bits(b)


def _reference_logits(oracle, Wf, rpc, h, eps, w, cfg_scale, bf16_rows=False):
    x = oracle.out_norm(h, eps, w)
    if bf16_rows:   # the tensor-core head reads the normalised rows rounded to bf16
        x = _bf16(x)[1]
    lg = oracle.head_softcap(Wf, rpc, 9, 1024, x)
    if cfg_scale is not None:
        lg = oracle.cfg_blend(lg[0::2], lg[1::2], cfg_scale)
    return x, lg


@pytest.mark.parametrize("S,cfg", [(1, None), (2, 1.8)])
def test_out_norm_cfg_f32(z2, oracle, cuda, S, cfg):
    """f32 head (the batch-1 path), 1026 rows per codebook as in output.bin."""
    import torch
    rs = np.random.default_rng(5 + S)
    rpc, D = 1026, 2048
    Wf = rs.normal(0, 0.02, size=(9 * rpc, D)).astype(np.float32)
    gamma = rs.normal(1, 0.1, D).astype(np.float32)
    rows = S * (2 if cfg else 1)
    h = rs.normal(0, 4, (rows, D)).astype(np.float32)
    ctx = z2.Context(0, S, 9, 1024, D, 0, seed=42)
    ctx.set_head(Wf, z2.F32, rpc)
    ctx.set_out_norm(gamma, 1e-5)
    if cfg:
        ctx.set_cfg(cfg)
    p = z2.SampleParams(0.7, 50, 0.9, 0.02, 1.0, 1023)
    codes = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, 9, 1024), dtype=torch.float32, device=cuda)
    ctx.step(_dev(h, cuda), z2.F32, p, codes, logits_out=logits)
    torch.cuda.synchronize()
    x, ref = _reference_logits(oracle, Wf, rpc, h, 1e-5, gamma, cfg)
    got = logits.cpu().numpy()
    # the head's own bound: f64 dot products against the reference's f32 sums
    Wr = Wf.reshape(9, rpc, D)[:, :1024].reshape(9 * 1024, D)
    bound = D * 2.0 ** -24 * (np.abs(x) @ np.abs(Wr).T).reshape(rows, 9, 1024)
    if cfg:
        bound = bound[0::2] * abs(cfg) + bound[1::2] * abs(1 - cfg)
    assert (np.abs(got - ref) <= F32_TOL * np.maximum(1.0, np.abs(ref)) + bound + 1e-6).all()
    prm = make_params(0.7, 50, 0.9, 0.02, 1.0, 1023)
    oc, _, _ = oracle.step(got, prm, oracle.rng_seed_streams(42, S), exp_mode=1)
    assert (codes.cpu().numpy() == oc).all()
    assert z2.device_error() == 0
    ctx.close()


@pytest.mark.parametrize("S,cfg,weight", [(128, 2.0, True), (256, None, True), (512, 1.5, True),
                                          (1024, 1.25, True), (64, None, False)])
def test_out_norm_cfg_bf16(z2, oracle, cuda, S, cfg, weight):
    """bf16 tensor-core head: S=128 pairs and S=256 (256 hidden rows) on the
    one-SM kernel with 128-wide N tiles; 512 and 1024 pairs (1024 and 2048
    hidden rows) on the two-SM kernel, whose epilogue stores 16 blended output
    rows per 32-row chunk.  The bf16 head folds the norm: its weight scales W's
    columns (rounded to bf16 once) and each row's 1 / rms multiplies the row's
    dot products in the epilogue, so the logits are held to the stated bf16
    tolerance against the oracle's f32 norm and head."""
    import torch
    rs = np.random.default_rng(9 + S)
    D = 2048
    Wb, Wf = _bf16(rs.normal(0, 0.02, size=(9 * 1024, D)).astype(np.float32))
    gamma = rs.normal(1, 0.1, D).astype(np.float32) if weight else None
    rows = S * (2 if cfg else 1)
    hb, hf = _bf16(rs.normal(0, 4, (rows, D)).astype(np.float32))
    ctx = z2.Context(0, S, 9, 1024, D, 64, seed=7)
    ctx.set_head(Wb, z2.BF16, 1024)
    ctx.set_history(rs.integers(0, 1024, (S, 9, 64), dtype=np.int32), 0)
    ctx.set_out_norm(gamma, 1e-5)
    if cfg:
        ctx.set_cfg(cfg)
    p = z2.SampleParams(0.8, 50, 0.95, 0.02, 1.2, 1023)
    codes = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
    logits = torch.zeros((S, 9, 1024), dtype=torch.float32, device=cuda)
    hist = ctx.get_history()[0]
    ctx.step(_dev(hb, cuda), z2.BF16, p, codes, logits_out=logits)
    torch.cuda.synchronize()
    assert z2.device_error() == 0
    got = logits.cpu().numpy()
    pick = np.unique(np.array([0, 1, S // 2, S - 1]))
    sub = np.sort(np.concatenate([2 * pick, 2 * pick + 1])) if cfg else pick
    _, ref = _reference_logits(oracle, Wf, 1024, hf[sub], 1e-5, gamma, cfg)
    err = np.abs(got[pick] - ref).max()
    print(f"bf16 folded norm, S={S}: max |logit err| {err:.2e}")
    assert err <= 2e-2                                 # stated bf16 tolerance
    prm = make_params(0.8, 50, 0.95, 0.02, 1.2, 1023)
    oc, _, _ = oracle.step(got, prm, oracle.rng_seed_streams(7, S), hist, hist_pos=0, exp_mode=1)
    assert (codes.cpu().numpy() == oc).all()
    ctx.close()


def test_host_step_matches_device_step(z2, oracle, cuda):
    """zonos2cu_ctx_step_host with the norm and guidance on (it copies 2*S hidden
    rows) samples the same codes as the device call on the same state."""
    import torch
    rs = np.random.default_rng(31)
    S, D = 3, 2048
    Wb, _ = _bf16(rs.normal(0, 0.02, size=(9 * 1024, D)).astype(np.float32))
    gamma = rs.normal(1, 0.1, D).astype(np.float32)
    hb, _ = _bf16(rs.normal(0, 4, (2 * S, D)).astype(np.float32))
    p = z2.SampleParams(0.8, 50, 0.95, 0.02, 1.0, 1023)
    out = []
    for host in (False, True):
        ctx = z2.Context(0, S, 9, 1024, D, 0, seed=11)
        ctx.set_head(Wb, z2.BF16, 1024)
        ctx.set_out_norm(gamma, 1e-5)
        ctx.set_cfg(1.6)
        if host:
            codes = np.zeros((S, 9), np.int32)
            ctx.step_host(hb, z2.BF16, p, codes)
        else:
            c = torch.zeros((S, 9), dtype=torch.int32, device=cuda)
            ctx.step(_dev(hb, cuda), z2.BF16, p, c)
            torch.cuda.synchronize()
            codes = c.cpu().numpy()
        out.append(codes)
        ctx.close()
    assert (out[0] == out[1]).all()
