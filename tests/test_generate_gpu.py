"""The generation loop on the device (zonos2cu_gen_*): frames, counts and
end-of-audio frames against the oracle's restatement of the reference loop's
bookkeeping, shear_up against the oracle, and the next step's input
embeddings (embedding_sum) bit for bit."""
import numpy as np
import pytest

import oracle as O
from oracle import make_params

pytestmark = pytest.mark.gpu


def _dev(x, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_generation_rollout(z2, oracle, cuda):
    import torch
    rs = np.random.default_rng(12)
    S, Cb, V, D, F, EOA = 6, 9, 1024, 64, 5, 7
    ctx = z2.Context(0, S, Cb, V, D, 0, seed=3)
    cb_tab = rs.normal(0, 1, (Cb, 1026, D)).astype(np.float32)
    tx_tab = rs.normal(0, 1, (520, D)).astype(np.float32)
    ctx.set_embeddings(cb_tab, tx_tab)
    ctx.gen_begin(F, eoa_id=EOA, audio_pad_id=1025, text_pad_id=519)
    p = z2.SampleParams(0.7, 50, 0.9, 0.02, 1.0, 1023)
    codes = torch.zeros((S, Cb), dtype=torch.int32, device=cuda)
    frames = np.full((S, F, Cb), -1, np.int32)
    nf = np.zeros(S, np.int32)
    eos = np.full(S, -1, np.int32)
    for step in range(7):   # past max_frames
        lg = rs.normal(0, 3, (S, Cb, V)).astype(np.float32)
        lg[:, :, EOA] = -1e4                          # the end-of-audio id only where forced
        if step == 1:
            lg[2, 4, EOA] = 1e4
        if step == 3:
            lg[4, 0, EOA] = 1e4
        ctx.sample(_dev(lg, cuda), p, codes)
        torch.cuda.synchronize()
        O.gen_append(codes.cpu().numpy(), frames, nf, eos, F, codebook_size=V, eoa_id=EOA)
    got_frames, got_nf, got_eos = ctx.gen_read()
    assert (got_nf == nf).all() and (got_eos == eos).all()
    assert eos[2] == 1 and eos[4] == 3 and nf[2] == 2 and nf[4] == 4 and nf[0] == F
    assert (got_frames == frames).all()
    # shear_up of every stream
    sh = torch.zeros((S, F, Cb), dtype=torch.int32, device=cuda)
    ctx.gen_shear_up(sh)
    torch.cuda.synchronize()
    for s in range(S):
        want = np.full((F, Cb), 1025, np.int32)
        want[:nf[s]] = oracle.shear_up(frames[s, :nf[s]], 1025)
        assert (sh[s].cpu().numpy() == want).all(), s
    # the next step's input embeddings: each stream's last frame plus the text padding id
    nxt = np.concatenate([frames[np.arange(S), nf - 1], np.full((S, 1), 519, np.int32)], 1)
    emb = torch.zeros((S, D), dtype=torch.float32, device=cuda)
    ctx.gen_embed_next(emb)
    torch.cuda.synchronize()
    want = oracle.embed_frames(cb_tab, tx_tab, nxt)
    assert (emb.cpu().numpy().view(np.uint32) == want.view(np.uint32)).all()
    ctx.gen_end()
    ctx.close()


def test_embed_frames_stateless(z2, oracle, cuda):
    import torch
    rs = np.random.default_rng(13)
    D = 2048
    cb_tab = rs.normal(0, 1, (9, 1026, D)).astype(np.float32)
    tx_tab = rs.normal(0, 1, (520, D)).astype(np.float32)
    ids = np.concatenate([rs.integers(-2, 1028, (300, 9)), rs.integers(515, 522, (300, 1))],
                         1).astype(np.int32)
    out = torch.zeros((300, D), dtype=torch.float32, device=cuda)
    z2.embed_frames(_dev(cb_tab, cuda), _dev(tx_tab, cuda), _dev(ids, cuda), out)
    torch.cuda.synchronize()
    want = oracle.embed_frames(cb_tab, tx_tab, ids)
    assert (out.cpu().numpy().view(np.uint32) == want.view(np.uint32)).all()
