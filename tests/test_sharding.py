"""Batch sharding host logic: slice arithmetic, and a world_size-2/3 gloo run on
CPU where each rank samples its slice of a decode step (the oracle stands in
for the device sampler) and the gathered codes must equal one run over the
whole batch.  The GPU path shares the slice arithmetic and the gather."""
import os
import socket

import numpy as np
import pytest

import sharding


def test_shard_range_covers_batch():
    for n in (0, 1, 7, 64, 4097, 32768):
        for ws in (1, 2, 3, 4, 8):
            spans = [sharding.shard_range(n, ws, r) for r in range(ws)]
            assert spans[0][0] == 0
            for (f0, c0), (f1, _) in zip(spans, spans[1:]):
                assert f0 + c0 == f1
            assert sum(c for _, c in spans) == n
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
            assert max(c for _, c in spans) == sharding.max_shard(n, ws)


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharding.shard_range(8, 2, 2)
    with pytest.raises(ValueError):
        sharding.shard_range(8, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, n_streams, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (repo, os.path.join(repo, "zonos2.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import sharding as S
    import workloads as W
    from oracle import Oracle, make_params

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = W.CONFIGS[4]
        O = Oracle()
        prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
        # global state, then this rank's slice of it
        hist = W.initial_history(cfg, n_streams)[:, :, :64].copy()
        allow = W.allow_bits(cfg, n_streams)
        rng = O.rng_seed_streams(cfg.seed, n_streams)
        first, count = S.shard_range(n_streams, ws, rank)
        h_loc = hist[first:first + count].copy()
        a_loc = allow[first:first + count].copy()
        r_loc = rng[first:first + count].copy()
        steps = []
        for t in range(3):
            lg = W.step_logits(cfg, t, n_streams)[first:first + count]
            codes, _, _ = O.step(lg, prm, r_loc, h_loc, hist_pos=t % 64, allow=a_loc,
                                 delay_step=t)
            g = S.gather_codes(torch.from_numpy(codes), n_streams, ws, rank)
            steps.append(g.numpy().copy())
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), np.stack(steps))
            np.save(os.path.join(out_dir, "rng.npy"), r_loc)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws,n_streams", [(2, 64), (3, 37)])
def test_gloo_sharded_step_matches_whole_batch(tmp_path, oracle, ws, n_streams):
    import torch.multiprocessing as mp

    import workloads as W
    from oracle import make_params

    mp.start_processes(_rank_main, args=(ws, _free_port(), n_streams, str(tmp_path)),
                       nprocs=ws, start_method="spawn", join=True)
    got = np.load(tmp_path / "gathered.npy")

    cfg = W.CONFIGS[4]
    prm = make_params(cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p, cfg.penalty, W.PAD)
    hist = W.initial_history(cfg, n_streams)[:, :, :64].copy()
    allow = W.allow_bits(cfg, n_streams)
    rng = oracle.rng_seed_streams(cfg.seed, n_streams)
    for t in range(3):
        codes, _, _ = oracle.step(W.step_logits(cfg, t, n_streams), prm, rng, hist,
                                  hist_pos=t % 64, allow=allow, delay_step=t)
        np.testing.assert_array_equal(got[t], codes, err_msg=f"step {t}")
    # rank 0's generators advanced exactly as the whole batch's first slice
    f0, c0 = __import__("sharding").shard_range(n_streams, ws, 0)
    np.testing.assert_array_equal(np.load(tmp_path / "rng.npy"), rng[f0:f0 + c0])
