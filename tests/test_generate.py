"""Generation-loop pieces that run on the host: the codes.bin writer against the
reference's own decode_dac_to_wav, and the oracle's shear_up against an
independent formulation."""
import numpy as np
import pytest

from oracle import Reference


def test_write_codes_bin_matches_reference(tmp_path, z2):
    try:
        R = Reference()
    except Exception as e:   # the reference build is missing
        pytest.skip(str(e))
    rs = np.random.default_rng(4)
    frames = rs.integers(0, 1026, (13, 9), dtype=np.int32)
    ours = tmp_path / "ours.bin"
    z2.write_codes_bin(str(ours), frames)
    assert R.write_codes(str(tmp_path / "ref"), frames) == 1
    assert ours.read_bytes() == (tmp_path / "ref.codes.bin").read_bytes()
    empty = tmp_path / "empty.bin"
    z2.write_codes_bin(str(empty), np.zeros((0, 9), np.int32))
    assert empty.read_bytes() == np.array([0, 9], np.int32).tobytes()


@pytest.mark.parametrize("n_frames", [0, 1, 4, 9, 20])
def test_shear_up_restatement(oracle, n_frames):
    rs = np.random.default_rng(n_frames)
    codes = rs.integers(0, 1024, (n_frames, 9), dtype=np.int32)
    got = oracle.shear_up(codes, 1025)
    t = np.arange(n_frames)[:, None]
    j = np.arange(9)[None, :]
    src = t + j
    want = np.where(src < n_frames, codes[np.minimum(src, max(n_frames - 1, 0)), j]
                    if n_frames else 0, 1025)
    assert (got == want).all()
