"""KVarN4 oracle pinned against the reference's own float64 model.

tests/golden/kvarn4.npz holds O / LSE computed by the reference's
tests/rkva_range_kvarn4_opt_model.py (oracle_sources + oracle_attention) on
planes that oracle/kvarn4.make_plane rebuilds here from the stored seeds; the
SHA-256 of the planes guards against the builder drifting.
"""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import kvarn4 as ok

N_HEAD, N_HEAD_KV = 24, 4


def _case(g, i):
    origin, cap, tail, active, seed = (int(x) for x in g["c%d_cfg" % i])
    desc = ok.Desc(origin, cap, tail, N_HEAD_KV)
    kp = ok.make_plane(desc, active, seed)
    vp = ok.make_plane(desc, active, seed + 1000)
    return desc, active, kp, vp


@pytest.mark.parametrize("i", range(5))
def test_kvarn4_oracle_matches_reference_model(i):
    g = golden("kvarn4.npz")
    desc, active, kp, vp = _case(g, i)
    sha = hashlib.sha256(kp.tobytes() + vp.tobytes()).digest()
    assert np.array_equal(np.frombuffer(sha, np.uint8), g["c%d_sha" % i])
    out, lse = ok.attend(desc, kp, vp, active, g["c%d_q" % i], g["c%d_pos" % i], 1 / 16.0,
                         N_HEAD)
    np.testing.assert_allclose(out, g["c%d_out" % i], rtol=1e-9, atol=1e-12)
    np.testing.assert_array_equal(np.isinf(lse), np.isinf(g["c%d_lse" % i]))
    fin = np.isfinite(lse)
    np.testing.assert_allclose(lse[fin], g["c%d_lse" % i][fin], rtol=1e-9, atol=1e-12)


def test_kvarn4_wht_is_the_sylvester_matrix():
    """WHT256 as a 7-stage butterfly per 128-slice, 1/sqrt(128) per slice, then
    the (x + y, x - y) / sqrt(2) slice mix equals Sylvester H256 / 16."""
    h = ok.hadamard256()
    x = np.random.default_rng(3).normal(size=256)
    t = x.copy()
    for stride in (1, 2, 4, 8, 16, 32, 64):
        for half in (0, 128):
            seg = t[half:half + 128].copy()
            lane = np.arange(128)
            up = (lane & stride) != 0
            t[half:half + 128] = np.where(up, seg[lane ^ stride] - seg, seg + seg[lane ^ stride])
    a, b = t[:128] / np.sqrt(128), t[128:] / np.sqrt(128)
    y = np.concatenate([(a + b), (a - b)]) / np.sqrt(2)
    np.testing.assert_allclose(y, h @ x, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(h @ h, np.eye(256), atol=1e-12)
