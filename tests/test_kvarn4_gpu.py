"""B200 parity: native KVarN4 range attention through the C ABI.

Against the reference's own float64 model (tests/golden/kvarn4.npz, see
test_kvarn4_cpu.py) and against the oracle restatement (oracle/kvarn4.py) on
the edge cases: every row from the tail, records only, stage only, masked and
partial queries, other GQA widths, many splits, an empty range.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import kvarn4 as ok

pytestmark = pytest.mark.gpu


def _run(desc, kp, vp, active, q, pos, scale=1 / 16.0):
    import xq
    dev = torch.device("cuda", 0)
    out, lse = xq.attend_range_kvarn4(
        torch.from_numpy(kp).to(dev), torch.from_numpy(vp).to(dev),
        torch.from_numpy(np.ascontiguousarray(q)).to(dev),
        torch.from_numpy(np.asarray(pos, np.int32)).to(dev), desc.n_head_kv, desc.origin,
        desc.capacity, desc.tail, active, scale)
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


def _check(out, lse, ref_out, ref_lse):
    assert np.array_equal(np.isneginf(lse), np.isneginf(ref_lse))
    fin = np.isfinite(ref_lse)
    np.testing.assert_allclose(out, ref_out, rtol=1e-2, atol=2e-3)
    np.testing.assert_allclose(lse[fin], ref_lse[fin], rtol=1e-2, atol=2e-3)
    assert np.abs(out - ref_out).max() <= 1e-4 * max(np.abs(ref_out).max(), 1e-30)
    if fin.any():
        assert np.abs(lse[fin] - ref_lse[fin]).max() <= 1e-4 * np.abs(ref_lse[fin]).max()
    assert np.all(out[~fin] == 0.0)


@pytest.mark.parametrize("i", range(5))
def test_kvarn4_vs_reference_model(i):
    g = golden("kvarn4.npz")
    origin, cap, tail, active, seed = (int(x) for x in g["c%d_cfg" % i])
    desc = ok.Desc(origin, cap, tail, 4)
    kp = ok.make_plane(desc, active, seed)
    vp = ok.make_plane(desc, active, seed + 1000)
    out, lse = _run(desc, kp, vp, active, g["c%d_q" % i], g["c%d_pos" % i])
    _check(out, lse, g["c%d_out" % i], g["c%d_lse" % i])


# (origin, capacity, tail, active, n_head, n_head_kv, positions relative to origin)
CASES = [
    (0, 256, 128, 100, 24, 4, [99, 40]),          # every row from the tail
    (1280, 1024, 0, 1024, 24, 4, [1023]),         # records only
    (0, 256, 0, 127, 24, 4, [126]),               # stage only (sink group, live group)
    (384, 640, 128, 600, 16, 4, [599, -1, 250]),  # G = 4, masked and partial queries
    (0, 1024, 128, 777, 16, 2, [776, 700]),       # G = 8
    (128, 8192, 128, 8100, 24, 4, [8099]),        # many splits
    (0, 512, 128, 0, 24, 4, [5]),                 # empty range
    (0, 1024, 0, 700, 24, 4, [699, 300]),         # sink stage, records, live stage group
    (256, 768, 128, 700, 4, 4, [699, 500]),       # G = 1
    (0, 640, 128, 450, 12, 4, [449, 130]),        # G = 3, tail across the ring's end
]


@pytest.mark.parametrize("case", CASES)
def test_kvarn4_vs_oracle(case):
    origin, cap, tail, active, n_head, n_kv, rel = case
    desc = ok.Desc(origin, cap, tail, n_kv)
    seed = 500 + cap + active
    kp = ok.make_plane(desc, active, seed)
    vp = ok.make_plane(desc, active, seed + 1)
    q = np.random.default_rng(seed + 2).normal(0, 1, (len(rel), n_head, 256)).astype(np.float32)
    pos = [origin + r for r in rel]
    out, lse = _run(desc, kp, vp, active, q, pos)
    ref_out, ref_lse = ok.attend(desc, kp, vp, active, q, pos, 1 / 16.0, n_head)
    _check(out, lse, ref_out, ref_lse)


def test_kvarn4_pinned_host_buffers():
    """q, out and lse in pinned host memory (q staged by the library, out / lse
    written over PCIe by the merge) give the device-memory result bit for bit;
    pageable host memory is refused."""
    import ctypes as C
    import xq
    import xq._lib as XL
    dev = torch.device("cuda", 0)
    desc = ok.Desc(384, 640, 128, 4)
    kp = torch.from_numpy(ok.make_plane(desc, 600, 31)).to(dev)
    vp = torch.from_numpy(ok.make_plane(desc, 600, 32)).to(dev)
    q = torch.from_numpy(np.random.default_rng(33).normal(0, 1, (2, 24, 256)).astype(np.float32))
    pos = torch.tensor([384 + 599, 384 + 250], dtype=torch.int32, device=dev)
    out_d, lse_d = xq.attend_range_kvarn4(kp, vp, q.to(dev), pos, 4, 384, 640, 128, 600, 0.0625)
    q_h = q.pin_memory()
    out_h = torch.empty((2, 24, 256), dtype=torch.float32).pin_memory()
    lse_h = torch.empty((2, 24), dtype=torch.float32).pin_memory()
    xq.attend_range_kvarn4(kp, vp, q_h, pos, 4, 384, 640, 128, 600, 0.0625, out=out_h, lse=lse_h)
    torch.cuda.synchronize()
    assert torch.equal(out_h, out_d.cpu()) and torch.equal(lse_h, lse_d.cpu())
    # pageable q: refused before any launch
    L = XL.lib()
    d = XL.Kvarn4Desc(384, 640, 128, 4)
    nbytes = L.xq_attend_range_kvarn4_workspace(C.byref(d), 24, 600, 2)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    q_pageable = q.clone()
    rc = L.xq_attend_range_kvarn4(C.byref(d), kp.data_ptr(), vp.data_ptr(), 24, 600, 2,
                                  pos.data_ptr(), q_pageable.data_ptr(), 0.0625,
                                  out_d.data_ptr(), lse_d.data_ptr(), ws.data_ptr(), nbytes, None)
    assert rc == XL.XQ_ERR_INVALID and b"pageable" in L.xq_last_error()
