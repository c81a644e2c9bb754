"""The RKVA range server on a B200, end to end over TCP: a host's sequence of
HELLO, CREATE_SESSION, RANGE_CONFIG, chunked RANGE_UPLOAD, RANGE_ATTN,
RANGE_UPLOAD_ATTN and TRIM, with F16 / Q8_0 / Q4_0 rows.  Every (O, LSE)
reply equals xq_attend_range over the same rows bit for bit (the server runs
that call) and the oracle's restatement of the reference's range attention
within the north-star tolerance; the position rules answer BAD_POSITION."""
import struct

import numpy as np
import pytest
import torch

import oracle
import rkva_client as rc

pytestmark = pytest.mark.gpu

H, HKV, D, SCALE = 24, 4, 256, 1 / 16
CAP, ORIGIN = 3000, 1000


def _rows(ty, n, seed):
    rng = np.random.default_rng(seed)
    return oracle.quantize(ty, rng.normal(0, 1, (1, n, HKV, D)).astype(np.float32))[0]


def _attn_payload(positions, q):
    return (rc.U4.pack(rc.WIRE["F32"], 0, 0, 0) + np.asarray(positions, np.int32).tobytes() +
            np.ascontiguousarray(q, np.float32).tobytes())


def _decode(body, n):
    out = np.frombuffer(body[:n * H * D * 4], np.float32).reshape(n, H, D)
    lse = np.frombuffer(body[n * H * D * 4:], np.float32).reshape(n, H)
    return out, lse


def _expect(ty, k, v, q, positions, active):
    import xq
    dev = torch.device("cuda")
    o, l = xq.attend_range(ty, torch.from_numpy(np.ascontiguousarray(k[:max(active, 1)])).to(dev),
                           torch.from_numpy(np.ascontiguousarray(v[:max(active, 1)])).to(dev),
                           torch.from_numpy(q).to(dev),
                           torch.tensor(positions, dtype=torch.int32, device=dev), HKV, ORIGIN,
                           active, SCALE, split_mode=4)
    torch.cuda.synchronize()
    return o.cpu().numpy(), l.cpu().numpy()


@pytest.mark.parametrize("name,ty", [("Q8_0", oracle.Q8_0), ("F16", oracle.F16),
                                     ("Q4_0", oracle.Q4_0)])
def test_range_session_end_to_end(name, ty):
    p, port = rc.start_server()
    c = rc.Client(port)
    try:
        st, ack = c.hello(2, H, HKV, D, CAP, SCALE)
        assert st == rc.OK and ack[4] > 0          # the device's free memory
        assert c.call("CREATE_SESSION", rc.U4.pack(3, 0, CAP, 1))[0] == rc.OK
        assert c.call("RANGE_CONFIG", rc.U4.pack(ORIGIN, CAP, rc.STORAGE[name], 0),
                      session=3)[0] == rc.OK
        k0, v0 = _rows(ty, 2500, 1), _rows(ty, 2500, 2)
        wire = rc.WIRE[name]
        # layer 0: two chunks (the second appends); layer 1: one
        for lo, hi in ((0, 1500), (1500, 2500)):
            pl = rc.U4.pack(lo, hi - lo, wire, 0) + k0[lo:hi].tobytes() + v0[lo:hi].tobytes()
            assert c.call("RANGE_UPLOAD", pl, session=3, layer=0)[0] == rc.OK
        k1, v1 = _rows(ty, 716, 3), _rows(ty, 716, 4)
        pl = rc.U4.pack(0, 700, wire, 0) + k1[:700].tobytes() + v1[:700].tobytes()
        assert c.call("RANGE_UPLOAD", pl, session=3, layer=1)[0] == rc.OK
        # rule checks: a gap, a wrong encoding, a query before the end
        bad = rc.U4.pack(2600, 10, wire, 0) + k0[:10].tobytes() + v0[:10].tobytes()
        assert c.call("RANGE_UPLOAD", bad, session=3, layer=0)[0] == rc.ERR_BAD_POSITION
        bad = rc.U4.pack(0, 10, rc.WIRE["F32"], 0) + k0[:10].tobytes() + v0[:10].tobytes()
        assert c.call("RANGE_UPLOAD", bad, session=3, layer=0)[0] == rc.ERR_BAD_POSITION
        # attention: the last row, a causal limit inside the range, a query
        # before the origin (empty: O = 0, LSE = -inf)
        rng = np.random.default_rng(9)
        pos = [ORIGIN + 2499, ORIGIN + 1200, ORIGIN - 5]
        q = rng.normal(0, 1, (3, H, D)).astype(np.float32)
        st, body = c.call("RANGE_ATTN", _attn_payload(pos, q), session=3, layer=0, n_tokens=3)
        assert st == rc.OK
        out, lse = _decode(body, 3)
        eo, el = _expect(ty, k0, v0, q, pos, 2500)
        assert np.array_equal(out, eo) and np.array_equal(lse, el)
        assert np.all(out[2] == 0) and np.all(np.isneginf(lse[2]))
        ro, rl = oracle.range_attn(ty, k0, v0, q, pos, 2500, ORIGIN, H, HKV, D, SCALE)
        np.testing.assert_allclose(out, ro, rtol=1e-2, atol=2e-3)
        fin = np.isfinite(rl)
        np.testing.assert_allclose(lse[fin], rl[fin], rtol=1e-4, atol=1e-4)
        # upload + attention in one round trip: 16 new rows of layer 1, the
        # queries at its last four positions
        pos1 = [ORIGIN + 712 + i for i in range(4)]
        q1 = rng.normal(0, 1, (4, H, D)).astype(np.float32)
        pl = (rc.U4.pack(700, 16, wire, 0) + rc.U4.pack(rc.WIRE["F32"], 0, 0, 0) +
              k1[700:716].tobytes() + v1[700:716].tobytes() + np.int32(pos1).tobytes() +
              q1.tobytes())
        st, body = c.call("RANGE_UPLOAD_ATTN", pl, session=3, layer=1, n_tokens=4)
        assert st == rc.OK
        out1, lse1 = _decode(body, 4)
        eo1, el1 = _expect(ty, k1, v1, q1, pos1, 716)
        assert np.array_equal(out1, eo1) and np.array_equal(lse1, el1)
        # positions that are not the chunk's last ones
        bad = (rc.U4.pack(0, 16, wire, 0) + rc.U4.pack(rc.WIRE["F32"], 0, 0, 0) +
               k1[:16].tobytes() + v1[:16].tobytes() + np.int32([ORIGIN + 3, ORIGIN + 5]).tobytes() +
               q1[:2].tobytes())
        assert c.call("RANGE_UPLOAD_ATTN", bad, session=3, layer=1,
                      n_tokens=2)[0] == rc.ERR_BAD_POSITION
        # TRIM keeps positions < pos0: layer 0 back to 1000 rows
        assert c.call("TRIM", struct.pack("<i", ORIGIN + 1000), session=3)[0] == rc.OK
        st, body = c.call("RANGE_ATTN", _attn_payload(pos[:1], q[:1]), session=3, layer=0,
                          n_tokens=1)
        out2, lse2 = _decode(body, 1)
        eo2, el2 = _expect(ty, k0, v0, q[:1], pos[:1], 1000)
        assert st == rc.OK and np.array_equal(out2, eo2) and np.array_equal(lse2, el2)
        # RESET empties every layer
        assert c.call("RESET", session=3)[0] == rc.OK
        st, body = c.call("RANGE_ATTN", _attn_payload(pos[:1], q[:1]), session=3, layer=0,
                          n_tokens=1)
        out3, lse3 = _decode(body, 1)
        assert st == rc.OK and np.all(out3 == 0) and np.all(np.isneginf(lse3))
    finally:
        c.close()
        p.wait(timeout=60)
