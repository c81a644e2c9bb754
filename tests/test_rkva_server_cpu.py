"""The RKVA range server's protocol handling on CPU (no GPU visible): framing,
HELLO negotiation, session bookkeeping and the error statuses a host relies
on -- every request here is answered without touching a device, except
RANGE_CONFIG, which must fail cleanly (ERR_GPU) when no GPU is there."""
import json
import os
import struct

import pytest

import rkva_client as rc


@pytest.fixture
def server():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    p, port = rc.start_server(env)
    c = rc.Client(port)
    yield c
    c.close()
    p.wait(timeout=30)


def test_wire_struct_sizes_match_the_reference_protocol():
    assert (rc.REQ.size, rc.RSP.size, rc.HELLO.size, rc.HELLO_ACK.size, rc.U4.size) == (
        32, 56, 84, 40, 16)


def test_hello_session_and_error_statuses(server):
    c = server
    assert c.call("PING")[0] == rc.OK
    # range ops before HELLO / a session
    assert c.call("CREATE_SESSION", rc.U4.pack(1, 0, 0, 1))[0] == rc.ERR_STATE
    st, ack = c.hello(2, 24, 4, 256, 4096, 1 / 16)
    assert st == rc.OK
    ops, wire, max_sessions, _, mem, caps, _ = ack
    for op in ("HELLO", "CREATE_SESSION", "RANGE_CONFIG", "RANGE_UPLOAD", "RANGE_ATTN",
               "RANGE_UPLOAD_ATTN", "TRIM", "RESET"):
        assert ops & (1 << rc.OP[op]), op
    assert not ops & (1 << rc.OP["ATTN_DECODE"]) and not ops & (1 << rc.OP["KVARN_RANGE_CONFIG"])
    assert wire == rc.WIRE["F32"] and max_sessions == 64 and mem == 0
    assert caps & 3 == 3 and caps & (1 << 4)        # Q4_0, Q8_0 rows; upload+attention
    # geometry the server cannot take
    assert c.hello(2, 24, 5, 256, 4096, 1 / 16)[0] == rc.ERR_BAD_GEOMETRY
    assert c.hello(2, 24, 4, 96, 4096, 1 / 16)[0] == rc.ERR_BAD_GEOMETRY
    assert c.hello(2, 24, 4, 256, 4096, 1 / 16, cache_bits=4)[0] == rc.ERR_BAD_GEOMETRY
    assert c.hello(2, 24, 4, 256, 4096, 1 / 16)[0] == rc.OK
    assert c.call("CREATE_SESSION", rc.U4.pack(7, 0, 3000, 1))[0] == rc.OK
    assert c.call("CREATE_SESSION", rc.U4.pack(8, 0, 3000, 6))[0] == rc.ERR_BAD_PAYLOAD
    attn = rc.U4.pack(rc.WIRE["F32"], 0, 0, 0) + struct.pack("<i", 5) + bytes(24 * 256 * 4)
    assert c.call("RANGE_ATTN", attn, session=7, n_tokens=1)[0] == rc.ERR_BAD_SESSION
    assert c.call("RANGE_UPLOAD", rc.U4.pack(0, 1, 0, 0), session=7)[0] == rc.ERR_BAD_SESSION
    # capacity must equal the session's; origin + capacity within int32
    assert c.call("RANGE_CONFIG", rc.U4.pack(100, 2999, 0, 0), session=7)[0] == rc.ERR_BAD_POSITION
    assert c.call("RANGE_CONFIG", rc.U4.pack(100, 3000, 3, 0), session=7)[0] == rc.ERR_BAD_POSITION
    # no device here: a well-formed CONFIG fails cleanly
    assert c.call("RANGE_CONFIG", rc.U4.pack(100, 3000, 2, 0), session=7)[0] == rc.ERR_GPU
    assert c.call("RANGE_CONFIG", rc.U4.pack(100, 3000, 0, 0), session=99)[0] == rc.ERR_BAD_SESSION
    assert c.call("TRIM", struct.pack("<i", -1), session=7)[0] == rc.ERR_BAD_POSITION
    assert c.call("TRIM", struct.pack("<i", 5), session=7)[0] == rc.OK
    assert c.call("RESET", session=99)[0] == rc.ERR_BAD_SESSION
    assert c.call("ATTN_DECODE", b"", session=7)[0] == rc.ERR_UNSUPPORTED_OP
    assert c.call("RANGE_CONFIG", rc.U4.pack(100, 3000, 0, 0), session=7,
                  version=1)[0] == rc.ERR_UNSUPPORTED_OP
    st, body = c.call("GET_STATS")
    stats = json.loads(body)
    assert st == rc.OK and stats["sessions"] == 1 and stats["hello"] is True
    assert c.call("DESTROY_SESSION", session=7)[0] == rc.OK


def test_a_frame_with_a_bad_magic_closes_the_connection(server):
    c = server
    st, _ = c.call("PING", magic=0x12345678)
    assert st == rc.ERR_PROTOCOL
    with pytest.raises((ConnectionError, OSError)):
        c.call("PING")
